"""NVFP4 (e2m1 values, e4m3 scales per 16, fp32 global scale) on the CPU in numpy -- test infrastructure only
(see oracle/__init__.py).

Restates basal/nvfp4.py (rkinas/basal 2.8.1):
  swizzle / unswizzle   the 128 x 4 scale tiles of cuBLAS (nvfp4.py:49-63): scale (r, j) of R rows, C columns at
                        byte ((r // 128) * ceil(C / 4) + j // 4) * 512 + (r % 32) * 16 + (r % 128 // 32) * 4 + j % 4
  pack / unpack         two codes a byte, the even feature in the low nibble (nvfp4.py:66-72)
  act_ops(x, inv_g)     the activation quantiser's maths (nvfp4.py:106-112)
  act_quant(x, inv_g)   what the CUDA quantiser writes (nvfp4.py:148-158): codes [Mp, K/2], swizzled scales, Mp the
                        rows rounded up to 128, padding zero
  quantize(w)           the weight quantiser, 8 candidate scales by least squares (nvfp4.py:75-97)
  dequantize            nvfp4.py:100-103
  linear(x, ...)        the CPU branch of nvfp4.linear (nvfp4.py:205-210): both operands dequantised, fp32 matmul,
                        times alpha
"""
import numpy as np

from .fp8 import E2M1, e2m1_codes, e2m1_values, e4m3_decode, e4m3_encode

BLOCK = 16
FP4_MAX, E4M3_MAX = np.float32(E2M1[-1]), np.float32(448.0)
MARGIN = 2.0
CANDIDATES = tuple(1.0 - 0.04 * j for j in range(8))  # Python doubles, cast to fp32 where used (nvfp4.py:26)


def swizzle(s):
    """[rows, cols] uint8 scales -> flat uint8 in 128 x 4 tiles (rows padded to 128, cols to 4, with 0)."""
    s = np.asarray(s, np.uint8)
    r, c = s.shape
    R, C = -(-r // 128), -(-c // 4)
    p = np.zeros((R * 128, C * 4), np.uint8)
    p[:r, :c] = s
    b = p.reshape(R, 128, C, 4).transpose(0, 2, 1, 3)  # [R, C, 128, 4]
    return np.ascontiguousarray(b.reshape(-1, 4, 32, 4).transpose(0, 2, 1, 3)).reshape(-1)


def unswizzle(f, rows, cols):
    R, C = -(-rows // 128), -(-cols // 4)
    b = np.asarray(f, np.uint8).reshape(R * C, 32, 4, 4).transpose(0, 2, 1, 3).reshape(R, C, 128, 4)
    return np.ascontiguousarray(b.transpose(0, 2, 1, 3).reshape(R * 128, C * 4)[:rows, :cols])


def pack(c):
    c = np.asarray(c, np.uint8)
    return (c[:, 0::2] | (c[:, 1::2] << 4)).astype(np.uint8)


def unpack(p):
    p = np.asarray(p, np.uint8)
    return np.stack([p & 15, p >> 4], -1).reshape(p.shape[0], -1)


def _scale_of(amax_over_6):
    """min(., 448) cast to e4m3 -> (bits, fp32 value)."""
    bits = e4m3_encode(np.minimum(amax_over_6, E4M3_MAX))
    return bits, e4m3_decode(bits)


def act_ops(x, inv_g):
    """[M, K] -> (packed codes [M, K/2] uint8, e4m3 scale bits [M, K/16] uint8, not swizzled) (nvfp4.py:106-112)."""
    x = np.asarray(x, np.float32)
    M, K = x.shape
    b = x.reshape(M, K // BLOCK, BLOCK) * np.float32(inv_g)
    bits, s = _scale_of(np.abs(b).max(-1, keepdims=True) / FP4_MAX)
    with np.errstate(divide="ignore", invalid="ignore"):
        u = np.where(s > 0, b / s, np.float32(0.0))
    return pack(e2m1_codes(u).reshape(M, K)), bits[..., 0]


def act_quant(x, inv_g):
    """[M, K] -> (codes [Mp, K/2], swizzled scales [Mp * K/16]) as the CUDA quantiser writes them (nvfp4.py:148-158)."""
    M, K = np.asarray(x).shape
    Mp = -(-M // 128) * 128
    codes, bits = act_ops(x, inv_g)
    q = np.zeros((Mp, K // 2), np.uint8)
    q[:M] = codes
    s = np.zeros((Mp, K // BLOCK), np.uint8)
    s[:M] = bits
    return q, swizzle(s)


def sum16(d):
    """fp32 sum over the last axis (16 values, keepdims) in the order torch's CPU sum kernel takes for a contiguous
    run of 16 floats: eight lane sums p_k = d_k + d_(k+8), then 0 + p_0 + ... + p_7 in sequence (checked against
    torch 2.11 on 2^18 random rows, no mismatch; the order decides ties between candidate scales in quantize)."""
    p = d[..., 0:8] + d[..., 8:16]
    e = np.zeros(d.shape[:-1] + (1,), np.float32)
    for k in range(8):
        e = e + p[..., k:k + 1]
    return e


def quantize(w, rows=4096):
    """[N, K] -> (codes [N, K/2] uint8, swizzled e4m3 scale bits, fp32 global scale [1]) (nvfp4.py:75-97).
    The squared error of a block (nvfp4.py:89) is summed as torch's CPU kernel sums it (sum16)."""
    w = np.asarray(w, np.float32)
    N, K = w.shape
    g = np.maximum(np.abs(w).max() / np.float32(FP4_MAX * E4M3_MAX), np.float32(1e-12)).astype(np.float32)
    codes, scales = [], []
    for o in range(0, N, rows):
        b = w[o: o + rows].reshape(-1, K // BLOCK, BLOCK) / g
        amax = np.abs(b).max(-1, keepdims=True)
        best = err = sc = None
        for f in CANDIDATES:
            bits, s = _scale_of(amax * np.float32(f) / FP4_MAX)
            with np.errstate(divide="ignore", invalid="ignore"):
                u = np.where(s > 0, b / s, np.float32(0.0))
            c = e2m1_codes(u)
            d = (e2m1_values(c) * s - b) ** 2
            e = sum16(d)
            if best is None:
                best, err, sc = c, e, bits
            else:
                m = e < err
                best, err, sc = np.where(m, c, best), np.where(m, e, err), np.where(m, bits, sc)
        codes.append(pack(best.reshape(best.shape[0], K)))
        scales.append(sc[..., 0])
    return np.concatenate(codes), swizzle(np.concatenate(scales)), np.asarray([g], np.float32)


def dequantize(codes, scales, g, N, K):
    s = e4m3_decode(unswizzle(scales, N, K // BLOCK))
    return (e2m1_values(unpack(codes)).reshape(N, K // BLOCK, BLOCK) * s[..., None]).reshape(N, K) * np.float32(g)


def linear(x, w, ws, alpha, inv_g, bias=None):
    """The CPU branch of nvfp4.linear (nvfp4.py:205-210) -> fp32 [M, N] before the cast to x's dtype."""
    x = np.asarray(x, np.float32)
    M, K = x.shape
    N = w.shape[0]
    qc, sc = act_ops(x, inv_g)
    xd = (e2m1_values(unpack(qc)).reshape(M, K // BLOCK, BLOCK) * e4m3_decode(sc)[..., None]).reshape(M, K)
    wd = (e2m1_values(unpack(w)).reshape(N, K // BLOCK, BLOCK)
          * e4m3_decode(unswizzle(ws, N, K // BLOCK))[..., None]).reshape(N, K)
    y = (xd @ wd.T) * np.float32(alpha)
    if bias is not None:
        y = y + np.asarray(bias, np.float32)
    return y


def global_scale(amax):
    """The activation global scale of NVFP4Linear.of (nvfp4.py:234): max(amax, 1e-6) * 2 / (6 * 448)."""
    return np.float32(max(float(amax), 1e-6) * MARGIN / (6.0 * 448.0))
