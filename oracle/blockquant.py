"""FP8-block and INT8-block formats on the CPU in numpy -- test infrastructure only (see oracle/__init__.py).

Restates basal/blockquant.py (rkinas/basal 2.8.1):
  act_quant(x, fmt)        BlockFormat.act_quant_ops, blockquant.py:118-123 (per token, per 128 features)
  quantize(w, fmt)         BlockFormat.quantize, blockquant.py:126-135 (per 128 x 128 block)
  dequant_act / dequant_w  the two dequantisations of reference(), blockquant.py:58-59
  gemm(q, s, w, ws)        reference(), blockquant.py:54-60: both operands dequantised, one fp32 matmul
  linear(x, w, ws, fmt)    BlockFormat.linear on the CPU, blockquant.py:175-183 (act_quant + gemm + bias)

The formats: FP8 = e4m3 within +-448, saturated then cast (fp8block.py:28-30); INT8 = within +-127 rounded to the
nearest integer, ties to even (int8block.py:21, :43). Scales are amax clamped to >= 1e-12, then / qmax, in fp32.
All divisions are IEEE fp32 divisions, as torch's CPU kernels do them.
"""
import numpy as np

from .fp8 import e4m3_decode, e4m3_encode

BLOCK = 128
FORMATS = {"fp8": (448.0, False), "int8": (127.0, True)}


def _qmax(fmt):
    return np.float32(FORMATS[fmt][0]), FORMATS[fmt][1]


def _codes(v, fmt):
    qmax, rounded = _qmax(fmt)
    if rounded:
        v = np.rint(v)
    v = np.clip(v, -qmax, qmax).astype(np.float32)
    if fmt == "fp8":
        return e4m3_encode(v)
    return v.astype(np.int8)


def decode(q, fmt):
    """Codes (uint8 e4m3 bit patterns for fp8, int8 for int8) -> fp32."""
    if fmt == "fp8":
        return e4m3_decode(q)
    return np.asarray(q, np.int8).astype(np.float32)


def act_quant(x, fmt):
    """[M, K] -> (codes [M, K], fp32 scales [M, K / 128]) (blockquant.py:118-123)."""
    x = np.asarray(x, np.float32)
    M, K = x.shape
    qmax, _ = _qmax(fmt)
    b = x.reshape(M, K // BLOCK, BLOCK)
    s = np.maximum(np.abs(b).max(-1), np.float32(1e-12)) / qmax
    v = b / s[..., None]
    return _codes(v, fmt).reshape(M, K), s.astype(np.float32)


def quantize(w, fmt):
    """[N, K] -> (codes [N, K], fp32 scales [N / 128, K / 128]) (blockquant.py:126-135)."""
    w = np.asarray(w, np.float32)
    N, K = w.shape
    qmax, _ = _qmax(fmt)
    b = w.reshape(N // BLOCK, BLOCK, K // BLOCK, BLOCK)
    s = np.maximum(np.abs(b).max((1, 3)), np.float32(1e-12)) / qmax
    v = b / s[:, None, :, None]
    return _codes(v, fmt).reshape(N, K), np.ascontiguousarray(s, np.float32)


def dequant_act(q, s, fmt):
    M, K = q.shape
    return (decode(q, fmt).reshape(M, K // BLOCK, BLOCK) * s[..., None]).reshape(M, K)


def dequant_w(w, ws, fmt):
    N, K = w.shape
    return (decode(w, fmt).reshape(N // BLOCK, BLOCK, K // BLOCK, BLOCK) * ws[:, None, :, None]).reshape(N, K)


def gemm(q, s, w, ws, fmt):
    """The block GEMM's maths (blockquant.py:54-60) -> fp32 [M, N]."""
    return dequant_act(q, s, fmt) @ dequant_w(w, ws, fmt).T


def linear(x, w, ws, fmt, bias=None):
    """x [M, K] fp32 through a block-scaled weight -> fp32 [M, N] before the cast to x's dtype
    (blockquant.py:175-183, fp8block.py:74-85 on the CPU)."""
    q, s = act_quant(x, fmt)
    y = gemm(q, s, w, ws, fmt)
    if bias is not None:
        y = y + np.asarray(bias, np.float32)
    return y
