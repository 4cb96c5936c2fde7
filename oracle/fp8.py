"""e4m3 (float8_e4m3fn) and e2m1 codecs in numpy -- test infrastructure only (see oracle/__init__.py).

e4m3fn: 1 sign, 4 exponent (bias 7), 3 mantissa bits; no infinities; 0x7f / 0xff are NaN; largest finite 448.
The encoder restates the rounding of torch's fp32 -> float8_e4m3fn cast, which the reference applies in
basal/blockquant.py:123, :134 and basal/nvfp4.py:86, :110: round to nearest, ties to even, for normal and subnormal
results; |x| >= 480 (the first value past 448 after rounding), inf and NaN give NaN (0x7f with the sign).

e2m1: the table basal/nvfp4.py:19 (code k in 0..7 has magnitude E2M1[k], bit 3 the sign) and the cuts of
basal/nvfp4.py:22 (midpoints; a tie goes to the even code: '>' above an even code, '>=' above an odd one).
"""
import numpy as np

E4M3_MAX = 448.0
E2M1 = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
CUTS = tuple(((a + b) / 2, k % 2 == 1) for k, (a, b) in enumerate(zip(E2M1, E2M1[1:])))


def _e4m3_table():
    v = np.zeros(256, np.float32)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e, m = (b >> 3) & 0xF, b & 7
        if e == 0xF and m == 7:
            v[b] = np.nan
        elif e == 0:
            v[b] = s * m * 2.0 ** -9
        else:
            v[b] = s * (1 + m / 8) * 2.0 ** (e - 7)
    return v


E4M3_VALUES = _e4m3_table()


def e4m3_encode(x):
    """fp32 array -> uint8 e4m3fn bit patterns (round to nearest even; >= 480, inf, NaN -> NaN)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    sign = ((x.view(np.uint32) >> 24) & 0x80).astype(np.uint8)
    a = np.abs(x)
    out = np.empty(x.shape, np.uint8)
    nan = ~(a < 480.0)
    sub = a < np.float32(2.0 ** -6)
    # subnormal range: multiples of 2^-9, the scaling by 512 is exact, np.rint rounds half to even
    q_sub = np.rint(a * np.float32(512.0))
    # normal range: a = m * 2^e, m in [0.5, 1); mantissa (2m - 1) * 8 is exact in fp32 before rounding
    m, e = np.frexp(np.where(sub | nan, np.float32(1.0), a))
    mant = np.rint((m.astype(np.float32) * np.float32(2.0) - np.float32(1.0)) * np.float32(8.0))
    exp = e.astype(np.int64) - 1 + 7
    carry = mant >= 8
    mant = np.where(carry, 0, mant)
    exp = np.where(carry, exp + 1, exp)
    q_norm = (exp << 3) | mant.astype(np.int64)
    q_norm = np.minimum(q_norm, 0x7F)  # the (464, 480) band rounds to the NaN pattern, as the cast does
    out[...] = np.where(sub, q_sub, q_norm).astype(np.uint8)
    out[nan] = 0x7F
    return out | sign


def e4m3_decode(b):
    """uint8 e4m3fn bit patterns -> fp32 values."""
    return E4M3_VALUES[np.asarray(b, np.uint8)]


def e2m1_codes(u):
    """fp32 values in units of their block scale -> e2m1 codes (uint8, bit 3 the sign), nearest, ties to even
    (basal/nvfp4.py:36-41). The sign bit is set for every u < 0, also when the magnitude rounds to 0."""
    u = np.asarray(u, np.float32)
    a = np.abs(u)
    c = np.zeros(u.shape, np.int32)
    for t, odd in CUTS:
        c += (a >= np.float32(t)) if odd else (a > np.float32(t))
    return (c | ((u < 0).astype(np.int32) << 3)).astype(np.uint8)


def e2m1_values(c):
    """e2m1 codes -> fp32 values (basal/nvfp4.py:44-46)."""
    c = np.asarray(c, np.uint8)
    v = np.asarray(E2M1, np.float32)[c & 7]
    return np.where(c >= 8, -v, v).astype(np.float32)
