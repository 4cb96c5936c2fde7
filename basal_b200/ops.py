"""The torch ops of the hot path, under the reference's names where it has them, each a thin call of libbasal200.

  basal::fp8_block_gemm(q, s, w, ws, dtype)      reference op, basal/blockquant.py:151-159 (FP8 format)
  basal::int8_block_gemm(q, s, w, ws, dtype)     reference op, same, INT8 format (int8block.py:43)
  basal::nvfp4_linear(x, w, ws, alpha, inv_g)    reference op, basal/nvfp4.py:183-194
  basal::nvfp4_linear_bias(x, w, ws, alpha, inv_g, bias)
                                                 the same + bias in the epilogue (nvfp4.linear's bias, :211-212)
  basal::fp8_block_linear(x, w, ws, bias)        act_quant + GEMM (+ bias): what fp8block.linear computes
                                                 (fp8block.py:74-85); takes the place of basal::fp8_block_linear_sm90
  basal::int8_block_linear(x, w, ws, bias)       the same for INT8 (BlockFormat.linear, blockquant.py:175-183)
  basal::fp8_block_linear_glu(x, w, ws, act), basal::int8_block_linear_glu(...)
                                                 act(gate) * up of a merged [gate; up] weight in one GEMM: what
                                                 gemma4_graph.py:193-197 / gdn_graph.py:127-128 compute after the
                                                 merged gate/up linear
  basal::fp8_block_linear_residual(x, w, ws, bias, residual), basal::int8_block_linear_residual(...)
                                                 residual + linear in one GEMM: gdn_graph.py:128, :439, :466
  basal::fp8_act_quant(x), basal::int8_act_quant(x)
                                                 BlockFormat.act_quant (blockquant.py:137-144), as ops so that a
                                                 compiled layer keeps them whole
  basal::nvfp4_act_quant(x, inv_g)               nvfp4.act_quant (nvfp4.py:148-158)
  basal::nvfp4_gemm(q, s, w, ws, alpha, m, dtype)  nvfp4._mm (nvfp4.py:167-180)
  basal::code_logits(h, head, ids, bias, softcap)  CodeReadout.logits over the option rows (readout.py:71-74)
  basal::code_probs(z, idx, pad)                 CodeReadout.probs_of (readout.py:76-79)
  basal::fp8_block_gemm_glu(q, s, w, ws, act, dtype), basal::fp8_block_gemm_residual(q, s, w, ws, bias, residual)
                                                 the gated and residual linears from activation codes
  basal::rms_norm_fp8_quant(x, w, eps)           a Qwen 3.5 RMSNorm fused with the FP8 quantiser (gdn_graph.py:122-126)
  basal::gdn_prep(proj, tail, conv, A_log, dt_bias, rows, T, Hk, Hv, b_off, a_off)
                                                 the Gated DeltaNet's convolution, norms and gates (gdn_graph.py:131-140)
  basal::gdn_gate_fp8_quant(o, proj, z_off, gw, eps, rows, T)
                                                 its gated output norm fused with the FP8 quantiser (gdn_graph.py:432-438)
  basal::gdn_chunk_rule(q, k, v, g, beta, s0, o_16bit)
                                                 its gated delta rule over chunks of 64 tokens (gdn_graph.py:81-87)
  basal::attn_prep(qkv, q_norm, k_norm, eps, cos, sin, rot, H, Hk, rows, T, k_buf, v_buf, kv_off)
                                                 the attention's q / k norms and rotary embedding (gdn_graph.py:452-460)
  basal::attn_gate_fp8_quant(o, qkv, rows, T, H) its output gate fused with the FP8 quantiser (gdn_graph.py:464-466)

Every op but attn_prep is functional (mutates_args=(); attn_prep writes the keys and values into the buffers it is
given), allocates its outputs (and scratch) from the caching allocator, enqueues on
the current stream and never synchronises: Dynamo traces them through their fake kernels and a CUDA graph captures
their launches. They need CUDA tensors; there is no CPU implementation.
"""
from typing import Optional

import torch

from . import _lib
from ._lib import call, code, ptr, require_cuda

E4M3 = torch.float8_e4m3fn
Tensor = torch.Tensor


def _c(t):
    return t if t.is_contiguous() else t.contiguous()


# ---------------------------------------------------------------------------------------------------------------
# block formats
# ---------------------------------------------------------------------------------------------------------------
def _act_quant(x, integer):
    require_cuda(x)
    x = _c(x)
    M, K = x.shape
    q = torch.empty((M, K), dtype=torch.int8 if integer else E4M3, device=x.device)
    s = torch.empty((M, K // 128 if K % 128 == 0 else 0), dtype=torch.float32, device=x.device)
    name = "basal200_int8_act_quant" if integer else "basal200_fp8_act_quant"
    call(name, x.device, ptr(x), code(x.dtype), M, K, ptr(q), ptr(s))
    return q, s


@torch.library.custom_op("basal::fp8_act_quant", mutates_args=())
def fp8_act_quant(x: Tensor) -> tuple[Tensor, Tensor]:
    """[M, K] -> (e4m3 [M, K], fp32 scales [M, K / 128])."""
    return _act_quant(x, False)


@fp8_act_quant.register_fake
def _(x):
    return x.new_empty(x.shape, dtype=E4M3), x.new_empty((x.shape[0], x.shape[1] // 128), dtype=torch.float32)


@torch.library.custom_op("basal::int8_act_quant", mutates_args=())
def int8_act_quant(x: Tensor) -> tuple[Tensor, Tensor]:
    """[M, K] -> (int8 [M, K], fp32 scales [M, K / 128])."""
    return _act_quant(x, True)


@int8_act_quant.register_fake
def _(x):
    return x.new_empty(x.shape, dtype=torch.int8), x.new_empty((x.shape[0], x.shape[1] // 128), dtype=torch.float32)


def _block_gemm(q, s, w, ws, dtype, integer, bias=None):
    require_cuda(q, s, w, ws, bias)
    q, s, w, ws = _c(q), _c(s), _c(w), _c(ws)
    M, K = q.shape
    N = w.shape[0]
    c = torch.empty((M, N), dtype=dtype, device=q.device)
    if bias is not None:
        bias = _c(bias.to(dtype))
    name = "basal200_int8_block_gemm" if integer else "basal200_fp8_block_gemm"
    work = _lib.gemm_workspace(M, N, K, q.device)
    call(name, q.device, ptr(q), ptr(s), ptr(w), ptr(ws), ptr(bias), ptr(c), code(dtype), M, N, K, ptr(work),
         0 if work is None else work.numel())
    return c


@torch.library.custom_op("basal::fp8_block_gemm", mutates_args=())
def fp8_block_gemm(q: Tensor, s: Tensor, w: Tensor, ws: Tensor, dtype: torch.dtype) -> Tensor:
    """(q, s) [M, K] x (w, ws) [N, K]^T -> [M, N] in dtype (basal/blockquant.py:151-159)."""
    return _block_gemm(q, s, w, ws, dtype, False)


@fp8_block_gemm.register_fake
def _(q, s, w, ws, dtype):
    return q.new_empty((q.shape[0], w.shape[0]), dtype=dtype)


@torch.library.custom_op("basal::int8_block_gemm", mutates_args=())
def int8_block_gemm(q: Tensor, s: Tensor, w: Tensor, ws: Tensor, dtype: torch.dtype) -> Tensor:
    """The INT8 format of fp8_block_gemm (int8 codes, each 128-deep slice exact in int32)."""
    return _block_gemm(q, s, w, ws, dtype, True)


@int8_block_gemm.register_fake
def _(q, s, w, ws, dtype):
    return q.new_empty((q.shape[0], w.shape[0]), dtype=dtype)


def _block_linear(x, w, ws, bias, integer):
    require_cuda(x, w, ws, bias)
    x, w, ws = _c(x), _c(w), _c(ws)
    M, K = x.shape
    N = w.shape[0]
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    q = torch.empty((M, K), dtype=torch.uint8, device=x.device)
    s = torch.empty((M, max(K // 128, 1)), dtype=torch.float32, device=x.device)
    if bias is not None:
        bias = _c(bias.to(x.dtype))
    name = "basal200_int8_block_linear" if integer else "basal200_fp8_block_linear"
    work = _lib.gemm_workspace(M, N, K, x.device)
    call(name, x.device, ptr(x), code(x.dtype), ptr(w), ptr(ws), ptr(bias), ptr(y), M, N, K, ptr(q), ptr(s),
         ptr(work), 0 if work is None else work.numel())
    return y


@torch.library.custom_op("basal::fp8_block_linear", mutates_args=())
def fp8_block_linear(x: Tensor, w: Tensor, ws: Tensor, bias: Optional[Tensor] = None) -> Tensor:
    """x [M, K] -> [M, N] in x's dtype through an FP8-block weight: act_quant + GEMM (+ bias)."""
    return _block_linear(x, w, ws, bias, False)


@fp8_block_linear.register_fake
def _(x, w, ws, bias=None):
    return x.new_empty((x.shape[0], w.shape[0]))


_ACT = {"silu": 1, "gelu_tanh": 2}


def _block_linear_glu(x, w, ws, act, integer):
    require_cuda(x, w, ws)
    if act not in _ACT:
        raise ValueError(f"gated linear: act must be one of {sorted(_ACT)}, not {act!r}")
    x, w, ws = _c(x), _c(w), _c(ws)
    M, K = x.shape
    if w.shape[0] % 256:
        raise ValueError(f"gated linear: the merged [gate; up] weight has {w.shape[0]} rows, not a multiple of 256")
    I = w.shape[0] // 2
    y = torch.empty((M, I), dtype=x.dtype, device=x.device)
    q = torch.empty((M, K), dtype=torch.uint8, device=x.device)
    s = torch.empty((M, max(K // 128, 1)), dtype=torch.float32, device=x.device)
    name = "basal200_int8_block_linear_glu" if integer else "basal200_fp8_block_linear_glu"
    n = int(_lib.lib().basal200_block_linear_glu_workspace_bytes(M, I, K))
    work = torch.empty(n, dtype=torch.uint8, device=x.device) if n > 0 else None
    call(name, x.device, ptr(x), code(x.dtype), ptr(w), ptr(ws), ptr(y), M, I, K, _ACT[act], ptr(q), ptr(s),
         ptr(work), n)
    return y


@torch.library.custom_op("basal::fp8_block_linear_glu", mutates_args=())
def fp8_block_linear_glu(x: Tensor, w: Tensor, ws: Tensor, act: str) -> Tensor:
    """x [M, K] through a merged block-FP8 [gate; up] weight [2I, K] -> act(gate) * up [M, I] in x's dtype, one GEMM
    whose epilogue pairs the gate and up columns (act: "silu" or "gelu_tanh")."""
    return _block_linear_glu(x, w, ws, act, False)


@fp8_block_linear_glu.register_fake
def _(x, w, ws, act):
    return x.new_empty((x.shape[0], w.shape[0] // 2))


@torch.library.custom_op("basal::int8_block_linear_glu", mutates_args=())
def int8_block_linear_glu(x: Tensor, w: Tensor, ws: Tensor, act: str) -> Tensor:
    """The INT8 format of fp8_block_linear_glu."""
    return _block_linear_glu(x, w, ws, act, True)


@int8_block_linear_glu.register_fake
def _(x, w, ws, act):
    return x.new_empty((x.shape[0], w.shape[0] // 2))


def _block_linear_residual(x, w, ws, bias, residual, integer):
    require_cuda(x, w, ws, bias, residual)
    x, w, ws, residual = _c(x), _c(w), _c(ws), _c(residual)
    M, K = x.shape
    N = w.shape[0]
    if residual.shape != (M, N) or residual.dtype != x.dtype:
        raise ValueError(f"residual linear: the residual must be [{M}, {N}] {x.dtype}, not "
                         f"{list(residual.shape)} {residual.dtype}")
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    q = torch.empty((M, K), dtype=torch.uint8, device=x.device)
    s = torch.empty((M, max(K // 128, 1)), dtype=torch.float32, device=x.device)
    if bias is not None:
        bias = _c(bias.to(x.dtype))
    n = int(_lib.lib().basal200_block_linear_residual_workspace_bytes(M, N, K))
    work = torch.empty(n, dtype=torch.uint8, device=x.device) if n > 0 else None
    name = "basal200_int8_block_linear_residual" if integer else "basal200_fp8_block_linear_residual"
    call(name, x.device, ptr(x), code(x.dtype), ptr(w), ptr(ws), ptr(bias), ptr(residual), ptr(y), M, N, K, ptr(q),
         ptr(s), ptr(work), n)
    return y


@torch.library.custom_op("basal::fp8_block_linear_residual", mutates_args=())
def fp8_block_linear_residual(x: Tensor, w: Tensor, ws: Tensor, bias: Optional[Tensor], residual: Tensor) -> Tensor:
    """residual + (x [M, K] through an FP8-block weight, + bias) -> [M, N] in x's dtype, the sum in the GEMM's
    epilogue (torch's roundings: the linear's output cast, then the sum cast)."""
    return _block_linear_residual(x, w, ws, bias, residual, False)


@fp8_block_linear_residual.register_fake
def _(x, w, ws, bias, residual):
    return x.new_empty((x.shape[0], w.shape[0]))


@torch.library.custom_op("basal::int8_block_linear_residual", mutates_args=())
def int8_block_linear_residual(x: Tensor, w: Tensor, ws: Tensor, bias: Optional[Tensor], residual: Tensor) -> Tensor:
    """The INT8 format of fp8_block_linear_residual."""
    return _block_linear_residual(x, w, ws, bias, residual, True)


@int8_block_linear_residual.register_fake
def _(x, w, ws, bias, residual):
    return x.new_empty((x.shape[0], w.shape[0]))


@torch.library.custom_op("basal::int8_block_linear", mutates_args=())
def int8_block_linear(x: Tensor, w: Tensor, ws: Tensor, bias: Optional[Tensor] = None) -> Tensor:
    """x [M, K] -> [M, N] through an INT8-block weight."""
    return _block_linear(x, w, ws, bias, True)


@int8_block_linear.register_fake
def _(x, w, ws, bias=None):
    return x.new_empty((x.shape[0], w.shape[0]))


def block_quantize(w, integer):
    """Weight [N, K] -> (codes [N, K], fp32 scales [N / 128, K / 128]) on w's CUDA device (load time)."""
    require_cuda(w)
    w = _c(w if w.dtype in _lib.DTYPE_CODE else w.float())
    N, K = w.shape
    if N % 128 or K % 128:
        raise ValueError(f"block quantisation: weight {N} x {K}, both dimensions must be multiples of 128")
    q = torch.empty((N, K), dtype=torch.int8 if integer else E4M3, device=w.device)
    s = torch.empty((N // 128, K // 128), dtype=torch.float32, device=w.device)
    name = "basal200_int8_block_quantize" if integer else "basal200_fp8_block_quantize"
    call(name, w.device, ptr(w), code(w.dtype), N, K, ptr(q), ptr(s))
    return q, s


# ---------------------------------------------------------------------------------------------------------------
# NVFP4
# ---------------------------------------------------------------------------------------------------------------
@torch.library.custom_op("basal::nvfp4_act_quant", mutates_args=())
def nvfp4_act_quant(x: Tensor, inv_g: Tensor) -> tuple[Tensor, Tensor]:
    """[M, K] -> (codes [Mp, K / 2] uint8, swizzled e4m3 scales [Mp * K / 16] uint8), Mp = M rounded up to 128."""
    require_cuda(x, inv_g)
    x = _c(x)
    M, K = x.shape
    Mp = (M + 127) // 128 * 128
    q = torch.empty((Mp, K // 2), dtype=torch.uint8, device=x.device)
    s = torch.empty((Mp * (K // 16),), dtype=torch.uint8, device=x.device)
    call("basal200_nvfp4_act_quant", x.device, ptr(x), code(x.dtype), ptr(_c(inv_g.float())), M, K, ptr(q), ptr(s))
    return q, s


@nvfp4_act_quant.register_fake
def _(x, inv_g):
    M, K = x.shape
    Mp = (M + 127) // 128 * 128
    return x.new_empty((Mp, K // 2), dtype=torch.uint8), x.new_empty((Mp * (K // 16),), dtype=torch.uint8)


@torch.library.custom_op("basal::nvfp4_gemm", mutates_args=())
def nvfp4_gemm(q: Tensor, s: Tensor, w: Tensor, ws: Tensor, alpha: Tensor, m: int, dtype: torch.dtype) -> Tensor:
    """Codes q [Mp, K / 2] with swizzled scales s, weight codes w [N, K / 2] with ws -> [m, N] in dtype, times alpha."""
    require_cuda(q, s, w, ws, alpha)
    q, s, w, ws = _c(q), _c(s), _c(w), _c(ws)
    K = q.shape[1] * 2
    N = w.shape[0]
    y = torch.empty((m, N), dtype=dtype, device=q.device)
    call("basal200_nvfp4_gemm", q.device, ptr(q), ptr(s), ptr(w), ptr(ws), ptr(_c(alpha.float())), None, ptr(y),
         code(dtype), m, N, K)
    return y


@nvfp4_gemm.register_fake
def _(q, s, w, ws, alpha, m, dtype):
    return q.new_empty((m, w.shape[0]), dtype=dtype)


def _nvfp4_linear(x, w, ws, alpha, inv_g, bias):
    require_cuda(x, w, ws, alpha, inv_g, bias)
    x, w, ws = _c(x), _c(w), _c(ws)
    M, K = x.shape
    N = w.shape[0]
    Mp = (M + 127) // 128 * 128
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    q = torch.empty((max(Mp, 1), K // 2), dtype=torch.uint8, device=x.device)
    s = torch.empty((max(Mp, 1) * (K // 16),), dtype=torch.uint8, device=x.device)
    if bias is not None:
        bias = _c(bias.to(x.dtype))
    call("basal200_nvfp4_linear", x.device, ptr(x), code(x.dtype), ptr(w), ptr(ws), ptr(_c(alpha.float())),
         ptr(_c(inv_g.float())), ptr(bias), ptr(y), M, N, K, ptr(q), ptr(s))
    return y


@torch.library.custom_op("basal::nvfp4_linear", mutates_args=())
def nvfp4_linear(x: Tensor, w: Tensor, ws: Tensor, alpha: Tensor, inv_g: Tensor) -> Tensor:
    """x [M, K] -> [M, N] in x's dtype: the quantiser and the GEMM as one op (basal/nvfp4.py:183-189)."""
    return _nvfp4_linear(x, w, ws, alpha, inv_g, None)


@nvfp4_linear.register_fake
def _(x, w, ws, alpha, inv_g):
    return x.new_empty((x.shape[0], w.shape[0]))


@torch.library.custom_op("basal::nvfp4_linear_bias", mutates_args=())
def nvfp4_linear_bias(x: Tensor, w: Tensor, ws: Tensor, alpha: Tensor, inv_g: Tensor, bias: Tensor) -> Tensor:
    """nvfp4_linear + bias, the bias added in the GEMM's epilogue with torch's roundings (the output cast to x's
    dtype, the bias cast to it, the sum cast): what basal/nvfp4.py:211-212 computes after the op, in the op, so that
    a compiled layer rounds it as eager does (Inductor would otherwise fuse the bias cast into the addition)."""
    return _nvfp4_linear(x, w, ws, alpha, inv_g, bias)


@nvfp4_linear_bias.register_fake
def _(x, w, ws, alpha, inv_g, bias):
    return x.new_empty((x.shape[0], w.shape[0]))


def nvfp4_quantize(w):
    """Weight [N, K] -> (codes [N, K / 2] uint8, swizzled e4m3 scales, fp32 global scale [1]) on w's CUDA device."""
    require_cuda(w)
    w = _c(w if w.dtype in _lib.DTYPE_CODE else w.float())
    N, K = w.shape
    if K % 16:
        raise ValueError(f"NVFP4 quantisation: weight {N} x {K}, K must be a multiple of 16")
    Np, C = (N + 127) // 128 * 128, (K // 16 + 3) // 4 * 4
    codes = torch.empty((N, K // 2), dtype=torch.uint8, device=w.device)
    scales = torch.empty((Np * C,), dtype=torch.uint8, device=w.device)
    g = torch.empty((1,), dtype=torch.float32, device=w.device)
    call("basal200_nvfp4_quantize", w.device, ptr(w), code(w.dtype), N, K, ptr(codes), ptr(scales), ptr(g))
    return codes, scales.view(E4M3), g


# ---------------------------------------------------------------------------------------------------------------
# readout
# ---------------------------------------------------------------------------------------------------------------
@torch.library.custom_op("basal::code_logits", mutates_args=())
def code_logits(h: Tensor, head: Tensor, ids: Tensor, bias: Optional[Tensor] = None,
                softcap: float = 0.0) -> Tensor:
    """h [R, D] . head[ids]^T (+ bias[ids]), soft-capped -> fp32 [R, U]; the rows are read from the head by id."""
    require_cuda(h, head, ids, bias)
    if h.stride(-1) != 1:
        h = h.contiguous()
    if head.stride(-1) != 1:
        head = head.contiguous()
    ids = _c(ids.to(torch.int64))
    R, D = h.shape
    U = ids.numel()
    z = torch.empty((R, U), dtype=torch.float32, device=h.device)
    if bias is not None:
        bias = _c(bias)
    call("basal200_code_logits", h.device, ptr(h), code(h.dtype), R, D, h.stride(0), ptr(head), code(head.dtype),
         head.shape[0], head.stride(0), ptr(ids), U, ptr(bias), code(bias.dtype) if bias is not None else 0,
         float(softcap or 0.0), ptr(z))
    return z


@code_logits.register_fake
def _(h, head, ids, bias=None, softcap=0.0):
    return h.new_empty((h.shape[0], ids.numel()), dtype=torch.float32)


@torch.library.custom_op("basal::code_probs", mutates_args=())
def code_probs(z: Tensor, idx: Tensor, pad: Tensor) -> Tensor:
    """Code logits z [R, U] -> each prompt's probabilities over its codes [R, Kmax] (padding 0)."""
    require_cuda(z, idx, pad)
    z, idx = _c(z.float()), _c(idx.to(torch.int64))
    pad = _c(pad).view(torch.uint8) if pad.dtype == torch.bool else _c(pad.to(torch.uint8))  # bool: 0 / 1 bytes
    R, U = z.shape
    Kmax = idx.shape[1]
    p = torch.empty((R, Kmax), dtype=torch.float32, device=z.device)
    call("basal200_code_probs", z.device, ptr(z), R, U, ptr(idx), ptr(pad), Kmax, ptr(p))
    return p


@code_probs.register_fake
def _(z, idx, pad):
    return z.new_empty((z.shape[0], idx.shape[1]), dtype=torch.float32)


# ---------------------------------------------------------------------------------------------------------------
# the config-5 hybrid decoder's steps around its linears
# ---------------------------------------------------------------------------------------------------------------
@torch.library.custom_op("basal::fp8_block_gemm_glu", mutates_args=())
def fp8_block_gemm_glu(q: Tensor, s: Tensor, w: Tensor, ws: Tensor, act: str, dtype: torch.dtype) -> Tensor:
    """Activation codes (q, s) [M, K] through a merged block-FP8 [gate; up] weight [2I, K] -> act(gate) * up [M, I]
    in dtype (bf16 / fp16), the gate/up pairing in the GEMM's epilogue."""
    require_cuda(q, s, w, ws)
    if act not in _ACT:
        raise ValueError(f"gated linear: act must be one of {sorted(_ACT)}, not {act!r}")
    q, s, w, ws = _c(q), _c(s), _c(w), _c(ws)
    M, K = q.shape
    if w.shape[0] % 256:
        raise ValueError(f"gated linear: the merged [gate; up] weight has {w.shape[0]} rows, not a multiple of 256")
    I = w.shape[0] // 2
    y = torch.empty((M, I), dtype=dtype, device=q.device)
    n = int(_lib.lib().basal200_block_linear_glu_workspace_bytes(M, I, K))
    work = torch.empty(n, dtype=torch.uint8, device=q.device) if n > 0 else None
    call("basal200_fp8_block_gemm_glu", q.device, ptr(q), ptr(s), ptr(w), ptr(ws), ptr(y), code(dtype), M, I, K,
         _ACT[act], ptr(work), n)
    return y


@fp8_block_gemm_glu.register_fake
def _(q, s, w, ws, act, dtype):
    return q.new_empty((q.shape[0], w.shape[0] // 2), dtype=dtype)


@torch.library.custom_op("basal::fp8_block_gemm_residual", mutates_args=())
def fp8_block_gemm_residual(q: Tensor, s: Tensor, w: Tensor, ws: Tensor, bias: Optional[Tensor],
                            residual: Tensor) -> Tensor:
    """residual + (activation codes (q, s) [M, K] through an FP8-block weight, + bias) -> [M, N] in the residual's
    dtype, the sum in the GEMM's epilogue."""
    require_cuda(q, s, w, ws, bias, residual)
    q, s, w, ws, residual = _c(q), _c(s), _c(w), _c(ws), _c(residual)
    M, K = q.shape
    N = w.shape[0]
    if residual.shape != (M, N):
        raise ValueError(f"residual linear: the residual must be [{M}, {N}], not {list(residual.shape)}")
    y = torch.empty((M, N), dtype=residual.dtype, device=q.device)
    if bias is not None:
        bias = _c(bias.to(residual.dtype))
    n = int(_lib.lib().basal200_block_linear_residual_workspace_bytes(M, N, K))
    work = torch.empty(n, dtype=torch.uint8, device=q.device) if n > 0 else None
    call("basal200_fp8_block_gemm_residual", q.device, ptr(q), ptr(s), ptr(w), ptr(ws), ptr(bias), ptr(residual),
         ptr(y), code(residual.dtype), M, N, K, ptr(work), n)
    return y


@fp8_block_gemm_residual.register_fake
def _(q, s, w, ws, bias, residual):
    return residual.new_empty((q.shape[0], w.shape[0]))


@torch.library.custom_op("basal::rms_norm_fp8_quant", mutates_args=())
def rms_norm_fp8_quant(x: Tensor, w: Tensor, eps: float) -> tuple[Tensor, Tensor]:
    """Qwen3_5RMSNorm of the rows of x [M, D] (weight applied as 1 + w) -> the FP8 codes [M, D] and scales
    [M, D / 128] of the normed rows rounded to x's dtype (the normed rows are not written)."""
    require_cuda(x, w)
    x, w = _c(x), _c(w.to(x.dtype))
    M, D = x.shape
    q = torch.empty((M, D), dtype=E4M3, device=x.device)
    s = torch.empty((M, D // 128), dtype=torch.float32, device=x.device)
    call("basal200_rms_norm_fp8_quant", x.device, ptr(x), code(x.dtype), ptr(w), float(eps), M, D, None, ptr(q),
         ptr(s))
    return q, s


@rms_norm_fp8_quant.register_fake
def _(x, w, eps):
    return x.new_empty(x.shape, dtype=E4M3), x.new_empty((x.shape[0], x.shape[1] // 128), dtype=torch.float32)


@torch.library.custom_op("basal::gdn_prep", mutates_args=())
def gdn_prep(proj: Tensor, tail: Optional[Tensor], conv: Tensor, A_log: Tensor, dt_bias: Tensor, rows: int, T: int,
             Hk: int, Hv: int, b_off: int, a_off: int) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """The Gated DeltaNet's convolution (with the inputs before token 0 in tail [1 or rows, kw - 1, C]), SiLU, l2 norms
    and gates over proj [rows * T, ld] -> q, k [rows, Hk, T, 128] fp32, v [rows, Hv, T, 128] in proj's dtype (16-bit
    values already), beta, g [rows, Hv, T] fp32."""
    require_cuda(proj, tail, conv, A_log, dt_bias)
    if proj.stride(-1) != 1:
        proj = proj.contiguous()
    conv = _c(conv.to(proj.dtype))
    tail = None if tail is None else _c(tail.to(proj.dtype))
    dev = proj.device
    q = torch.empty((rows, Hk, T, 128), dtype=torch.float32, device=dev)
    k = torch.empty_like(q)
    v = torch.empty((rows, Hv, T, 128), dtype=proj.dtype, device=dev)
    beta = torch.empty((rows, Hv, T), dtype=torch.float32, device=dev)
    g = torch.empty_like(beta)
    call("basal200_gdn_prep", dev, ptr(proj), code(proj.dtype), proj.stride(0), ptr(tail),
         0 if tail is None else tail.shape[0], ptr(conv), conv.shape[1], ptr(_c(A_log.float())),
         ptr(_c(dt_bias.to(proj.dtype))), b_off, a_off, rows, T, Hk, Hv, ptr(q), ptr(k), ptr(v), ptr(beta), ptr(g))
    return q, k, v, beta, g


@gdn_prep.register_fake
def _(proj, tail, conv, A_log, dt_bias, rows, T, Hk, Hv, b_off, a_off):
    q = proj.new_empty((rows, Hk, T, 128), dtype=torch.float32)
    b = proj.new_empty((rows, Hv, T), dtype=torch.float32)
    return q, q.new_empty(q.shape), proj.new_empty((rows, Hv, T, 128)), b, b.new_empty(b.shape)


@torch.library.custom_op("basal::attn_prep", mutates_args=("k_buf", "v_buf"))
def attn_prep(qkv: Tensor, q_norm: Tensor, k_norm: Tensor, eps: float, cos: Tensor, sin: Tensor, rot: int, H: int,
              Hk: int, rows: int, T: int, k_buf: Tensor, v_buf: Tensor, kv_off: int) -> Tensor:
    """The attention layer's input steps over the merged projection qkv [rows * T, ld] (per token H heads of (128 q,
    128 gate), Hk of 128 k, Hk of 128 v): q and k RMS-normed with q_norm / k_norm, their first rot dims rotated by
    cos / sin [rows or 1, T, rot] -> q [rows, H, T, 128]; k and v written into k_buf / v_buf [rows, Hk, L, 128] at
    positions kv_off .. kv_off + T - 1."""
    require_cuda(qkv, q_norm, k_norm, cos, sin, k_buf, v_buf)
    if qkv.stride(-1) != 1:
        qkv = qkv.contiguous()
    dt = qkv.dtype
    q_norm, k_norm = _c(q_norm.to(dt)), _c(k_norm.to(dt))
    cos, sin = _c(cos.to(dt)), _c(sin.to(dt))
    if not (k_buf.is_contiguous() and v_buf.is_contiguous()):
        raise ValueError("attn_prep: the key and value buffers must be contiguous")
    q = torch.empty((rows, H, T, 128), dtype=dt, device=qkv.device)
    cs_row = 0 if cos.shape[0] == 1 else cos.stride(0)
    call("basal200_attn_prep", qkv.device, ptr(qkv), code(dt), qkv.stride(0), rows, T, H, Hk, ptr(q_norm),
         ptr(k_norm), float(eps), ptr(cos), ptr(sin), cs_row, rot, ptr(q), ptr(k_buf), ptr(v_buf), k_buf.shape[2],
         kv_off)
    return q


@attn_prep.register_fake
def _(qkv, q_norm, k_norm, eps, cos, sin, rot, H, Hk, rows, T, k_buf, v_buf, kv_off):
    return qkv.new_empty((rows, H, T, 128))


@torch.library.custom_op("basal::attn_gate_fp8_quant", mutates_args=())
def attn_gate_fp8_quant(o: Tensor, qkv: Tensor, rows: int, T: int, H: int) -> tuple[Tensor, Tensor]:
    """The attention's output o [rows, H, T, 128] times sigmoid of the gates in qkv (as for attn_prep), quantised for
    the output projection -> (e4m3 codes [rows * T, H * 128], fp32 scales [rows * T, H])."""
    require_cuda(o, qkv)
    o, qkv = _c(o), _c(qkv)
    q = torch.empty((rows * T, H * 128), dtype=E4M3, device=o.device)
    s = torch.empty((rows * T, H), dtype=torch.float32, device=o.device)
    call("basal200_attn_gate_fp8_quant", o.device, ptr(o), code(o.dtype), ptr(qkv), qkv.stride(0), rows, T, H, ptr(q),
         ptr(s))
    return q, s


@attn_gate_fp8_quant.register_fake
def _(o, qkv, rows, T, H):
    return o.new_empty((rows * T, H * 128), dtype=E4M3), o.new_empty((rows * T, H), dtype=torch.float32)


@torch.library.custom_op("basal::gdn_gate_fp8_quant", mutates_args=())
def gdn_gate_fp8_quant(o: Tensor, proj: Tensor, z_off: int, gw: Tensor, eps: float, rows: int,
                       T: int) -> tuple[Tensor, Tensor]:
    """The recurrence's output o [rows, Hv, Tp, 128] (Tp >= T; fp32, or proj's dtype) through the gated RMSNorm with
    z from proj [rows * T, ld] (columns z_off ..) -> the FP8 codes [rows * T, Hv * 128] and per-head scales
    [rows * T, Hv] of the output projection's input."""
    require_cuda(o, proj, gw)
    o = _c(o if o.dtype == proj.dtype else o.float())
    if proj.stride(-1) != 1:
        proj = proj.contiguous()
    Hv, Tp = o.shape[1], o.shape[2]
    q = torch.empty((rows * T, Hv * 128), dtype=E4M3, device=o.device)
    s = torch.empty((rows * T, Hv), dtype=torch.float32, device=o.device)
    call("basal200_gdn_gate_fp8_quant", o.device, ptr(o), code(o.dtype), Tp, ptr(proj), code(proj.dtype),
         proj.stride(0), z_off, ptr(_c(gw.to(proj.dtype))), float(eps), rows, T, Hv, None, ptr(q), ptr(s))
    return q, s


@gdn_gate_fp8_quant.register_fake
def _(o, proj, z_off, gw, eps, rows, T):
    Hv = o.shape[1]
    return o.new_empty((rows * T, Hv * 128), dtype=E4M3), o.new_empty((rows * T, Hv), dtype=torch.float32)


@torch.library.custom_op("basal::gdn_chunk_rule", mutates_args=())
def gdn_chunk_rule(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor, s0: Optional[Tensor],
                   o_16bit: bool = False) -> tuple[Tensor, Tensor]:
    """The gated delta rule (fp32) over q, k [rows, Hk, T, 128] (value head h reads key head h / (H / Hk)), v [rows, H,
    T, 128] (fp32 or 16-bit), g, beta [rows, H, T] from the state s0 [1 or rows, H, 128, 128] (None: zeros) -> (o
    [rows, H, T, 128] fp32, or in v's 16-bit dtype when o_16bit (each value rounded once), the final state
    [rows, H, 128, 128] fp32)."""
    require_cuda(q, k, v, g, beta, s0)
    q, k, g, beta = (_c(t.float()) for t in (q, k, g, beta))
    v = _c(v if v.dtype in (torch.bfloat16, torch.float16) else v.float())
    rows, Hk, T, _ = q.shape
    H = v.shape[1]
    o_dtype = v.dtype if o_16bit and v.dtype != torch.float32 else torch.float32
    o = torch.empty(v.shape, dtype=o_dtype, device=q.device)
    s = torch.empty((rows, H, 128, 128), dtype=torch.float32, device=q.device)
    if s0 is not None:
        s0 = _c(s0.float())
    call("basal200_gdn_chunk_rule", q.device, ptr(q), ptr(k), ptr(v), code(v.dtype), ptr(g), ptr(beta), ptr(s0),
         0 if s0 is None else s0.shape[0], ptr(o), code(o_dtype), ptr(s), rows, Hk, H, T)
    return o, s


@gdn_chunk_rule.register_fake
def _(q, k, v, g, beta, s0, o_16bit=False):
    rows, H = v.shape[0], v.shape[1]
    o_dtype = v.dtype if o_16bit and v.dtype != torch.float32 else torch.float32
    return q.new_empty(v.shape, dtype=o_dtype), q.new_empty((rows, H, 128, 128), dtype=torch.float32)
