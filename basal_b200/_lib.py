"""ctypes binding of libbasal200.so, the C ABI of include/basal200.h.

The library is the only compute path of basal_b200: when it is missing, importing this module's `lib()` raises
ImportError (there is no CPU or PyTorch fallback). Every call passes raw device pointers and the current CUDA stream
of the tensors' device, and maps a non-zero status to ValueError (arguments, shapes, alignment, dtypes, limits) or
RuntimeError (architecture, launch, TMA descriptor).
"""
import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libbasal200.so")

BF16, F16, F32 = 0, 1, 2
DTYPE_CODE = {torch.bfloat16: BF16, torch.float16: F16, torch.float32: F32}

OK, ERR_ARG, ERR_SHAPE, ERR_ALIGN, ERR_DTYPE, ERR_ARCH, ERR_LAUNCH, ERR_TMAP, ERR_LIMIT = range(9)
_VALUE_ERRORS = {ERR_ARG, ERR_SHAPE, ERR_ALIGN, ERR_DTYPE, ERR_LIMIT}

_P, _I64, _I, _F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float

# name -> argument types (every entry point returns int, except the diagnostics below)
SIGNATURES = {
    "basal200_fp8_act_quant": [_P, _I, _I64, _I64, _P, _P, _P],
    "basal200_int8_act_quant": [_P, _I, _I64, _I64, _P, _P, _P],
    "basal200_fp8_block_quantize": [_P, _I, _I64, _I64, _P, _P, _P],
    "basal200_int8_block_quantize": [_P, _I, _I64, _I64, _P, _P, _P],
    "basal200_fp8_block_gemm": [_P, _P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _P, _I64, _P],
    "basal200_fp8_block_gemm_gather": [_P, _P, _P, _P, _P, _I, _I64, _I64, _I, _I64, _I64, _I64, _P, _P],
    "basal200_peer_barrier": [_P, _I, _I, _I64, _P],
    "basal200_int8_block_gemm": [_P, _P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _P, _I64, _P],
    "basal200_fp8_block_linear": [_P, _I, _P, _P, _P, _P, _I64, _I64, _I64, _P, _P, _P, _I64, _P],
    "basal200_int8_block_linear": [_P, _I, _P, _P, _P, _P, _I64, _I64, _I64, _P, _P, _P, _I64, _P],
    "basal200_fp8_block_linear_noalloc": [_P, _I, _P, _P, _P, _P, _I64, _I64, _I64, _P],
    "basal200_fp8_block_linear_glu": [_P, _I, _P, _P, _P, _I64, _I64, _I64, _I, _P, _P, _P, _I64, _P],
    "basal200_int8_block_linear_glu": [_P, _I, _P, _P, _P, _I64, _I64, _I64, _I, _P, _P, _P, _I64, _P],
    "basal200_fp8_block_linear_residual": [_P, _I, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P, _P, _P, _I64, _P],
    "basal200_int8_block_linear_residual": [_P, _I, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P, _P, _P, _I64, _P],
    "basal200_nvfp4_act_quant": [_P, _I, _P, _I64, _I64, _P, _P, _P],
    "basal200_nvfp4_gemm": [_P, _P, _P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _P],
    "basal200_nvfp4_linear": [_P, _I, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P, _P, _P],
    "basal200_nvfp4_quantize": [_P, _I, _I64, _I64, _P, _P, _P, _P],
    "basal200_attn_prep": [_P, _I, _I64, _I, _I, _I, _I, _P, _P, _F, _P, _P, _I64, _I, _P, _P, _P, _I64, _I64, _P],
    "basal200_attn_gate_fp8_quant": [_P, _I, _P, _I64, _I, _I, _I, _P, _P, _P],
    "basal200_code_logits": [_P, _I, _I64, _I64, _I64, _P, _I, _I64, _I64, _P, _I64, _P, _I, _F, _P, _P],
    "basal200_code_probs": [_P, _I64, _I64, _P, _P, _I64, _P, _P],
    "basal200_fp8_block_gemm_glu": [_P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I, _P, _I64, _P],
    "basal200_fp8_block_gemm_residual": [_P, _P, _P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _P, _I64, _P],
    "basal200_rms_norm_fp8_quant": [_P, _I, _P, _F, _I64, _I64, _P, _P, _P, _P],
    "basal200_gdn_prep": [_P, _I, _I64, _P, _I, _P, _I, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P],
    "basal200_gdn_gate_fp8_quant": [_P, _I, _I, _P, _I, _I64, _I, _P, _F, _I, _I, _I, _P, _P, _P, _P],
    "basal200_gdn_chunk_rule": [_P, _P, _P, _I, _P, _P, _P, _I, _P, _I, _P, _I, _I, _I, _I, _P],
}

_lib = None


def lib():
    """The loaded library (loaded once); ImportError when it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python basal_b200/build.py` (nvcc, sm_100a). "
                              "basal_b200 has no CPU or fallback path.")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            f = getattr(L, name)
            f.argtypes, f.restype = args, ctypes.c_int
        L.basal200_status_string.argtypes, L.basal200_status_string.restype = [_I], ctypes.c_char_p
        L.basal200_version.argtypes, L.basal200_version.restype = [], _I
        L.basal200_block_gemm_workspace_bytes.argtypes = [_I64, _I64, _I64]
        L.basal200_block_gemm_workspace_bytes.restype = _I64
        L.basal200_block_linear_glu_workspace_bytes.argtypes = [_I64, _I64, _I64]
        L.basal200_block_linear_glu_workspace_bytes.restype = _I64
        L.basal200_block_linear_residual_workspace_bytes.argtypes = [_I64, _I64, _I64]
        L.basal200_block_linear_residual_workspace_bytes.restype = _I64
        L.basal200_device_faults.argtypes, L.basal200_device_faults.restype = [_I, _I], ctypes.c_uint
        _lib = L
    return _lib


def ptr(t):
    return None if t is None else t.data_ptr()


def code(dtype):
    try:
        return DTYPE_CODE[dtype]
    except KeyError:
        raise ValueError(f"basal_b200: dtype {dtype} is not supported (bfloat16, float16, float32)") from None


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("basal_b200 computes on CUDA tensors only (sm_100a); the CPU maths of the reference "
                             "is not part of this package")


def call(name, device, *args):
    """Calls entry point `name` with `args` and the current stream of `device` appended; raises on a bad status."""
    L = lib()
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        rc = getattr(L, name)(*args, stream)
    if rc != OK:
        msg = f"{name}: {L.basal200_status_string(rc).decode()} (status {rc})"
        raise (ValueError if rc in _VALUE_ERRORS else RuntimeError)(msg)


def gemm_workspace(M, N, K, device):
    """A workspace tensor for the block GEMM of (M, N, K), or None when the shape takes none (ptr(None) is NULL)."""
    n = int(lib().basal200_block_gemm_workspace_bytes(int(M), int(N), int(K)))
    return torch.empty(n, dtype=torch.uint8, device=device) if n > 0 else None


def device_faults(device=0, clear=True):
    """Fault bits of bounded waits that gave up on `device` (0: none). Synchronises the device."""
    return int(lib().basal200_device_faults(int(device), int(bool(clear))))
