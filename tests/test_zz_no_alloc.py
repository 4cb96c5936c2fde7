"""basal200_fp8_block_linear_noalloc, the FP8-block linear for callers that cannot allocate device memory (a runtime
that plans all device memory up front, a host language without a device allocator of its own, a caller that must not
let cudaMalloc synchronise the device mid-request): called through the C ABI and compared with the allocating entry
point basal200_fp8_block_linear on the same inputs, for two calls in a row (the second call finds the first call's
codes in the library's shared array), on the large-M kernel and on the few-rows kernel (M = 16). Its size limit is
checked without a GPU in test_capi.py (the refusal comes before any device call). Collected last on purpose: it
needs nothing from the other test files and runs the same alone in a fresh process."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

BF16 = 0
MAX_ELEMS = 1 << 24  # BASAL200_NOALLOC_MAX_ELEMS of include/basal200.h


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from basal_b200 import _lib
    return _lib.lib()


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _p(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _weight(N, K, seed):
    import basal_b200
    g = torch.Generator(device="cuda").manual_seed(seed)
    return basal_b200.fp8block.quantize(torch.randn(N, K, device="cuda", generator=g) * 0.02)


def _allocating(lib, x, w, ws, bias, M, N, K):
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    q = torch.empty(M, K, dtype=torch.uint8, device="cuda")
    s = torch.empty(M, K // 128, dtype=torch.float32, device="cuda")
    rc = lib.basal200_fp8_block_linear(_p(x), BF16, _p(w), _p(ws), _p(bias), _p(y), M, N, K, _p(q), _p(s), None, 0,
                                       _stream())
    assert rc == 0
    return y


def _noalloc(lib, x, w, ws, bias, M, N, K):
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    rc = lib.basal200_fp8_block_linear_noalloc(_p(x), BF16, _p(w), _p(ws), _p(bias), _p(y), M, N, K, _stream())
    assert rc == 0
    return y


def test_noalloc_matches_the_allocating_linear_on_two_calls_in_a_row(lib):
    torch.manual_seed(0)
    cases = [(1000, 768, 1024, None), (4096, 2048, 4096, torch.randn(2048, device="cuda").bfloat16()),
             (16, 2048, 2048, None), (16, 1280, 6144, torch.randn(1280, device="cuda").bfloat16())]
    for i, (M, N, K, bias) in enumerate(cases):
        x = torch.randn(M, K, device="cuda").bfloat16()
        w, ws = _weight(N, K, seed=i)
        want = _allocating(lib, x, w, ws, bias, M, N, K)
        got = _noalloc(lib, x, w, ws, bias, M, N, K)
        torch.cuda.synchronize()
        err = (got.float() - want.float()).abs().max() / want.float().abs().max()
        assert err <= 1e-2, err  # the north-star tolerance of the other GEMM tests
        assert torch.equal(got, want)  # the same two kernels on the same inputs: the same bits


def test_noalloc_runs_at_the_small_end_and_at_its_limit(lib):
    """One row, and exactly BASAL200_NOALLOC_MAX_ELEMS activation values (M * K at the limit), both within bounds."""
    w, ws = _weight(256, 2048, seed=3)
    x = torch.randn(1, 2048, device="cuda").bfloat16()
    assert torch.equal(_noalloc(lib, x, w, ws, None, 1, 256, 2048), _allocating(lib, x, w, ws, None, 1, 256, 2048))
    M = MAX_ELEMS // 2048
    x = torch.randn(M, 2048, device="cuda").bfloat16()
    got = _noalloc(lib, x, w, ws, None, M, 256, 2048)
    assert torch.equal(got, _allocating(lib, x, w, ws, None, M, 256, 2048))
