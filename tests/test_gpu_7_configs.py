"""The BASELINE configurations as parity cases, at their own sizes (GPU against the oracle; tolerances of the north
star: codes and scales bit-exact, outputs within 1e-2 of each row's largest value for 16-bit outputs, the reference
tests' 2e-3 (FP8) / 1e-5 (INT8) for fp32 outputs):

  C1  the single FP8-block linear, X [512, 2048] ~ N(0, 1), W [6144, 2048] ~ N(0, 0.02), at full size
  C2  the four projections at the benchmarked packed M = 77,431 (64 requests, lengths U[128, 2048], seed 0): sampled
      rows against the oracle, the sampled rows recomputed alone bit for bit, and every row the same bits whether it
      is computed among all rows or in either half of them
  C4  the INT8-block sweep, M in {16, 128, 1024, 8192} x (N, K) in {(2048, 2048), (12288, 2048), (2048, 6144)}
  lean.linear with each parameter tuple the reference's compiled layers pass (basal/lean.py:56-93) on CUDA tensors:
      2 (F.linear), 3 (block FP8, block INT8), 5 (NVFP4), equal to the modules' own forwards
"""
import numpy as np
import pytest
import torch

from oracle import blockquant as obq

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def b2():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import basal_b200
    return basal_b200


def _u8(t):
    return t.view(torch.uint8).cpu().numpy() if t.dtype == torch.float8_e4m3fn else t.cpu().numpy()


def _row_err(got, ref):
    return (np.abs(got - ref).max(1) / np.maximum(np.abs(ref).max(1), 1e-30)).max()


def test_c1_single_fp8_linear_at_full_size(b2):
    """C1: seed 0, X [512, 2048] ~ N(0, 1) bf16, W [6144, 2048] ~ N(0, 0.02). The weight and
    activation codes and scales bit for bit, the bf16 output within 1e-2 of the oracle's linear row by row, and the
    fp32 GEMM within 2e-3 (tests/test_fp8block.py:145)."""
    g = torch.Generator().manual_seed(0)
    x = torch.randn(512, 2048, generator=g).bfloat16()
    w = torch.randn(6144, 2048, generator=g) * 0.02
    q, s = b2.fp8block.quantize(w.cuda())
    qo, so = obq.quantize(w.numpy(), "fp8")
    assert np.array_equal(_u8(q), qo) and np.array_equal(s.cpu().numpy(), so)
    qa, sa = b2.fp8block.act_quant(x.cuda())
    qao, sao = obq.act_quant(x.float().numpy(), "fp8")
    assert np.array_equal(_u8(qa), qao) and np.array_equal(sa.cpu().numpy(), sao)
    y = b2.fp8block.linear(x.cuda(), q, s).float().cpu().numpy()
    ref = obq.linear(x.float().numpy(), qo, so, "fp8")
    assert _row_err(y, ref) < 1e-2
    y32 = b2.fp8block.gemm(qa, sa, q, s, torch.float32).cpu().numpy()
    ref32 = obq.gemm(qao, sao, qo, so, "fp8")
    assert np.allclose(y32, ref32, rtol=2e-3, atol=2e-3), np.abs(y32 - ref32).max()


C2_PROJ = (("qkv", 5120, 2048), ("o", 2048, 2048), ("gate_up", 12288, 2048), ("down", 2048, 6144))


@pytest.mark.parametrize("name, N, K", C2_PROJ)
def test_c2_projections_at_the_benchmarked_rows(b2, name, N, K):
    from basal_b200.shard import varlen_lengths
    M = int(varlen_lengths(64, 128, 2048, seed=0).sum())
    assert M == 77431
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(N + K)
    x = torch.randn(M, K, device=dev, generator=g).bfloat16()
    q, s = b2.fp8block.quantize(torch.randn(N, K, device=dev, generator=g) * 0.02)
    y = b2.fp8block.linear(x, q, s)
    # every row: the same bits among all rows and in either half (a row's output does not depend on the others)
    h = M // 2
    assert torch.equal(b2.fp8block.linear(x[:h], q, s), y[:h])
    assert torch.equal(b2.fp8block.linear(x[h:], q, s), y[h:])
    # sampled rows, spread over every row tile of the persistent schedule, against the oracle
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(1))[:64].sort().values.to(dev)
    qa, sa = b2.fp8block.act_quant(x[rows])
    ref = obq.gemm(_u8(qa), sa.cpu().numpy(), _u8(q), s.cpu().numpy(), "fp8")
    assert _row_err(y[rows].float().cpu().numpy(), ref) < 1e-2
    assert torch.equal(b2.fp8block.linear(x[rows], q, s), y[rows])
    assert torch.equal(b2.fp8block.linear(x[rows[:1]], q, s), y[rows[:1]])  # one row alone: the few-rows kernel
    assert b2._lib.device_faults(0) == 0


@pytest.mark.parametrize("M", [16, 128, 1024, 8192])
@pytest.mark.parametrize("N, K", [(2048, 2048), (12288, 2048), (2048, 6144)])
def test_c4_int8_sweep(b2, M, N, K):
    """C4's INT8-block linears: the fp32 GEMM within 1e-5 of the oracle (tests/test_int8block.py:82) on sampled rows,
    the bf16 linear within 1e-2 per row, and the sampled rows recomputed alone bit for bit."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(M + N + K)
    x = torch.randn(M, K, device=dev, generator=g).bfloat16()
    q, s = b2.int8block.quantize(torch.randn(N, K, device=dev, generator=g) * 0.02)
    qa, sa = b2.int8block.act_quant(x)
    y32 = b2.int8block.gemm(qa, sa, q, s, torch.float32)
    y = b2.int8block.linear(x, q, s)
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(M))[:16].sort().values.to(dev)
    ref = obq.gemm(qa[rows].cpu().numpy(), sa[rows].cpu().numpy(), q.cpu().numpy(), s.cpu().numpy(), "int8")
    got = y32[rows].cpu().numpy()
    assert np.allclose(got, ref, rtol=1e-5, atol=1e-5), np.abs(got - ref).max()
    assert _row_err(y[rows].float().cpu().numpy(), ref) < 1e-2
    assert torch.equal(b2.int8block.linear(x[rows], q, s), y[rows])


def test_lean_linear_dispatch_on_cuda(b2):
    """lean._params / lean.linear (basal/lean.py:56-93) on CUDA tensors: the 2-tuple runs F.linear, 3-tuples the block
    FP8 and INT8 linears (by the weight's dtype), the 5-tuple the NVFP4 linear; each equals its module's forward bit for
    bit, with and without a bias, for [..., K] inputs (tests/test_int8block.py:38-39 dispatches the same way)."""
    from basal_b200 import lean
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(11)
    x = torch.randn(3, 37, 512, generator=g).bfloat16().to(dev)
    for bias in (False, True):
        lin = torch.nn.Linear(512, 384, bias=bias).to(dev)
        with torch.no_grad():
            lin.weight.copy_(torch.randn(384, 512, generator=g) * 0.02)
            if bias:
                lin.bias.copy_(torch.randn(384, generator=g) * 0.1)
        mods = [lin.bfloat16(), b2.fp8block.BlockFP8Linear.of(lin), b2.int8block.Int8BlockLinear.of(lin),
                b2.nvfp4.NVFP4Linear.of(lin, float(x.float().abs().max()))]
        for m, n in zip(mods, (2, 3, 3, 5)):
            p = lean._params(m)
            assert len(p) == n, type(m)
            got = lean.linear(x, p)
            assert got.shape == (3, 37, 384) and got.dtype == x.dtype
            assert torch.equal(got, m(x)), type(m)
        # the block tuples reach the format the weight's dtype names
        assert lean._params(mods[2])[0].dtype == torch.int8 and lean._params(mods[1])[0].dtype == torch.float8_e4m3fn
    assert b2._lib.device_faults(0) == 0
