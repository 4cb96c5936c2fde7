"""The tcgen05 NVFP4 GEMM (kind::mxf4nvf4, hardware e4m3 block scales) against the oracle's dequantised maths
(the CPU branch of basal/nvfp4.py:205-210) and the reference's tests (tests/test_nvfp4.py:41-51: the linear within
0.2 of the bf16 product, part() a column slice, a row's output independent of the other rows)."""
import numpy as np
import pytest
import torch

from conftest import golden, widen_bf16
from oracle import nvfp4 as onv

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def b2():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import basal_b200
    return basal_b200


def c3_input(M, K, seed):
    """C3 activations: N(0, 1) with 1% of the values x 20."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    return torch.where(torch.rand(M, K, generator=g) < 0.01, x * 20, x).bfloat16()


@pytest.mark.parametrize("M, N, K", [(128, 128, 256), (1, 128, 64), (37, 256, 512), (300, 384, 192),
                                     (16, 2048, 2048), (1024, 2048, 6144), (129, 272, 1024)])
def test_gemm_equals_the_maths(b2, M, N, K):
    g = torch.Generator().manual_seed(M * 7 + N + K)
    w = torch.randn(N, K, generator=g) * 0.02
    x = c3_input(M, K, seed=M + K)
    codes, scales, wg = b2.nvfp4.quantize(w.cuda())
    xg = onv.global_scale(float(x.float().abs().max()))
    inv_g = torch.tensor([1.0 / xg], dtype=torch.float32)
    alpha = (wg.cpu() * xg).float()
    q, s = b2.nvfp4.act_quant(x.cuda(), inv_g.cuda())
    y = torch.ops.basal.nvfp4_gemm(q, s, codes, scales.view(torch.uint8), alpha.cuda(), M, torch.float32)
    ref = onv.linear(x.float().numpy(), codes.cpu().numpy(), scales.view(torch.uint8).cpu().numpy(),
                     float(alpha[0]), float(inv_g[0]))
    got = y.cpu().numpy()
    assert np.abs(got - ref).max() <= 1e-4 * np.abs(ref).max() + 1e-6, np.abs(got - ref).max()


def test_linear_golden_and_parts(b2):
    g = golden("nvfp4")
    x = torch.from_numpy(widen_bf16(g["x_bf16"])).bfloat16().cuda()
    torch.manual_seed(0)
    lin = torch.nn.Linear(512, 256, bias=False)
    with torch.no_grad():
        lin.weight.copy_(torch.from_numpy(g["lin_w"]))
    f = b2.nvfp4.NVFP4Linear.of(lin.cuda(), x.float().abs().amax())
    assert np.array_equal(f.weight.cpu().numpy(), g["lin_codes"])
    y = f(x).float().cpu()
    ref = torch.from_numpy(g["lin_y_bf16"])
    assert (y - ref).abs().max() / ref.abs().max() < 1e-2
    want = x.float().cpu() @ lin.weight.detach().float().cpu().t()
    assert (y - want).norm() / want.norm() < 0.2                      # tests/test_nvfp4.py:47-48
    assert torch.equal(f.part(128, 128)(x), f(x)[:, 128:])           # :49
    assert torch.equal(f(x[:1]), f(x)[:1])                            # :51


@pytest.mark.parametrize("M", [16, 128, 1024, 8192])
@pytest.mark.parametrize("N, K", [(2048, 2048), (12288, 2048), (2048, 6144)])
def test_c3_sweep_by_row_samples(b2, M, N, K):
    """The C3 sweep shapes, every M of the sweep: sampled rows against the oracle within 1e-2 of each row's largest
    output, and the sampled rows recomputed alone bit for bit."""
    g = torch.Generator().manual_seed(N + K + M)
    w = torch.randn(N, K, generator=g) * 0.02
    x = c3_input(M, K, seed=N + M)
    lin = torch.nn.Linear(K, N, bias=False)
    with torch.no_grad():
        lin.weight.copy_(w)
    f = b2.nvfp4.NVFP4Linear.of(lin.cuda(), x.float().abs().amax())
    y = f(x.cuda())
    rows = torch.randperm(M, generator=g)[:16].sort().values
    ref = onv.linear(x[rows].float().numpy(), f.weight.cpu().numpy(), f.weight_scale.view(torch.uint8).cpu().numpy(),
                     float(f.alpha.cpu()[0]), float(f.inv_g.cpu()[0]))
    ref = torch.from_numpy(ref).bfloat16().float().numpy()
    got = y[rows.cuda()].float().cpu().numpy()
    err = np.abs(got - ref).max(1) / np.abs(ref).max(1)
    assert err.max() < 1e-2, err.max()
    assert torch.equal(f(x.cuda()[rows.cuda()]), y[rows.cuda()])


@pytest.mark.parametrize("M, N", [(300, 640), (128, 272), (4096, 2064)])
def test_output_casts_and_bias(b2, M, N):
    """bf16 / fp16 outputs are the fp32 output cast; a bias in the output type is added to the cast value and rounded
    again (torch adds a bias to the cast product). Called through the C-ABI entry point, which takes the bias."""
    from basal_b200 import _lib
    K = 512
    g = torch.Generator().manual_seed(M + N)
    w = torch.randn(N, K, generator=g) * 0.02
    x = c3_input(M, K, seed=N)
    codes, scales, wg = b2.nvfp4.quantize(w.cuda())
    xg = onv.global_scale(float(x.float().abs().max()))
    inv_g = torch.tensor([1.0 / xg], dtype=torch.float32).cuda()
    alpha = (wg * xg).float().cuda()
    q, s = b2.nvfp4.act_quant(x.cuda(), inv_g)
    ws = scales.view(torch.uint8)
    y32 = torch.ops.basal.nvfp4_gemm(q, s, codes, ws, alpha, M, torch.float32)
    for dt in (torch.bfloat16, torch.float16):
        bias = (torch.randn(N, generator=g) * 0.1).to(dt).cuda()
        for b in (None, bias):
            y = torch.empty(M, N, dtype=dt, device="cuda")
            _lib.call("basal200_nvfp4_gemm", y.device, _lib.ptr(q), _lib.ptr(s), _lib.ptr(codes), _lib.ptr(ws),
                      _lib.ptr(alpha), _lib.ptr(b), _lib.ptr(y), _lib.code(dt), M, N, K)
            want = y32.to(dt)
            if b is not None:
                want = (want.float() + b.float()).to(dt)
            assert torch.equal(y, want), dt
    assert b2._lib.device_faults(0) == 0


def test_tile_widths_give_the_same_bits(b2):
    """Rows of a many-row GEMM (128 x 256 tiles) equal the same rows computed alone (128 x 128 tiles): a row's output
    does not depend on the batch around it (tests/test_nvfp4.py:51)."""
    M, N, K = 4096, 2048, 1024
    g = torch.Generator().manual_seed(5)
    w = torch.randn(N, K, generator=g) * 0.02
    x = c3_input(M, K, seed=6)
    lin = torch.nn.Linear(K, N, bias=False)
    with torch.no_grad():
        lin.weight.copy_(w)
    f = b2.nvfp4.NVFP4Linear.of(lin.cuda(), x.float().abs().amax())
    xc = x.cuda()
    y = f(xc)
    rows = torch.tensor([0, 1, 777, 4095], device="cuda")
    assert torch.equal(f(xc[rows]), y[rows])
    assert torch.equal(f(xc[:1]), y[:1])
