"""The CUDA quantisers against the oracle and the reference's golden outputs, bit for bit: FP8 / INT8 activations
(basal/blockquant.py:118-124) and weights (:126-135), NVFP4 activations with their swizzled scales
(basal/nvfp4.py:106-158) and NVFP4 weights with the 8-candidate search (nvfp4.py:75-97)."""
import numpy as np
import pytest
import torch

from conftest import golden, widen_bf16
from oracle import blockquant as obq
from oracle import nvfp4 as onv

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def b2():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import basal_b200
    return basal_b200


def u8(t):
    return t.contiguous().view(torch.uint8).cpu().numpy()


def f32bits(t):
    return t.float().cpu().numpy().view(np.uint32)


def heavy(M, K, seed, dtype=torch.bfloat16):
    """N(0, 1) with 1% of the values x 20, plus a zero group, a tiny group and exact ties."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    x = torch.where(torch.rand(M, K, generator=g) < 0.01, x * 20, x)
    if M > 3 and K >= 256:
        x[1, :128] = 0.0
        x[2, 128:256] *= 1e-20
        x[3, :8] = torch.tensor([448.0, 1.5, 2.5, -3.5, 0.5, 104.0, 232.0, -240.0])
    return x.to(dtype)


def fmt_mod(b2, fmt):
    return b2.fp8block if fmt == "fp8" else b2.int8block


@pytest.mark.parametrize("fmt", ["fp8", "int8"])
def test_act_quant_golden(b2, fmt):
    g = golden("blockquant")
    mod = fmt_mod(b2, fmt)
    x = torch.from_numpy(widen_bf16(g["x_bf16"])).cuda().bfloat16()
    q, s = mod.act_quant(x)
    assert q.dtype == mod.FORMAT.dtype and s.shape == (64, 8)
    assert np.array_equal(u8(q), g[f"{fmt}_act_q"])
    assert np.array_equal(f32bits(s), g[f"{fmt}_act_s"].view(np.uint32))
    q, s = mod.act_quant(torch.from_numpy(g["xf"]).cuda())  # fp32 activations
    assert np.array_equal(u8(q), g[f"{fmt}_actf_q"])
    assert np.array_equal(f32bits(s), g[f"{fmt}_actf_s"].view(np.uint32))


@pytest.mark.parametrize("fmt", ["fp8", "int8"])
@pytest.mark.parametrize("M, K, dtype", [(1, 128, torch.bfloat16), (37, 1024, torch.bfloat16),
                                         (1000, 2048, torch.bfloat16), (4099, 6144, torch.bfloat16),
                                         (77, 512, torch.float16), (65, 384, torch.float32),
                                         (9500, 2048, torch.float32), (10007, 2048, torch.float16)])
def test_act_quant_bit_exact(b2, fmt, M, K, dtype):
    x = heavy(M, K, seed=M + K, dtype=dtype)
    q, s = fmt_mod(b2, fmt).act_quant(x.cuda())
    qo, so = obq.act_quant(x.float().numpy(), fmt)
    assert np.array_equal(u8(q), qo.view(np.uint8))
    assert np.array_equal(f32bits(s), so.view(np.uint32))


def e4m3_boundary_rows(rows, seed):
    """fp32 activations whose quotients x / s land on and within 3 fp32 ulps of every e4m3 rounding midpoint (normal
    and subnormal, both signs), each 1 x 128 group led by its amax so that s = amax / 448 is known."""
    rng = np.random.default_rng(seed)
    mids = [2.0 ** e * (1 + (2 * m + 1) / 16) for e in range(-6, 9) for m in range(8)]
    mids += [(2 * m + 1) * 2.0 ** -10 for m in range(8)]  # subnormal midpoints, and the one below 2^-6
    mids = np.array([v for v in mids if v < 448], dtype=np.float32)
    G = rows * 8
    amax = (rng.uniform(0.5, 8.0, G) * 2.0 ** rng.integers(-6, 7, G)).astype(np.float32)
    s = (amax / np.float32(448)).astype(np.float32)
    t = (rng.choice(mids, (G, 127)) * s[:, None]).astype(np.float32)
    t = (t.view(np.int32) + rng.integers(-3, 4, (G, 127)).astype(np.int32)).view(np.float32)
    t = t * np.where(rng.random((G, 127)) < 0.5, -1, 1).astype(np.float32)
    t = np.clip(t, -amax[:, None], amax[:, None])
    return np.concatenate([amax[:, None], t], axis=1).reshape(rows, 1024)


@pytest.mark.parametrize("rows", [64, 19000])  # 512 groups (the few-groups kernel), 152000 (the wide kernel)
def test_act_quant_fp8_code_boundaries(b2, rows):
    """Codes of quotients at and beside the e4m3 rounding midpoints: the quantiser's bounding products leave these open
    and its exact division settles them; every code and scale equals the oracle's."""
    x = e4m3_boundary_rows(rows, seed=5)
    q, s = b2.fp8block.act_quant(torch.from_numpy(x).cuda())
    qo, so = obq.act_quant(x, "fp8")
    assert np.array_equal(u8(q), qo.view(np.uint8))
    assert np.array_equal(f32bits(s), so.view(np.uint32))


def test_act_quant_empty_and_refusals(b2):
    q, s = b2.fp8block.act_quant(torch.empty(0, 256, device="cuda", dtype=torch.bfloat16))
    assert q.shape == (0, 256) and s.shape == (0, 2)
    with pytest.raises(ValueError):
        b2.fp8block.act_quant(torch.zeros(4, 200, device="cuda", dtype=torch.bfloat16))


@pytest.mark.parametrize("fmt", ["fp8", "int8"])
def test_weight_quantize_golden(b2, fmt):
    g = golden("blockquant")
    mod = fmt_mod(b2, fmt)
    q, s = mod.quantize(torch.from_numpy(g["w"]).cuda())
    assert np.array_equal(u8(q), g[f"{fmt}_w_q"])
    assert np.array_equal(f32bits(s), g[f"{fmt}_w_s"].view(np.uint32))
    # a CPU weight is quantised on the GPU and comes back on the CPU
    qc, sc = mod.quantize(torch.from_numpy(g["w"]))
    assert qc.device.type == "cpu" and np.array_equal(qc.view(torch.uint8).numpy(), g[f"{fmt}_w_q"])


@pytest.mark.parametrize("fmt", ["fp8", "int8"])
@pytest.mark.parametrize("N, K", [(128, 128), (768, 1024), (5120, 2048)])
def test_weight_quantize_bit_exact(b2, fmt, N, K):
    g = torch.Generator().manual_seed(N + K)
    w = (torch.randn(N, K, generator=g) * 0.02).bfloat16()
    q, s = fmt_mod(b2, fmt).quantize(w.cuda())
    qo, so = obq.quantize(w.float().numpy(), fmt)
    assert np.array_equal(u8(q), qo.view(np.uint8))
    assert np.array_equal(f32bits(s), so.view(np.uint32))


def test_nvfp4_act_quant_golden(b2):
    g = golden("nvfp4")
    x = torch.from_numpy(widen_bf16(g["x_bf16"])).cuda().bfloat16()
    q, s = b2.nvfp4.act_quant(x, torch.from_numpy(g["inv_g"]).cuda())
    assert np.array_equal(q.cpu().numpy(), g["act_q_padded"])
    assert np.array_equal(s.cpu().numpy(), g["act_s_swizzled"])


@pytest.mark.parametrize("M, K, dtype", [(1, 64, torch.bfloat16), (37, 512, torch.bfloat16),
                                         (128, 2048, torch.bfloat16), (1000, 2048, torch.bfloat16),
                                         (4099, 6144, torch.bfloat16), (4099, 6208, torch.bfloat16),
                                         (2500, 4160, torch.float32), (3000, 2048, torch.float16)])
def test_nvfp4_act_quant_bit_exact(b2, M, K, dtype):
    """Also the two-tiles-a-CTA kernel (large M x K) with an odd number of 64-feature tiles, and 16- / 32-bit input."""
    x = heavy(M, K, seed=7 * M + K, dtype=dtype)
    inv_g = np.float32(1.0) / onv.global_scale(float(x.float().abs().max()))
    q, s = b2.nvfp4.act_quant(x.cuda(), torch.tensor([inv_g], device="cuda"))
    qo, so = onv.act_quant(x.float().numpy(), inv_g)
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(s.cpu().numpy(), so)


@pytest.mark.parametrize("name", ["w1", "w2", "lin_w"])
def test_nvfp4_weight_quantize_golden(b2, name):
    g = golden("nvfp4")
    c, s, wg = b2.nvfp4.quantize(torch.from_numpy(g[name]).cuda())
    tag = "lin" if name == "lin_w" else name
    assert np.array_equal(c.cpu().numpy(), g[f"{tag}_codes"])
    assert np.array_equal(u8(s), g[f"{tag}_scales"])
    if tag != "lin":
        assert np.array_equal(f32bits(wg), g[f"{tag}_g"].view(np.uint32))


@pytest.mark.parametrize("N, K", [(256, 2048), (2048, 6144)])
def test_nvfp4_weight_quantize_bit_exact(b2, N, K):
    g = torch.Generator().manual_seed(N * 3 + K)
    w = torch.randn(N, K, generator=g) * 0.02
    c, s, wg = b2.nvfp4.quantize(w.cuda())
    co, so, go = onv.quantize(w.numpy())
    assert np.array_equal(c.cpu().numpy(), co)
    assert np.array_equal(u8(s), so)
    assert np.array_equal(f32bits(wg), go.view(np.uint32))


def test_nvfp4_act_quant_code_thresholds(b2):
    """Quotients exactly at the e2m1 code thresholds (ties to even), one fp32 ulp either side, signed zeros and tiny
    values, under scales 1, 1.25 and 0.875 (fp32 input, inv_g = 1): the kernel's product-then-check path must give
    the codes of the reference's IEEE division."""
    cuts = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
    up, down = np.nextafter(cuts, np.float32(9)), np.nextafter(cuts, np.float32(0))
    rows = []
    for sc in (1.0, 1.25, 0.875):
        for vals in (cuts, up, down, -cuts, -up, -down):
            g = np.zeros(16, np.float32)
            g[0] = 6.0 * sc                       # amax: the group's scale is e4m3(6 sc / 6) = sc
            g[1:8] = vals * np.float32(sc)
            g[8:15] = np.nextafter(vals * np.float32(sc), np.float32(0))
            g[15] = -0.0
            rows.append(g)
    z = np.zeros(16, np.float32)
    z[[1, 3, 5]] = -0.0
    z[2], z[4], z[6] = np.float32(-1e-40), np.float32(1e-40), np.float32(-1e-30)
    z[0] = 6.0
    rows.append(z)
    rows.append(np.linspace(-7, 7, 16, dtype=np.float32))
    x = np.stack(rows).reshape(-1, 64)            # 20 groups: 5 rows of 64 features
    q, s = b2.nvfp4.act_quant(torch.from_numpy(x).cuda(), torch.tensor([1.0], device="cuda"))
    qo, so = onv.act_quant(x, np.float32(1.0))
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(s.cpu().numpy(), so)
