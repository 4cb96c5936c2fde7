"""The tcgen05 block GEMM (FP8 kind::f8f6f4, INT8 kind::i8) against the oracle's maths (basal/blockquant.py:54-60),
the reference's own GPU tests restated (tests/test_fp8block.py:134-148, tests/test_int8block.py:71-84: the maths
within 2e-3 (FP8) / 1e-5 (INT8), a row's output bit-identical alone and among other rows), the bf16 output within
1e-2 relative, the edge cases (M = 0, partial tiles, N % 256 = 128, bias) and the full
C2 projection shapes through row samples."""
import numpy as np
import pytest
import torch

from oracle import blockquant as obq

pytestmark = pytest.mark.gpu

TOL = {"fp8": 2e-3, "int8": 1e-5}


@pytest.fixture(scope="module")
def b2():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import basal_b200
    return basal_b200


def mod(b2, fmt):
    return b2.fp8block if fmt == "fp8" else b2.int8block


def operands(b2, fmt, M, N, K, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).bfloat16().cuda()
    w = (torch.randn(N, K, generator=g) / 32).cuda()
    m = mod(b2, fmt)
    q, s = m.quantize(w)
    qa, sa = m.act_quant(x)
    return x, q, s, qa, sa


def oracle_y(fmt, qa, sa, q, s):
    c = lambda t: t.view(torch.uint8).cpu().numpy() if fmt == "fp8" else t.cpu().numpy()  # noqa: E731
    return obq.gemm(c(qa), sa.cpu().numpy(), c(q), s.cpu().numpy(), fmt)


@pytest.mark.parametrize("fmt", ["fp8", "int8"])
@pytest.mark.parametrize("M, N, K", [(128, 256, 128), (1, 256, 128), (37, 768, 1024), (128, 768, 1024),
                                     (1000, 768, 1024), (300, 384, 256), (129, 128, 512)])
def test_gemm_equals_the_maths(b2, fmt, M, N, K):
    x, q, s, qa, sa = operands(b2, fmt, M, N, K, seed=M + N + K)
    y = mod(b2, fmt).gemm(qa, sa, q, s, torch.float32)
    ref = oracle_y(fmt, qa, sa, q, s)
    got = y.cpu().numpy()
    assert np.allclose(got, ref, rtol=TOL[fmt], atol=TOL[fmt]), np.abs(got - ref).max()


@pytest.mark.parametrize("fmt", ["fp8", "int8"])
@pytest.mark.parametrize("M", [1, 37, 128, 1000])
def test_kernel_ignores_the_other_rows(b2, fmt, M):
    """tests/test_fp8block.py:134-148: a row's output alone and among other rows, bit for bit."""
    x, q, s, qa, sa = operands(b2, fmt, M, 768, 1024)
    m = mod(b2, fmt)
    alone = m.gemm(qa[-1:], sa[-1:], q, s, torch.bfloat16)
    many = m.gemm(torch.cat([qa, qa]), torch.cat([sa, sa]), q, s, torch.bfloat16)
    assert torch.equal(alone[0], many[M - 1]) and torch.equal(many[M - 1], many[2 * M - 1])


@pytest.mark.parametrize("fmt", ["fp8", "int8"])
@pytest.mark.parametrize("M", [1, 16, 32, 33, 64, 65, 100, 128])
def test_few_rows_kernel_equals_the_maths_and_the_large_kernel(b2, fmt, M):
    """M <= 128 runs the weight-streaming kernel (weights as the MMA's M side): within the maths' tolerance, and
    every row bit-identical to the same row computed by the large-M kernel among 300 rows, for fp32 and bf16."""
    N, K = 640, 1152
    x, q, s, qa, sa = operands(b2, fmt, 300, N, K, seed=M)
    m = mod(b2, fmt)
    for dt in (torch.float32, torch.bfloat16, torch.float16):
        small = m.gemm(qa[:M].contiguous(), sa[:M].contiguous(), q, s, dt)
        large = m.gemm(qa, sa, q, s, dt)
        assert torch.equal(small, large[:M]), (dt, (small.float() - large[:M].float()).abs().max())
    ref = oracle_y(fmt, qa[:M], sa[:M], q, s)
    got = m.gemm(qa[:M].contiguous(), sa[:M].contiguous(), q, s, torch.float32).cpu().numpy()
    assert np.allclose(got, ref, rtol=TOL[fmt], atol=TOL[fmt]), np.abs(got - ref).max()


def capi_gemm(fmt, qa, sa, q, s, dt, bias, work):
    """The block GEMM through the C ABI, with the caller's workspace (a uint8 tensor) or none."""
    from basal_b200 import _lib
    M, K = qa.shape
    N = q.shape[0]
    c = torch.empty(M, N, dtype=dt, device=qa.device)
    name = "basal200_int8_block_gemm" if fmt == "int8" else "basal200_fp8_block_gemm"
    _lib.call(name, qa.device, _lib.ptr(qa), _lib.ptr(sa), _lib.ptr(q), _lib.ptr(s), _lib.ptr(bias), _lib.ptr(c),
              _lib.code(dt), M, N, K, _lib.ptr(work), 0 if work is None else work.numel())
    return c


@pytest.mark.parametrize("fmt", ["fp8", "int8"])
@pytest.mark.parametrize("M, N, K", [(1, 2048, 2048), (16, 2048, 6144), (33, 1280, 2048), (64, 2048, 2048),
                                     (16, 8192, 2048), (5, 640, 1152), (64, 256, 8192)])
def test_split_few_rows_gemm_is_bit_identical_to_the_unsplit_kernel(b2, fmt, M, N, K):
    """The few-rows GEMM spread over every SM (each slice's product into the workspace, then the slice-ordered sum in
    a second kernel) gives the unsplit kernel's bits: fp32, bf16 and fp16 outputs, with and without bias, on two calls
    in a row that share one workspace. The workspace starts as NaN bytes, so a product the sum reads without the call
    having written it shows. Runs of units that cross weight tiles (N = 8192: 1024 units on the SMs) included."""
    from basal_b200 import _lib
    need = _lib.lib().basal200_block_gemm_workspace_bytes(M, N, K)
    assert need == M * N * (K // 128) * 4
    work = torch.full((need,), 0xFF, dtype=torch.uint8, device="cuda")
    for seed in (1, 2):
        x, q, s, qa, sa = operands(b2, fmt, M, N, K, seed=seed * 1000 + M)
        for dt in (torch.float32, torch.bfloat16, torch.float16):
            bias = None if dt == torch.float32 else torch.randn(N, generator=torch.Generator().manual_seed(seed)).to(
                dt).cuda()
            split = capi_gemm(fmt, qa, sa, q, s, dt, bias, work)
            whole = capi_gemm(fmt, qa, sa, q, s, dt, bias, None)
            assert torch.equal(split, whole), (dt, (split.float() - whole.float()).abs().max())
        if seed == 1:  # within the maths' tolerance, fp32
            ref = oracle_y(fmt, qa, sa, q, s)
            got = capi_gemm(fmt, qa, sa, q, s, torch.float32, None, work).cpu().numpy()
            assert np.allclose(got, ref, rtol=TOL[fmt], atol=TOL[fmt]), np.abs(got - ref).max()
    assert b2._lib.device_faults(0) == 0


def capi_linear(fmt, x, q, s, bias, work):
    """The block linear through the C ABI (output in x's type); returns the output and the activation scales."""
    from basal_b200 import _lib
    M, K = x.shape
    N = q.shape[0]
    y = torch.empty(M, N, dtype=x.dtype, device=x.device)
    qs = torch.empty(M, K, dtype=torch.uint8, device=x.device)
    ss = torch.full((M, K // 128), float("nan"), dtype=torch.float32, device=x.device)
    name = "basal200_int8_block_linear" if fmt == "int8" else "basal200_fp8_block_linear"
    _lib.call(name, x.device, _lib.ptr(x), _lib.code(x.dtype), _lib.ptr(q), _lib.ptr(s), _lib.ptr(bias), _lib.ptr(y),
              M, N, K, _lib.ptr(qs), _lib.ptr(ss), _lib.ptr(work), 0 if work is None else work.numel())
    return y, ss


@pytest.mark.parametrize("fmt", ["fp8", "int8"])
@pytest.mark.parametrize("M, N, K", [(1, 2048, 2048), (16, 2048, 6144), (33, 1280, 2048), (64, 2048, 2048),
                                     (7, 8192, 1152)])
def test_fused_quantiser_linear_is_bit_identical(b2, fmt, M, N, K):
    """A few-rows linear whose activation quantiser runs inside the split GEMM (16-bit x: codes written straight into
    the GEMM's operand stages, scales into the scratch) gives the bits of the quantiser kernel + unsplit GEMM: the same
    output and the same scales, bf16 and fp16 activations, with and without bias, on two calls in a row sharing a
    workspace. Activations include an all-zero token, a tiny one and an outlier."""
    from basal_b200 import _lib
    need = _lib.lib().basal200_block_gemm_workspace_bytes(M, N, K)
    assert need > 0
    work = torch.full((need,), 0xFF, dtype=torch.uint8, device="cuda")
    g = torch.Generator().manual_seed(M * 7 + K)
    w = (torch.randn(N, K, generator=g) * 0.02).cuda()
    q, s = mod(b2, fmt).quantize(w)
    for seed in (1, 2):
        x = torch.randn(M, K, generator=g) * (1 + seed)
        x[0, :128] = 0.0
        if M > 2:
            x[1] *= 1e-30
            x[2, 5] = 3e4
        for dt in (torch.bfloat16, torch.float16):
            xd = x.to(dt).cuda()
            bias = None if seed == 1 else torch.randn(N, generator=g).to(dt).cuda()
            fused, s_f = capi_linear(fmt, xd, q, s, bias, work)
            plain, s_p = capi_linear(fmt, xd, q, s, bias, None)
            assert torch.equal(s_f, s_p), (dt, seed)
            assert torch.equal(fused, plain), (dt, seed, (fused.float() - plain.float()).abs().max())
    assert b2._lib.device_faults(0) == 0


def test_split_workspace_too_small_or_misaligned(b2):
    """A workspace smaller than asked for runs the unsplit kernel (same bits); a misaligned one is refused."""
    from basal_b200 import _lib
    M, N, K = 16, 2048, 2048
    x, q, s, qa, sa = operands(b2, "fp8", M, N, K, seed=9)
    need = _lib.lib().basal200_block_gemm_workspace_bytes(M, N, K)
    small = torch.empty(need - 16, dtype=torch.uint8, device="cuda")
    assert torch.equal(capi_gemm("fp8", qa, sa, q, s, torch.bfloat16, None, small),
                       capi_gemm("fp8", qa, sa, q, s, torch.bfloat16, None, None))
    big = torch.empty(need + 16, dtype=torch.uint8, device="cuda")
    with pytest.raises(ValueError, match="align"):
        capi_gemm("fp8", qa, sa, q, s, torch.bfloat16, None, big[4:])


@pytest.mark.parametrize("fmt", ["fp8", "int8"])
@pytest.mark.parametrize("M", [517, 7])
def test_bf16_linear_within_north_star_tolerance(b2, fmt, M):
    """linear (act_quant + GEMM, bf16 out, bias) against the oracle's linear: 1e-2 relative, for the large-M and
    the few-rows kernel."""
    N, K = 1280, 2048
    g = torch.Generator().manual_seed(5)
    x = torch.randn(M, K, generator=g).bfloat16()
    w = torch.randn(N, K, generator=g) * 0.02
    bias = torch.randn(N, generator=g).bfloat16()
    m = mod(b2, fmt)
    q, s = m.quantize(w.cuda())
    y = m.linear(x.cuda(), q, s, bias.cuda())
    assert y.dtype == torch.bfloat16 and y.shape == (M, N)
    qc = q.view(torch.uint8).cpu().numpy() if fmt == "fp8" else q.cpu().numpy()
    ref = obq.linear(x.float().numpy(), qc, s.cpu().numpy(), fmt)
    ref = torch.from_numpy(ref).bfloat16().float() + bias.float()  # the bias added to the cast output
    err = (y.float().cpu() - ref).abs().max() / ref.abs().max()
    assert err < 1e-2, err


def test_empty_rows_and_refusals(b2):
    x, q, s, qa, sa = operands(b2, "fp8", 4, 256, 256)
    y = b2.fp8block.gemm(qa[:0], sa[:0], q, s, torch.bfloat16)
    assert y.shape == (0, 256)
    assert b2.fp8block.linear(x[:0], q, s).shape == (0, 256)
    with pytest.raises(ValueError, match="not a multiple of 128"):
        b2.blockquant.grid(4, 200)
    with pytest.raises(ValueError):
        b2.fp8block.gemm(qa, sa, q[:200], s[:2], torch.bfloat16)


@pytest.mark.parametrize("fmt", ["fp8", "int8"])
@pytest.mark.parametrize("name, N, K", [("qkv", 5120, 2048), ("o", 2048, 2048), ("gate_up", 12288, 2048),
                                        ("down", 2048, 6144)])
def test_c2_projection_shapes_by_row_samples(b2, fmt, name, N, K):
    """The config-2 projections at a packed M of 8,320 rows: 64 sampled rows against the oracle (within the
    north-star 1e-2 of each row's largest output) and the sampled rows recomputed alone, bit for bit."""
    M = 8320
    g = torch.Generator().manual_seed(N + K)
    x = torch.randn(M, K, generator=g).bfloat16().cuda()
    w = (torch.randn(N, K, generator=g) * 0.02).cuda()
    m = mod(b2, fmt)
    q, s = m.quantize(w)
    y = m.linear(x, q, s)
    rows = torch.randperm(M, generator=g)[:64].sort().values
    qa, sa = m.act_quant(x[rows.cuda()])
    qc = q.view(torch.uint8).cpu().numpy() if fmt == "fp8" else q.cpu().numpy()
    qac = qa.view(torch.uint8).cpu().numpy() if fmt == "fp8" else qa.cpu().numpy()
    ref = obq.gemm(qac, sa.cpu().numpy(), qc, s.cpu().numpy(), fmt)
    got = y[rows.cuda()].float().cpu().numpy()
    err = np.abs(got - ref).max(1) / np.abs(ref).max(1)
    assert err.max() < 1e-2, err.max()
    assert torch.equal(m.linear(x[rows.cuda()], q, s), y[rows.cuda()])


@pytest.mark.parametrize("fmt", ["fp8", "int8"])
@pytest.mark.parametrize("act", ["silu", "gelu_tanh"])
@pytest.mark.parametrize("M, I, K, dt", [(1, 128, 256, torch.bfloat16), (37, 384, 1024, torch.bfloat16),
                                         (300, 256, 512, torch.float16), (1000, 640, 2048, torch.bfloat16)])
def test_gated_linear_equals_the_unfused_ops(b2, fmt, act, M, I, K, dt):
    """act(gate) * up of a merged [gate; up] weight in one GEMM (the epilogue pairs gate block n with up block n):
    within one unit in the last place of x's dtype of the unfused ops on the same GPU (the merged linear, cast, then
    torch's activation and product on those tensors: the gate and up values are the same bits, only the activation's
    implementation may differ), and within the north-star 1e-2 of the oracle's fp32 linear followed by the same ops
    on CPU; rows past M and every 128-column output tile covered."""
    g = torch.Generator().manual_seed(M + I + K)
    x = torch.randn(M, K, generator=g).to(dt)
    w = torch.randn(2 * I, K, generator=g) * 0.02
    m = mod(b2, fmt)
    q, s = m.quantize(w.cuda())
    fused = m.FORMAT.linear_glu(x.cuda(), q, s, act)
    assert fused.shape == (M, I) and fused.dtype == dt
    f = torch.nn.functional.silu if act == "silu" else (lambda t: torch.nn.functional.gelu(t, approximate="tanh"))
    full = m.linear(x.cuda(), q, s)
    want = f(full[:, :I]) * full[:, I:]
    eps = 2.0 ** -7 if dt == torch.bfloat16 else 2.0 ** -10
    diff = (fused.float() - want.float()).abs()
    assert bool((diff <= eps * want.float().abs() + 1e-6).all()), diff.max()
    qc = q.view(torch.uint8).cpu().numpy() if fmt == "fp8" else q.cpu().numpy()
    ref_full = torch.from_numpy(obq.linear(x.float().numpy(), qc, s.cpu().numpy(), fmt)).to(dt)
    ref = (f(ref_full[:, :I].float()).to(dt).float() * ref_full[:, I:].float()).to(dt).float()
    err = (fused.float().cpu() - ref).abs().max() / ref.abs().max()
    assert err < 1e-2, err
    assert b2._lib.device_faults(0) == 0


@pytest.mark.parametrize("fmt", ["fp8", "int8"])
@pytest.mark.parametrize("act", ["silu", "gelu_tanh"])
@pytest.mark.parametrize("I", [256, 6144])
def test_gated_linear_rows_alone_and_among_others(b2, fmt, act, I):
    """A row's gated output is the same bits alone (few rows: the merged linear into a temporary, then the activation
    kernel; split over the SMs at I = 256) and among 300 rows (the large-M kernel's gated epilogue)."""
    K = 1024
    g = torch.Generator().manual_seed(I + len(act))
    x = torch.randn(300, K, generator=g).bfloat16().cuda()
    m = mod(b2, fmt)
    q, s = m.quantize((torch.randn(2 * I, K, generator=g) * 0.02).cuda())
    many = m.FORMAT.linear_glu(x, q, s, act)
    for M in (1, 16, 64):
        few = m.FORMAT.linear_glu(x[:M].contiguous(), q, s, act)
        assert torch.equal(few, many[:M]), (M, (few.float() - many[:M].float()).abs().max())


@pytest.mark.parametrize("fmt", ["fp8", "int8"])
def test_gated_linear_without_workspace(b2, fmt):
    """Through the C ABI with no workspace, a few-rows gated linear runs the many-rows kernel's gated epilogue: the
    same bits as the op (which passes a workspace: the few-rows linear into a temporary, then the activation)."""
    from basal_b200 import _lib
    M, I, K = 16, 384, 512
    g = torch.Generator().manual_seed(11)
    x = torch.randn(M, K, generator=g).bfloat16().cuda()
    m = mod(b2, fmt)
    q, s = m.quantize((torch.randn(2 * I, K, generator=g) * 0.02).cuda())
    y = torch.empty(M, I, dtype=torch.bfloat16, device="cuda")
    qs = torch.empty(M, K, dtype=torch.uint8, device="cuda")
    ss = torch.empty(M, K // 128, dtype=torch.float32, device="cuda")
    name = "basal200_int8_block_linear_glu" if fmt == "int8" else "basal200_fp8_block_linear_glu"
    _lib.call(name, x.device, _lib.ptr(x), _lib.BF16, _lib.ptr(q), _lib.ptr(s), _lib.ptr(y), M, I, K, 1,
              _lib.ptr(qs), _lib.ptr(ss), None, 0)
    assert torch.equal(y, m.FORMAT.linear_glu(x, q, s, "silu"))


def test_gated_linear_module_and_refusals(b2):
    """BlockFP8Linear.glu on a merged layer is the op; a bias, an odd row count or an unknown activation is refused."""
    g = torch.Generator().manual_seed(5)
    lin = torch.nn.Linear(512, 512, bias=False)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(512, 512, generator=g) * 0.02)
    layer = b2.fp8block.BlockFP8Linear.of(lin.cuda())
    x = torch.randn(3, 7, 512, generator=g).bfloat16().cuda()
    y = layer.glu(x, "gelu_tanh")
    assert y.shape == (3, 7, 256)
    assert torch.equal(y.reshape(21, 256),
                       torch.ops.basal.fp8_block_linear_glu(x.reshape(21, 512), layer.weight, layer.weight_scale,
                                                            "gelu_tanh"))
    with pytest.raises(ValueError):
        layer.glu(x, "relu")
    with pytest.raises(ValueError):
        torch.ops.basal.fp8_block_linear_glu(x.reshape(21, 512), layer.weight[:384], layer.weight_scale[:3], "silu")


@pytest.mark.parametrize("fmt", ["fp8", "int8"])
@pytest.mark.parametrize("M, N, K, dt, with_bias", [(1, 256, 256, torch.bfloat16, False),
                                                    (16, 2048, 2048, torch.bfloat16, True),
                                                    (64, 384, 1024, torch.float16, False),
                                                    (300, 384, 512, torch.bfloat16, True),
                                                    (1000, 2048, 1024, torch.float16, True)])
def test_residual_linear_equals_linear_then_add(b2, fmt, M, N, K, dt, with_bias):
    """residual + linear(x) with the sum in the GEMM's epilogue (many rows: the residual tile TMA-loaded into the
    staging buffer; few rows: the few-rows linear into a temporary, then the addition) is bit for bit the linear
    followed by torch's addition, with and without bias, N % 256 = 128 (a half tile past N), bf16 and fp16."""
    g = torch.Generator().manual_seed(M + N + K)
    x = torch.randn(M, K, generator=g).to(dt).cuda()
    h = torch.randn(M, N, generator=g).to(dt).cuda()
    bias = torch.randn(N, generator=g).to(dt).cuda() if with_bias else None
    m = mod(b2, fmt)
    q, s = m.quantize((torch.randn(N, K, generator=g) * 0.02).cuda())
    got = m.FORMAT.linear_residual(x, q, s, bias, h)
    want = h + m.linear(x, q, s, bias)
    assert torch.equal(got, want), (got.float() - want.float()).abs().max()
    assert b2._lib.device_faults(0) == 0


@pytest.mark.parametrize("fmt", ["fp8", "int8"])
def test_residual_linear_in_place(b2, fmt):
    """Through the C ABI with y = the residual (h += o_proj(x)) and no workspace: the many-rows kernel reads each
    residual tile before its output tile is stored, so the update in place equals the two-step result."""
    from basal_b200 import _lib
    M, N, K = 300, 640, 512
    g = torch.Generator().manual_seed(21)
    x = torch.randn(M, K, generator=g).bfloat16().cuda()
    h = torch.randn(M, N, generator=g).bfloat16().cuda()
    m = mod(b2, fmt)
    q, s = m.quantize((torch.randn(N, K, generator=g) * 0.02).cuda())
    want = h + m.linear(x, q, s)
    qs = torch.empty(M, K, dtype=torch.uint8, device="cuda")
    ss = torch.empty(M, K // 128, dtype=torch.float32, device="cuda")
    name = "basal200_int8_block_linear_residual" if fmt == "int8" else "basal200_fp8_block_linear_residual"
    _lib.call(name, x.device, _lib.ptr(x), _lib.BF16, _lib.ptr(q), _lib.ptr(s), None, _lib.ptr(h), _lib.ptr(h),
              M, N, K, _lib.ptr(qs), _lib.ptr(ss), None, 0)
    assert torch.equal(h, want)
