"""The CPU oracle (oracle/) against the golden fixtures the reference itself wrote (tests/golden/make_golden.py):
codes and scales bit for bit, GEMM / linear / readout outputs to fp32 rounding. Also the reference's own
known-answer tests for this path (tests/test_nvfp4.py:13-23, tests/test_blockquant.py:55-68,
tests/test_fp8block.py:16-26, tests/test_int8block.py:14-22) restated on the oracle. No GPU."""
import numpy as np
import pytest

from conftest import golden, widen_bf16
from oracle import blockquant as bq
from oracle import fp8, nvfp4, readout


@pytest.fixture(scope="module")
def gb():
    return golden("blockquant")


@pytest.fixture(scope="module")
def gn():
    return golden("nvfp4")


@pytest.mark.parametrize("fmt", ["fp8", "int8"])
def test_act_quant_bit_exact(gb, fmt):
    for x, tag in ((widen_bf16(gb["x_bf16"]), "act"), (gb["xf"], "actf")):
        q, s = bq.act_quant(x, fmt)
        assert np.array_equal(q.view(np.uint8), gb[f"{fmt}_{tag}_q"])
        assert np.array_equal(s.view(np.uint32), gb[f"{fmt}_{tag}_s"].view(np.uint32))


@pytest.mark.parametrize("fmt", ["fp8", "int8"])
def test_weight_quantize_bit_exact(gb, fmt):
    q, s = bq.quantize(gb["w"], fmt)
    assert np.array_equal(q.view(np.uint8), gb[f"{fmt}_w_q"])
    assert np.array_equal(s.view(np.uint32), gb[f"{fmt}_w_s"].view(np.uint32))


@pytest.mark.parametrize("fmt", ["fp8", "int8"])
def test_gemm_and_linear(gb, fmt):
    x, w = widen_bf16(gb["gemm_x_bf16"]), widen_bf16(gb["gemm_w_bf16"])
    q, s = bq.quantize(w, fmt)
    assert np.array_equal(q.view(np.uint8), gb[f"{fmt}_gemm_wq"])
    qa, sa = bq.act_quant(x, fmt)
    y = bq.gemm(qa, sa, q, s, fmt)
    ref = gb[f"{fmt}_gemm_y"]
    assert np.allclose(y, ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())
    yl = bq.linear(x, q, s, fmt, gb["gemm_bias"])
    assert np.allclose(yl, gb[f"{fmt}_linear_y"], rtol=1e-5, atol=1e-5 * np.abs(ref).max())


def test_known_answers_block_formats(gb):
    """Every block reaches qmax exactly; FP8 error within |w| 2^-4 + s 2^-9, INT8 within half a step
    (tests/test_fp8block.py:16-26, tests/test_int8block.py:14-22)."""
    w = gb["w"]
    for fmt, qmax in (("fp8", 448.0), ("int8", 127.0)):
        q, s = bq.quantize(w, fmt)
        deq = bq.dequant_w(q, s, fmt)
        assert np.all(np.abs(bq.decode(q, fmt)).reshape(2, 128, 3, 128).max((1, 3)) == qmax)
        step = np.repeat(np.repeat(s, 128, 0), 128, 1)
        bound = np.abs(w) * 2 ** -4 + step * 2 ** -9 if fmt == "fp8" else step * 0.5
        assert np.all(np.abs(deq - w) <= bound * 1.0001)


def test_e2m1_table_and_cuts(gn):
    assert np.array_equal(fp8.e2m1_codes(gn["table_u"]), gn["table_codes"])
    assert fp8.e2m1_values(fp8.e2m1_codes(gn["table_u"])).tolist() == \
        [0, 0, .5, 1, 1, 1, 1.5, 2, 2, 2, 3, 4, 4, 4, 6, 6, -1, -4]
    assert [t for t, _ in fp8.CUTS] == [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0]


def test_nvfp4_act_quant_bit_exact(gn):
    x = widen_bf16(gn["x_bf16"])
    codes, scales = nvfp4.act_ops(x, gn["inv_g"][0])
    assert np.array_equal(codes, gn["act_codes"]) and np.array_equal(scales, gn["act_scales"])
    q, s = nvfp4.act_quant(x, gn["inv_g"][0])
    assert np.array_equal(q, gn["act_q_padded"]) and np.array_equal(s, gn["act_s_swizzled"])


def test_swizzle_round_trip(gn):
    f = nvfp4.swizzle(gn["swz_in"])
    assert np.array_equal(f, gn["swz_out"]) and f.size == 384 * 52
    assert np.array_equal(nvfp4.unswizzle(f, 300, 52), gn["swz_in"])


@pytest.mark.parametrize("name", ["w1", "w2"])
def test_nvfp4_weight_quantize_bit_exact(gn, name):
    c, s, g = nvfp4.quantize(gn[name])
    assert np.array_equal(c, gn[f"{name}_codes"])
    assert np.array_equal(s, gn[f"{name}_scales"])
    assert np.array_equal(g.view(np.uint32), gn[f"{name}_g"].view(np.uint32))


def test_nvfp4_linear(gn):
    c, s, g = nvfp4.quantize(gn["lin_w"])
    assert np.array_equal(c, gn["lin_codes"]) and np.array_equal(s, gn["lin_scales"])
    x = widen_bf16(gn["x_bf16"])
    y = nvfp4.linear(x, c, s, gn["lin_alpha"][0], gn["lin_inv_g"][0])
    ref = gn["lin_y_f32"]
    assert np.allclose(y, ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())


@pytest.mark.parametrize("tag, cap, bias", [("cap", 30.0, True), ("plain", None, False)])
def test_readout(tag, cap, bias):
    g = golden("readout")
    lids = [[int(i) for i in row if i >= 0] for row in g["lids"]]
    hb = g["head_b"] if bias else None
    for fn, key in ((readout.probs, "probs"), (readout.probs_each, "probs_each")):
        got = fn(g["head_w"], hb, g["h"], lids, cap)
        for row, ids, want in zip(got, lids, g[f"{key}_{tag}"]):
            assert np.allclose(row, want[: len(ids)], atol=1e-6)
