"""Host-side logic of basal_b200 without a GPU: the reference's interface (names, layouts, refusals), the storage
layout helpers against the oracle, the readout's row bookkeeping, the dispatch shim, and that the product path refuses
to compute on the CPU (no fallback)."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import fp8 as ofp8
from oracle import nvfp4 as onv


@pytest.fixture(scope="module")
def b2():
    import basal_b200
    return basal_b200


def test_formats_share_one_core(b2):
    """tests/test_blockquant.py:13-29 restated: FP8 and INT8 are formats of one core, one layer class."""
    for mod, cls, dtype, qmax in ((b2.fp8block, b2.fp8block.BlockFP8Linear, torch.float8_e4m3fn, 448.0),
                                  (b2.int8block, b2.int8block.Int8BlockLinear, torch.int8, 127.0)):
        f = mod.FORMAT
        assert isinstance(f, b2.blockquant.BlockFormat)
        assert (f.dtype, f.qmax, f.rounded) == (dtype, qmax, dtype == torch.int8)
        assert mod.quantize.__self__ is f and mod.act_quant.__self__ is f and mod.gemm.__self__ is f
        assert issubclass(cls, b2.blockquant.BlockLinear) and cls.FORMAT is f
    assert b2.fp8block.grid is b2.int8block.grid is b2.blockquant.grid
    assert b2.fp8block.sm90() is False


def test_grid_refuses_partial_output_tiles(b2):
    """tests/test_fp8block.py:29-38: N not a multiple of 128 is refused; the count is of 128 x 256 tiles here."""
    g = b2.blockquant.grid
    assert g(1, 384) == (2,) and g(129, 384) == (4,) and g(0, 128) == (0,) and g(1, 256) == (1,)
    for n in (200, 64):
        with pytest.raises(ValueError, match="not a multiple of 128"):
            g(4, n)


def test_fuse_makes_the_layers_views_of_one_weight(b2):
    """tests/test_blockquant.py:42-52."""
    torch.manual_seed(0)
    mods = [torch.nn.Linear(16, n, bias=False) for n in (8, 4, 4)]
    before = [m.weight.detach().clone() for m in mods]
    w, sizes = b2.blockquant.fuse(mods)
    assert sizes == [8, 4, 4] and torch.equal(w, torch.cat(before))
    for m, b in zip(mods, before):
        assert torch.equal(m.weight, b) and m.weight.untyped_storage().data_ptr() == w.untyped_storage().data_ptr()


def test_block_linear_part_is_a_view(b2):
    q = torch.zeros(384, 256, dtype=torch.float8_e4m3fn)
    s = torch.ones(3, 2)
    m = b2.fp8block.BlockFP8Linear(q, s)
    p = m.part(128, 256)
    assert type(p) is b2.fp8block.BlockFP8Linear and p.weight.shape == (256, 256) and p.weight_scale.shape == (2, 2)
    assert p.weight.data_ptr() == m.weight.data_ptr() + 128 * 256
    assert (m.in_features, m.out_features) == (256, 384)


def test_nvfp4_constants_and_layout_match_the_oracle(b2):
    n = b2.nvfp4
    assert n.E2M1 == ofp8.E2M1 and n.CUTS == ofp8.CUTS and n.CANDIDATES == onv.CANDIDATES
    assert [t for t, _ in n.CUTS] == [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0]
    g = golden("nvfp4")
    s = torch.from_numpy(g["swz_in"]).view(torch.float8_e4m3fn)
    f = n.swizzle(s)
    assert np.array_equal(f.view(torch.uint8).numpy(), g["swz_out"])
    assert torch.equal(n.unswizzle(f, 300, 52).view(torch.uint8), s.view(torch.uint8))
    c = torch.randint(0, 16, (5, 64), dtype=torch.uint8)
    assert torch.equal(n.unpack(n.pack(c)), c)
    assert np.array_equal(n.pack(c).numpy(), onv.pack(c.numpy()))


def test_nvfp4_part_views(b2):
    n = b2.nvfp4
    w = torch.zeros(256, 64, dtype=torch.uint8)
    sc = torch.zeros(256 * 8, dtype=torch.uint8).view(torch.float8_e4m3fn)
    f = n.NVFP4Linear(w, sc, torch.tensor([1.0]), torch.tensor([2.0]))
    assert (f.in_features, f.out_features) == (128, 256)
    p = f.part(128, 128)
    assert p.weight.shape == (128, 64) and p.weight_scale.numel() == 128 * 8
    assert float(f.alpha) == 2.0 and float(f.inv_g) == 0.5
    with pytest.raises(AssertionError):
        f.part(64, 128)


def test_readout_rows_bookkeeping(b2):
    """CodeReadout.rows: the sorted union of the prompts' codes, each prompt's columns into it, the padding
    (basal/readout.py:57-69); the cache keeps entries by key within WROWS_BYTES."""
    head = torch.nn.Linear(8, 20)
    r = b2.readout.CodeReadout(head, softcap=2.0)
    (ids, b), idx, pad = r.rows([[3, 4], [5, 6, 7], [4, 3]])
    assert ids.tolist() == [3, 4, 5, 6, 7] and b is None
    assert idx.tolist() == [[0, 1, 0], [2, 3, 4], [1, 0, 0]]
    assert pad.tolist() == [[False, False, True], [False, False, False], [False, False, True]]
    assert list(r.cache) == [(3, 4, 5, 6, 7)]
    cache = {}
    big = lambda: torch.zeros(b2.readout.WROWS_BYTES // 4 // 2 + 1)  # noqa: E731  (over half the budget)
    b2.readout.code_rows(cache, "a", big)
    b2.readout.code_rows(cache, "b", big)
    assert list(cache) == ["b"]


def test_lean_dispatch(b2):
    lin = torch.nn.Linear(8, 4)
    assert len(b2.lean._params(lin)) == 2
    x = torch.randn(3, 8)
    assert torch.equal(b2.lean.linear(x, b2.lean._params(lin)), torch.nn.functional.linear(x, lin.weight, lin.bias))
    m = b2.fp8block.BlockFP8Linear(torch.zeros(128, 128, dtype=torch.float8_e4m3fn), torch.ones(1, 1))
    assert len(b2.lean._params(m)) == 3
    with pytest.raises(NotImplementedError):
        b2.lean.linear(x, (1, 2, 3, 4))


def test_no_cpu_fallback(b2):
    """The product path computes on CUDA tensors only: a CPU activation is refused, not computed on the CPU."""
    x = torch.randn(4, 256)
    with pytest.raises(ValueError, match="CUDA"):
        b2.fp8block.act_quant(x)
    with pytest.raises(ValueError, match="CUDA"):
        b2.int8block.linear(x, torch.zeros(128, 256, dtype=torch.int8), torch.ones(1, 2))
    if not torch.cuda.is_available():
        with pytest.raises(ValueError, match="CUDA"):
            b2.fp8block.quantize(torch.randn(128, 128))


def test_product_never_imports_the_oracle():
    """Nothing under basal_b200/ imports oracle/ (the oracle is test infrastructure)."""
    import pathlib
    root = pathlib.Path(__file__).resolve().parents[1] / "basal_b200"
    for p in root.rglob("*.py"):
        src = p.read_text()
        assert "import oracle" not in src and "from oracle" not in src, p
