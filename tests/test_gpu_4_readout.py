"""The readout kernels (basal::code_logits, basal::code_probs) against the reference's golden probabilities and the
oracle (basal/readout.py:57-104): golden to 1e-5, the C4 shapes (R = 256 answer positions, D = 2048, a 151,936-row
bf16 head, 2 / 8 / 64 / 255 options) with identical argmax and max |diff| <= 1e-3 (checked here
at 1e-5), and a prompt's probabilities the same bits alone and in any batch."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import readout as oro

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def b2():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import basal_b200
    return basal_b200


class Head(torch.nn.Module):
    def __init__(self, w, b=None):
        super().__init__()
        self.weight = torch.nn.Parameter(w, requires_grad=False)
        self.bias = None if b is None else torch.nn.Parameter(b, requires_grad=False)


@pytest.mark.parametrize("tag, cap, bias", [("cap", 30.0, True), ("plain", None, False)])
def test_golden(b2, tag, cap, bias):
    g = golden("readout")
    lids = [[int(i) for i in row if i >= 0] for row in g["lids"]]
    w = torch.from_numpy(g["head_w"]).bfloat16().cuda()
    b = torch.from_numpy(g["head_b"]).bfloat16().cuda() if bias else None
    r = b2.readout.CodeReadout(Head(w, b), softcap=cap)
    h = torch.from_numpy(g["h"]).cuda()
    for fn, key in ((r.probs, "probs"), (r.probs_each, "probs_each")):
        got = fn(h, lids)
        for row, ids, want in zip(got, lids, g[f"{key}_{tag}"]):
            assert np.allclose(row, want[: len(ids)], atol=1e-5)


@pytest.fixture(scope="module")
def c4_head():
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(151936, 2048, generator=g) * 0.02).bfloat16()
    h = torch.randn(256, 2048, generator=g).bfloat16()
    return w, h


@pytest.mark.parametrize("k", [2, 8, 64, 255])
@pytest.mark.parametrize("cap", [None, 30.0])
def test_c4_shapes(b2, c4_head, k, cap):
    w, h = c4_head
    g = torch.Generator().manual_seed(k)
    ids = torch.randperm(151936, generator=g)[:k].tolist()
    lids = [ids] * 256
    r = b2.readout.CodeReadout(Head(w.cuda()), softcap=cap)
    got = np.asarray(r.probs(h.cuda(), lids))
    rows = w[ids].float().numpy()
    ref = oro.softmax(oro.logits(h.float().numpy(), (rows, None), cap))
    assert np.array_equal(got.argmax(1), ref.argmax(1))
    assert np.abs(got - ref).max() <= 1e-5


def test_batch_invariance(b2, c4_head):
    """Per-row code sets whose union is <= 255: each prompt's probabilities read alone are the same bits."""
    w, h = c4_head
    g = torch.Generator().manual_seed(9)
    pool = torch.randperm(151936, generator=g)[:255].tolist()
    lids = [pool[i % 200: i % 200 + 2 + i % 9] for i in range(64)]
    r = b2.readout.CodeReadout(Head(w.cuda()), softcap=30.0)
    hh = h[:64].cuda()
    batch = r.probs(hh, lids)
    assert batch == r.probs_each(hh, lids)
    for i in (0, 5, 63):
        assert r.probs(hh[i:i + 1], [lids[i]])[0] == batch[i]


@pytest.mark.parametrize("D, hdt", [(2560, torch.bfloat16), (1000, torch.float32), (300, torch.bfloat16)])
def test_code_tile_widths_agree_bit_for_bit(b2, D, hdt):
    """One code's logit is the same bits whether it is read among 3, 7 or 37 codes (items of 4, 8 or 16 codes a
    warp), at any position among them, for whole 256-feature chunks (D = 2560), a ragged tail (D = 1000, fp32 h) and a
    row stride off the 16-byte boundary (D = 300 bf16 in a 301-wide buffer: every feature on the lane-strided path);
    each within 1e-5 of the oracle's fp32 logits, with a bf16 bias and the Gemma soft cap."""
    g = torch.Generator().manual_seed(D)
    V = 5000
    w = (torch.randn(V, D, generator=g) * 0.02).bfloat16()
    bias = (torch.randn(V, generator=g) * 0.1).bfloat16()
    hbuf = torch.randn(19, D + (1 if D == 300 else 0), generator=g).to(hdt)
    h = hbuf[:, :D]
    pool = torch.randperm(V, generator=g)[:37].tolist()
    target = pool[2]
    head = Head(w.cuda(), bias.cuda())
    zs = []
    for ids in (pool[:3], [pool[5], pool[6], target, pool[8], pool[9], pool[10], pool[11]], pool):
        ids_t = torch.tensor(ids, dtype=torch.int64).cuda()
        z = b2.ops.code_logits(h.cuda(), head.weight, ids_t, head.bias, 30.0)
        zs.append(z[:, ids.index(target)].cpu())
    assert torch.equal(zs[0], zs[1]) and torch.equal(zs[1], zs[2])
    ref = oro.logits(h.float().numpy(), (w[pool].float().numpy(), bias[pool].float().numpy()), 30.0)
    got = b2.ops.code_logits(h.cuda(), head.weight, torch.tensor(pool).cuda(), head.bias, 30.0).cpu().numpy()
    assert np.abs(got - ref).max() <= 1e-5
    assert b2._lib.device_faults(0) == 0


# ---- the tensor-core path: h and head of one 16-bit type, 16-byte aligned rows, D % 8 == 0 ----

def _head(D, V, seed, dt=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(V, D, generator=g) / D ** 0.5).to(dt)
    bias = (torch.randn(V, generator=g) * 0.1).to(dt)
    return g, w, bias


@pytest.mark.parametrize("D", [8, 24, 200, 2048, 8192])
@pytest.mark.parametrize("R, U", [(1, 1), (130, 17), (300, 40)])
def test_tensor_core_shapes(b2, D, R, U):
    """Slices shorter than a swizzle row or empty (D = 8, 24, 200), one round (2048), four rounds a slice (8192);
    ragged prompt tiles (R = 130, 300) and code tiles (U = 17, 40): within 1e-5 of the oracle's fp32 logits."""
    g, w, bias = _head(D, 3000, D * 7 + R + U)
    h = torch.randn(R, D, generator=g).bfloat16()
    ids = torch.randperm(3000, generator=g)[:U]
    z = b2.ops.code_logits(h.cuda(), w.cuda(), ids.cuda(), bias.cuda(), 0.0).cpu().numpy()
    ref = oro.logits(h.float().numpy(), (w[ids].float().numpy(), bias[ids].float().numpy()), None)
    assert np.abs(z - ref).max() <= 1e-5
    assert b2._lib.device_faults(0) == 0


@pytest.mark.parametrize("cap", [None, 30.0])
def test_tensor_core_fp16(b2, cap):
    """fp16 h and head (the MMA's f16 operands): the C4 readout shape, within 1e-5 of the oracle."""
    g, w, bias = _head(2048, 20000, 11, torch.float16)
    h = torch.randn(256, 2048, generator=g).half()
    ids = torch.randperm(20000, generator=g)[:64]
    z = b2.ops.code_logits(h.cuda(), w.cuda(), ids.cuda(), None, cap or 0.0).cpu().numpy()
    ref = oro.logits(h.float().numpy(), (w[ids].float().numpy(), None), cap)
    assert np.abs(z - ref).max() <= 1e-5


def test_tensor_core_positions_bit_for_bit(b2):
    """A prompt's logit for a code is the same bits at any row of any prompt tile (rows 0, 127, 128, 299 of 300) and
    at any column of a 16- or 32-code tile (among 5 codes or 40), with a bf16 bias and the soft cap."""
    D, V = 2560, 4000
    g, w, bias = _head(D, V, 5)
    h = torch.randn(300, D, generator=g).bfloat16()
    pool = torch.randperm(V, generator=g)[:40]
    wc, bc = w.cuda(), bias.cuda()
    target_row, target_code = 7, int(pool[3])
    seen = []
    for pos in (0, 127, 128, 299):
        perm = list(range(300))
        perm[pos], perm[target_row] = perm[target_row], perm[pos]
        hp = h[perm].cuda()
        for ids in (pool[:5].tolist(), pool.tolist(), [int(pool[9]), target_code] + pool[20:23].tolist()):
            z = b2.ops.code_logits(hp, wc, torch.tensor(ids).cuda(), bc, 30.0)
            seen.append(z[pos, ids.index(target_code)].item())
    assert len(set(seen)) == 1, seen
    ref = oro.logits(h[target_row:target_row + 1].float().numpy(),
                     (w[[target_code]].float().numpy(), bias[[target_code]].float().numpy()), 30.0)
    assert abs(seen[0] - float(ref[0, 0])) <= 1e-5


def test_tensor_core_bad_id(b2):
    """An id outside [0, V) gives NaN logits in its column and the BAD_ID fault bit; the other columns are the bits
    they have without it."""
    D, V = 512, 1000
    g, w, bias = _head(D, V, 3)
    h = torch.randn(40, D, generator=g).bfloat16().cuda()
    wc = w.cuda()
    b2._lib.device_faults(0)
    good = b2.ops.code_logits(h, wc, torch.tensor([5, 17]).cuda(), None, 0.0)
    z = b2.ops.code_logits(h, wc, torch.tensor([5, -1, V + 3, 17]).cuda(), None, 0.0)
    assert b2._lib.device_faults(0) == 16  # BASAL200_FAULT_BAD_ID
    assert torch.isnan(z[:, 1]).all() and torch.isnan(z[:, 2]).all()
    assert torch.equal(z[:, 0], good[:, 0]) and torch.equal(z[:, 3], good[:, 1])


def test_tensor_core_c5_readout(b2):
    """C5's readout shape: 4096 prompts, 8 options, D = 2560 (32 prompt tiles x 1 code tile x 8 slices)."""
    D, V = 2560, 151936
    g = torch.Generator().manual_seed(21)
    w = (torch.randn(V, D, generator=g) * 0.02).bfloat16()
    h = torch.randn(4096, D, generator=g).bfloat16()
    ids = torch.randperm(V, generator=g)[:8]
    z = b2.ops.code_logits(h.cuda(), w.cuda(), ids.cuda(), None, 0.0).cpu().numpy()
    ref = oro.logits(h.float().numpy(), (w[ids].float().numpy(), None), None)
    assert np.abs(z - ref).max() <= 1e-5
    assert b2._lib.device_faults(0) == 0

