"""The config-5 oracle (oracle/hybrid.py) pinned to the reference's own Qwen 3.5 graph forward: tests/golden/hybrid.npz
holds Qwen35Graph's outputs (basal/gdn_graph.py:622-656: the prefix pass from position 0 and the suffix pass that
continues its keys, values, recurrent states and convolution tails) for a tiny float32 model, written by
tests/golden/make_golden_hybrid.py. The oracle, run in float32 (no bf16 rounding) on the same weights and ids, must
give the same hidden states to fp32 rounding (its delta rule is the per-token definition, the reference's the
chunked form). Also: the bf16 rounding helper against torch's cast. No GPU."""
import importlib.util
import os

import numpy as np
import pytest
import torch

import torch.nn.functional as F

from conftest import GOLDEN, golden
from oracle import hybrid as ohy


def l2norm(x, eps=1e-6):
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def chunk_delta_rule(q, k, v, g, beta, s0, chunk):
    """The gated delta rule over chunks in plain torch (fp32; the chunked form the CUDA kernel basal::gdn_chunk_rule
    computes): q, k [b, H, T, dk], v [b, H, T, dv], g, beta [b, H, T], s0 [b or 1, H, dk, dv] -> (o [b, H, Tp, dv],
    the final state), Tp = T rounded up to whole chunks. Within a chunk with cumulative gates G, the rows' updates
    solve the unit lower-triangular system (I + A), A_ij = beta_i (k_i . k_j) e^{G_i - G_j} for j < i."""
    b, H, T, dk = k.shape
    dv = v.shape[-1]
    pad = -T % chunk
    if pad:
        q, k, v = (F.pad(t, (0, 0, 0, pad)) for t in (q, k, v))
        g, beta = F.pad(g, (0, pad)), F.pad(beta, (0, pad))
    n = (T + pad) // chunk
    q, k, v = (t.reshape(b, H, n, chunk, -1) for t in (q, k, v))
    G = g.reshape(b, H, n, chunk).cumsum(-1)
    beta = beta.reshape(b, H, n, chunk)
    low = torch.ones(chunk, chunk, dtype=torch.bool, device=q.device).tril(-1)
    both = torch.ones(chunk, chunk, dtype=torch.bool, device=q.device).tril(0)
    diff = (G[..., :, None] - G[..., None, :]).masked_fill(~both, 0.0).exp().masked_fill(~both, 0.0)
    A = (beta[..., None] * (k @ k.transpose(-1, -2)) * diff).masked_fill(~low, 0.0)
    eye = torch.eye(chunk, dtype=q.dtype, device=q.device)
    Tinv = torch.linalg.solve_triangular(A + eye, eye.expand_as(A), upper=False, unitriangular=True)
    U = Tinv @ (beta[..., None] * v)
    W = Tinv @ (beta[..., None] * G.exp()[..., None] * k)
    qk = (q @ k.transpose(-1, -2)) * diff
    qg = q * G.exp()[..., None]
    kd = k * (G[..., -1:] - G).exp()[..., None]
    S = s0.expand(b, H, dk, dv).contiguous()
    out = torch.empty(b, H, n, chunk, dv, dtype=q.dtype, device=q.device)
    for c in range(n):
        vn = U[:, :, c] - W[:, :, c] @ S
        out[:, :, c] = qg[:, :, c] @ S + qk[:, :, c] @ vn
        S = G[:, :, c, -1, None, None].exp() * S + kd[:, :, c].transpose(-1, -2) @ vn
    return out.reshape(b, H, n * chunk, dv), S


def sizes():
    spec = importlib.util.spec_from_file_location("make_golden_hybrid", os.path.join(GOLDEN, "make_golden_hybrid.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.SIZES


@pytest.fixture(scope="module")
def fixture():
    from basal_b200.hybrid import HybridConfig
    g = golden("hybrid")
    cfg = HybridConfig(**sizes())
    W = {"embed": g["embed"], "head": g["head"], "final_norm": g["final_norm"], "layers": []}
    for i, kind in enumerate(cfg.kinds):
        L = {"kind": kind}
        for k in g:
            if k.startswith(f"l{i}."):
                L[k.split(".", 1)[1]] = g[k]
        W["layers"].append(L)
    return cfg, W, g


def test_oracle_equals_the_reference_graph_forward(fixture):
    cfg, W, g = fixture
    h1, st = ohy.prefix(W, cfg, g["prefix_ids"], rnd=ohy.exact)
    ref1 = g["prefix_hidden"]
    assert np.abs(h1 - ref1).max() <= 1e-5 * np.abs(ref1).max(), np.abs(h1 - ref1).max()
    for r in range(2):
        h2 = ohy.suffix(W, cfg, st, g["suffix_ids"][r], rnd=ohy.exact)
        ref2 = g["suffix_hidden"][r]
        assert np.abs(h2 - ref2).max() <= 1e-5 * np.abs(ref2).max(), (r, np.abs(h2 - ref2).max())


def test_bf16_rounding_equals_torch():
    x = torch.randn(1 << 16) * torch.logspace(-30, 30, 1 << 16)
    x[:4] = torch.tensor([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -(1.0 + 2 ** -8), 0.0])  # ties to even, both ways
    want = x.to(torch.bfloat16).float().numpy()
    assert np.array_equal(ohy.bf16(x.numpy()), want)


@pytest.mark.parametrize("T, chunk", [(150, 64), (64, 64), (5, 64), (130, 32)])
def test_chunked_delta_rule_equals_the_per_token_definition(T, chunk):
    """The chunked form (chunk_delta_rule above, the algorithm of the CUDA kernel basal::gdn_chunk_rule) against
    oracle.hybrid.delta_rule (the per-token definition), from a non-zero initial state, with ragged last chunks."""
    g = torch.Generator().manual_seed(T)
    b, H, dk, dv = 2, 3, 16, 8
    q = l2norm(torch.randn(b, H, T, dk, generator=g)) * dk ** -0.5
    k = l2norm(torch.randn(b, H, T, dk, generator=g))
    v = torch.randn(b, H, T, dv, generator=g)
    gl = -torch.rand(b, H, T, generator=g)
    beta = torch.rand(b, H, T, generator=g)
    s0 = torch.randn(1, H, dk, dv, generator=g) * 0.1
    o, S = chunk_delta_rule(q, k, v, gl, beta, s0, chunk)
    assert o.shape[2] == -(-T // chunk) * chunk  # whole chunks; the rows past T are padding
    o = o[:, :, :T]
    for i in range(b):
        t = lambda x: x[i].transpose(0, 1).numpy()  # noqa: E731
        oo, SS = ohy.delta_rule(t(q), t(k), t(v), gl[i].T.numpy(), beta[i].T.numpy(), s0[0].numpy())
        assert np.abs(o[i].transpose(0, 1).numpy() - oo).max() < 1e-5
        assert np.abs(S[i].numpy() - SS).max() < 1e-5
