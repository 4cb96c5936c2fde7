"""The config-5 hybrid classifier's forward on the CPU, in numpy -- TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

The layer maths of the reference's Qwen 3.5 graph forward (basal/gdn_graph.py:122-140 norms, MLP, Gated DeltaNet
input; :432-451 gated norm, output, rotary embedding; :452-466 attention input and output; :559-604 a Gated DeltaNet
layer and an attention layer with a prefix; :607-620 the layer loop) with every F.linear replaced by the FP8-block
linear of oracle.blockquant (the reference's CPU maths, basal/blockquant.py:54-60, :118-123), and the gated delta rule
in its per-token definition (transformers' torch_recurrent_gated_delta_rule, which the reference runs on the CPU,
basal/gdn_graph.py:492-493): per head, S <- e^{g_t} S; S <- S + k_t (beta_t (v_t - S^T k_t))^T; o_t = S^T q_t.

bf16 tensors are fp32 arrays holding bf16 values; `bf16()` rounds to nearest even where the reference's bf16 ops
round (each torch op on bf16 computes in fp32 and rounds its result). Every function takes the rounding `rnd`: bf16
(a bf16 model) or `exact` (a float32 model: no rounding; how the reference's own forward is pinned, in fp32). The
weights are a dict: "embed", "head", "final_norm", "layers" (one dict per layer, keys as basal_b200.hybrid's); a
linear is either FP8-block (codes uint8 [N, K], scales fp32 [N / 128, K / 128]) or a plain fp32 weight [N, K].
"""
import numpy as np

from . import blockquant as obq


def bf16(x):
    """fp32 -> the nearest bf16 value (ties to even), as fp32."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    r = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + r) & np.uint32(0xFFFF0000)).view(np.float32)


def exact(x):
    return np.asarray(x, np.float32)


def rms(x, w, eps, rnd):
    """Qwen3_5RMSNorm: fp32 inside, weight as 1 + w, rounded out (basal/gdn_graph.py:122-126)."""
    h = x * (1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + np.float32(eps)))
    return rnd(h.astype(np.float32) * (np.float32(1.0) + w))


def linear(x, w, rnd):
    """An FP8-block linear (w = (codes, scales)) or a plain one (w [N, K] fp32), rounded out."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]).astype(np.float32)
    if isinstance(w, tuple):
        y = obq.linear(x2, w[0], w[1], "fp8")
        n = w[0].shape[0]
    else:
        y = x2 @ w.T
        n = w.shape[0]
    return rnd(y).reshape(*shape[:-1], n)


def silu(x):
    return x / (np.float32(1.0) + np.exp(-x))


def sigmoid(x):
    return np.float32(1.0) / (np.float32(1.0) + np.exp(-x))


def softplus(x):
    """torch's softplus (beta 1, threshold 20)."""
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0)))).astype(np.float32)


def mlp(L, h, eps, rnd):
    """h + down(silu(gate) * up)(rms(h)), each op rounded to bf16 (basal/gdn_graph.py:127-128)."""
    x = rms(h, L["mlp_nw"], eps, rnd)
    gu = linear(x, L["gate_up"], rnd)
    I = gu.shape[-1] // 2
    a = rnd(rnd(silu(gu[..., :I])) * gu[..., I:])
    return rnd(h + linear(a, L["down"], rnd))


def delta_rule(q, k, v, g, beta, s0):
    """Per token, per head (fp32): q, k [T, H, dk] (l2-normed, q scaled), v [T, H, dv], g, beta [T, H], s0 [H, dk, dv]
    -> (o [T, H, dv], final state)."""
    S = s0.astype(np.float32).copy()
    o = np.empty(v.shape, np.float32)
    for t in range(q.shape[0]):
        S *= np.exp(g[t])[:, None, None]
        mem = np.einsum("hk,hkv->hv", k[t], S)
        delta = (v[t] - mem) * beta[t][:, None]
        S += k[t][:, :, None] * delta[:, None, :]
        o[t] = np.einsum("hk,hkv->hv", q[t], S)
    return o, S


def gdn(L, cfg, h, s0, tail0, rnd):
    """One Gated DeltaNet layer on one row h [T, D] from state s0 and convolution inputs tail0 [k - 1, C] ->
    (h, state, last convolution inputs) (basal/gdn_graph.py:131-140, :559-576, :432-439)."""
    T = h.shape[0]
    x = rms(h, L["nw"], cfg.eps, rnd)
    sizes = np.cumsum(cfg.in_sizes)[:-1]
    qkv, z, b, a, _ = np.split(linear(x, L["w_in"], rnd), sizes, -1)
    beta = rnd(sigmoid(b))
    g = -np.exp(L["A_log"]) * softplus(a + L["dt_bias"])
    xin = np.concatenate([tail0, qkv], 0)
    w = L["conv"]  # [C, k]
    acc = xin[0:T] * w[:, 0]
    for j in range(1, w.shape[1]):
        acc = acc + xin[j:j + T] * w[:, j]
    y = rnd(silu(acc.astype(np.float32)))
    kd, vd = cfg.key_dim, cfg.value_dim
    q, k, v = y[:, :kd], y[:, kd:2 * kd], y[:, 2 * kd:]
    r = cfg.lin_v_heads // cfg.lin_k_heads
    q = np.repeat(q.reshape(T, cfg.lin_k_heads, cfg.lin_k_dim), r, 1)
    k = np.repeat(k.reshape(T, cfg.lin_k_heads, cfg.lin_k_dim), r, 1)
    v = v.reshape(T, cfg.lin_v_heads, cfg.lin_v_dim)
    q = q / np.sqrt((q * q).sum(-1, keepdims=True) + np.float32(1e-6)) * np.float32(1.0 / np.sqrt(cfg.lin_k_dim))
    k = k / np.sqrt((k * k).sum(-1, keepdims=True) + np.float32(1e-6))
    o, S = delta_rule(q.astype(np.float32), k.astype(np.float32), v, g.astype(np.float32), beta, s0)
    o = rnd(o)
    on = rnd(o / np.sqrt((o * o).mean(-1, keepdims=True) + np.float32(cfg.eps)))
    on = rnd(L["gnorm"] * on)
    on = rnd(on * silu(z.reshape(T, cfg.lin_v_heads, cfg.lin_v_dim)))
    return rnd(h + linear(on.reshape(T, -1), L["out"], rnd)), S, xin[T:]


def rope_tables(cfg, pos, rnd):
    r = cfg.rotary_dims
    inv = (1.0 / (cfg.rope_theta ** (np.arange(0, r, 2, dtype=np.float32) / np.float32(r)))).astype(np.float32)
    f = pos.astype(np.float32)[:, None] * inv
    emb = np.concatenate([f, f], -1)
    return rnd(np.cos(emb)), rnd(np.sin(emb))


def rope(x, cos, sin, r, rnd):
    """x [heads, T, d]: the first r dims rotated (half split), bf16 ops (basal/gdn_graph.py:446-451)."""
    xr = x[..., :r]
    rot = np.concatenate([-xr[..., r // 2:], xr[..., : r // 2]], -1)
    return np.concatenate([rnd(rnd(xr * cos) + rnd(rot * sin)), x[..., r:]], -1)


def attention(L, cfg, h, pos, pk, pv, rnd):
    """One attention layer on one row h [T, D] at positions pos over the prefix keys / values pk, pv [Hk, P, d] (or
    None) and its own tokens, causally -> (h, keys, values) (basal/gdn_graph.py:452-466, :578-604)."""
    T = h.shape[0]
    H, Hk, d = cfg.heads, cfg.kv_heads, cfg.head_dim
    x = rms(h, L["nw"], cfg.eps, rnd)
    sizes = np.cumsum(cfg.qkv_sizes)[:-1]
    qg, k, v = np.split(linear(x, L["w_qkv"], rnd), sizes, -1)
    qg = qg.reshape(T, H, 2 * d)
    q, gate = qg[..., :d], qg[..., d:]
    cos, sin = rope_tables(cfg, pos, rnd)
    q = rope(rms(q, L["q_norm"], cfg.eps, rnd).transpose(1, 0, 2), cos, sin, cfg.rotary_dims, rnd)
    k = rope(rms(k.reshape(T, Hk, d), L["k_norm"], cfg.eps, rnd).transpose(1, 0, 2), cos, sin, cfg.rotary_dims, rnd)
    v = v.reshape(T, Hk, d).transpose(1, 0, 2)
    P = 0 if pk is None else pk.shape[1]
    kk = k if pk is None else np.concatenate([pk, k], 1)
    vv = v if pv is None else np.concatenate([pv, v], 1)
    allow = np.concatenate([np.ones((T, P), bool), np.tril(np.ones((T, T), bool))], 1)
    G = H // Hk
    o = np.empty((H, T, d), np.float32)
    for hh in range(H):
        s = (q[hh] @ kk[hh // G].T) * np.float32(1.0 / np.sqrt(d))
        s = np.where(allow, s, -np.inf)
        p = np.exp(s - s.max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True)
        o[hh] = p @ vv[hh // G]
    o = rnd(o).transpose(1, 0, 2).reshape(T, H * d)
    a = rnd(o * rnd(sigmoid(gate.reshape(T, H * d))))
    return rnd(h + linear(a, L["o"], rnd)), k, v


def layers(W, cfg, ids, pos, st, rnd=bf16):
    """The layer loop (basal/gdn_graph.py:607-620) over one row -> (h, per attention layer (K, V), per Gated
    DeltaNet layer (state, tail))."""
    h = W["embed"][ids]
    kv, states = [], []
    ia = ig = 0
    for L in W["layers"]:
        if L["kind"] == "linear_attention":
            if st is None:
                s0 = np.zeros((cfg.lin_v_heads, cfg.lin_k_dim, cfg.lin_v_dim), np.float32)
                c0 = np.zeros((cfg.conv - 1, cfg.conv_dim), np.float32)
            else:
                s0, c0 = st["states"][ig]
            h, s, tail = gdn(L, cfg, h, s0, c0, rnd)
            states.append((s, tail))
            ig += 1
        else:
            pk, pv = (None, None) if st is None else st["kv"][ia]
            h, k, v = attention(L, cfg, h, pos, pk, pv, rnd)
            kv.append((k, v))
            ia += 1
        h = mlp(L, h, cfg.eps, rnd)
    return h, kv, states


def prefix(W, cfg, ids, rnd=bf16):
    """The shared prefix ids [P] -> (final-normed hidden states [P, D], its state: keys / values, recurrent states
    and convolution tails)."""
    h, kv, states = layers(W, cfg, np.asarray(ids), np.arange(len(ids)), None, rnd)
    return rms(h, W["final_norm"], cfg.eps, rnd), {"length": len(ids), "kv": kv, "states": states}


def suffix(W, cfg, st, ids, rnd=bf16):
    """One request's suffix ids [S] after the prefix st -> its final-normed hidden states [S, D]."""
    ids = np.asarray(ids)
    pos = np.arange(st["length"], st["length"] + len(ids))
    h, _, _ = layers(W, cfg, ids, pos, st, rnd)
    return rms(h, W["final_norm"], cfg.eps, rnd)


def decide(W, cfg, st, ids, option_ids, rnd=bf16):
    """One request's suffix ids [S] after the prefix st -> (final-normed hidden state of its last token [D],
    probabilities over option_ids: the fp32 readout of basal/readout.py:71-79)."""
    hl = suffix(W, cfg, st, ids, rnd)[-1]
    z = W["head"][np.asarray(option_ids)] @ hl
    p = np.exp(z - z.max())
    return hl, p / p.sum()
