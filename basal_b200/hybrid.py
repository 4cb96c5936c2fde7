"""The config-5 classifier: a random-init Gated-DeltaNet / attention hybrid decoder (the layer maths of the reference's
Qwen 3.5 graph forward, basal/gdn_graph.py:122-603, and of transformers' Qwen3_5 modules) whose every linear is an
FP8-block BlockFP8Linear of this package, answering decision requests with the option-code readout.

  HybridConfig          the sizes (C5: 32 layers, 3 Gated DeltaNet : 1 attention, hidden 2560, 16 query / 4 key-value
                        heads of 128, SwiGLU 9728, vocab 151,936; the Gated DeltaNet sizes are transformers'
                        Qwen3_5TextConfig defaults: 16 key / 32 value heads of 128, convolution 4)
  HybridClassifier      random-init weights (seeded, on one GPU), quantised to FP8 blocks at build time
      .prefix(ids)      the shared prefix [P] from position 0 -> PrefixState (per attention layer its keys and values,
                        per Gated DeltaNet layer its recurrent state and convolution tail), computed once per GPU
      .suffix_hidden(ids, st)   rows [B, S] that continue the prefix -> the final-normed hidden state of each row's
                        last token [B, D]
      .decide(ids, st, readout, rows, idx, pad)   -> option probabilities [B, k]

The linears are basal::fp8_block_linear (the projections that read one input merged into one weight, as
blockquant.fuse does for the reference: the Gated DeltaNet's q/k/v/z/b/a, the attention's q+gate/k/v), the gated MLP
input basal::fp8_block_linear_glu (SwiGLU in the GEMM's epilogue) and the output projections
basal::fp8_block_linear_residual (the residual add in the GEMM's epilogue). The norms, the convolution, the gates and
the rotary embedding follow the reference's roundings (bf16 between operations, fp32 inside the norms); the
recurrence runs in fp32 over chunks of 64 tokens (basal::gdn_chunk_rule); the attention over the prefix and the rows'
own tokens is torch's scaled_dot_product_attention. Everything runs on the GPU.
"""
import dataclasses
import math

import torch
import torch.nn.functional as F

from . import ops
from .fp8block import BlockFP8Linear

LINEAR, FULL = "linear_attention", "full_attention"


@dataclasses.dataclass(frozen=True)
class HybridConfig:
    layers: int = 32
    hidden: int = 2560
    heads: int = 16
    kv_heads: int = 4
    head_dim: int = 128
    inter: int = 9728
    vocab: int = 151936
    lin_k_heads: int = 16
    lin_v_heads: int = 32
    lin_k_dim: int = 128
    lin_v_dim: int = 128
    conv: int = 4
    full_every: int = 4          # every 4th layer is full attention (3 : 1)
    eps: float = 1e-6
    rotary_frac: float = 0.25    # partial rotary: the first 32 of 128 dimensions of a head
    rope_theta: float = 10000.0

    @property
    def kinds(self):
        return [FULL if (i + 1) % self.full_every == 0 else LINEAR for i in range(self.layers)]

    @property
    def key_dim(self):
        return self.lin_k_heads * self.lin_k_dim

    @property
    def value_dim(self):
        return self.lin_v_heads * self.lin_v_dim

    @property
    def conv_dim(self):
        return 2 * self.key_dim + self.value_dim

    @property
    def in_sizes(self):
        """The merged Gated DeltaNet input projection's parts: q/k/v, z, b, a, and zero rows up to whole 128-row
        blocks (b and a have one row per value head)."""
        used = self.conv_dim + self.value_dim + 2 * self.lin_v_heads
        return (self.conv_dim, self.value_dim, self.lin_v_heads, self.lin_v_heads, -used % 128)

    @property
    def qkv_sizes(self):
        return (2 * self.heads * self.head_dim, self.kv_heads * self.head_dim, self.kv_heads * self.head_dim)

    @property
    def rotary_dims(self):
        return int(self.head_dim * self.rotary_frac)


C5 = HybridConfig()


def rms(x, w, eps):
    """Qwen3_5RMSNorm (weight stored as w, applied as 1 + w), fp32 inside, x's dtype out (basal/gdn_graph.py:122-126)."""
    h = x.float()
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return (h * (1.0 + w.float())).to(x.dtype)


def rope_tables(cfg, pos, dtype):
    """cos, sin [b, T, r] of positions pos [b, T] (fp32 maths, then dtype, as the rotary embedding module returns)."""
    r = cfg.rotary_dims
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, r, 2, device=pos.device, dtype=torch.float32) / r))
    f = pos.float()[..., None] * inv
    emb = torch.cat([f, f], -1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


@dataclasses.dataclass
class PrefixState:
    """What the rows continue: per attention layer (K, V) [1, kv heads, P, d] bf16; per Gated DeltaNet layer the
    recurrent state [1, value heads, dk, dv] fp32 and the convolution's last inputs [1, k - 1, channels] bf16."""
    length: int
    kv: list
    states: list
    buffers: dict = dataclasses.field(default_factory=dict)

    def kv_buffers(self, i, b, T):
        """Key and value buffers [b, kv heads, P + T, d] of attention layer i whose first P positions hold the prefix's
        keys and values (copied once, kept for later rows): the rows' own T positions are written into them."""
        kb, vb = self.buffers.get((i, T), (None, None))
        if kb is None or kb.shape[0] < b:
            pk, pv = self.kv[i]
            P = self.length
            kb = pk.new_empty(b, pk.shape[1], P + T, pk.shape[3])
            vb = pv.new_empty(b, pv.shape[1], P + T, pv.shape[3])
            kb[:, :, :P].copy_(pk.expand(b, -1, -1, -1))
            vb[:, :, :P].copy_(pv.expand(b, -1, -1, -1))
            self.buffers[(i, T)] = kb, vb
        return kb[:b], vb[:b]


class HybridClassifier:
    """The C5 hybrid with random weights (generator `seed`) on `device`; every linear FP8-block quantised."""

    def __init__(self, cfg=C5, device="cuda", seed=0, dtype=torch.bfloat16, residual_std=None):
        if cfg.head_dim != 128 or cfg.lin_k_dim != 128 or cfg.lin_v_dim != 128:
            raise ValueError("the attention and Gated DeltaNet kernels of this build take heads of 128")
        self.cfg, self.dtype = cfg, dtype
        dev = torch.device(device)
        self.device = dev
        g = torch.Generator(device=dev).manual_seed(seed)

        def normal(*shape, std=0.02):
            return torch.randn(*shape, device=dev, generator=g) * std

        def fp8(n, k, std=0.02):
            lin = torch.nn.Linear(k, n, bias=False, device=dev)
            with torch.no_grad():
                lin.weight.copy_(normal(n, k, std=std))
            return BlockFP8Linear.of(lin)

        D = cfg.hidden
        # GPT-2's scaled initialisation: unit-variance embeddings, the linears N(0, 0.02) and the projections that
        # write into the residual stream N(0, 0.02 / sqrt(2 * layers)). With N(0, 0.02) everywhere the random model is
        # chaotic: a one-ulp change of 1% of the embedding values moves the last hidden state by 7-28% (8-32 layers),
        # so no two correct implementations would agree on a decision; with this one it moves it by 0.25%.
        out_std = residual_std if residual_std is not None else 0.02 / math.sqrt(2 * cfg.layers)
        self.embed = normal(cfg.vocab, D, std=1.0).to(dtype)
        self.head = torch.nn.Linear(D, cfg.vocab, bias=False, device=dev, dtype=dtype)
        with torch.no_grad():
            self.head.weight.copy_(normal(cfg.vocab, D))
        self.final_norm = normal(D).to(dtype)
        self.layers = []
        for kind in cfg.kinds:
            L = dict(kind=kind, nw=normal(D).to(dtype), mlp_nw=normal(D).to(dtype),
                     gate_up=fp8(2 * cfg.inter, D), down=fp8(D, cfg.inter, out_std))
            if kind == LINEAR:
                L["w_in"] = fp8(sum(cfg.in_sizes), D)
                L["conv"] = (torch.rand(cfg.conv_dim, cfg.conv, device=dev, generator=g) - 0.5).to(dtype)
                L["A_log"] = torch.log(1.0 + 15.0 * torch.rand(cfg.lin_v_heads, device=dev, generator=g))
                L["dt_bias"] = (1.0 + normal(cfg.lin_v_heads, std=0.1)).to(dtype)
                L["gnorm"] = (1.0 + normal(cfg.lin_v_dim, std=0.1)).to(dtype)
                L["out"] = fp8(D, cfg.value_dim, out_std)
            else:
                L["w_qkv"] = fp8(sum(cfg.qkv_sizes), D)
                L["q_norm"] = normal(cfg.head_dim).to(dtype)
                L["k_norm"] = normal(cfg.head_dim).to(dtype)
                L["o"] = fp8(D, cfg.heads * cfg.head_dim, out_std)
            self.layers.append(L)

    # -------------------------------------------------------------------------------------------------------------
    def _mlp(self, L, h):
        """h + down(silu(gate) * up)(rms(h)) (basal/gdn_graph.py:127-128): the norm fused with the gate/up GEMM's
        activation quantiser, the gated product in that GEMM's epilogue, the residual add in the down GEMM's."""
        b, T, D = h.shape
        q, s = ops.rms_norm_fp8_quant(h.reshape(-1, D), L["mlp_nw"], self.cfg.eps)
        gu = L["gate_up"]
        a = ops.fp8_block_gemm_glu(q, s, gu.weight, gu.weight_scale, "silu", h.dtype)
        return L["down"].forward_residual(a, h.reshape(-1, D)).view(b, T, D)

    def _gdn(self, L, h, s0, tail0):
        """h + Gated DeltaNet(rms(h)) continuing state s0 / convolution inputs tail0 (basal/gdn_graph.py:131-140,
        :559-576, :432-439) -> (h, final state, last convolution inputs). The norm is fused with the input
        projection's quantiser; the convolution, SiLU, l2 norms and gates are one kernel (basal::gdn_prep); the
        recurrence runs over chunks; the gated output norm is fused with the output projection's quantiser, and the
        residual add is in that GEMM's epilogue."""
        cfg = self.cfg
        b, T, D = h.shape
        h2 = h.reshape(-1, D)
        q8, s8 = ops.rms_norm_fp8_quant(h2, L["nw"], cfg.eps)
        w_in = L["w_in"]
        proj = ops.fp8_block_gemm(q8, s8, w_in.weight, w_in.weight_scale, h.dtype)  # [b * T, in_sizes]
        C, z_off = cfg.conv_dim, cfg.conv_dim
        b_off, a_off = C + cfg.value_dim, C + cfg.value_dim + cfg.lin_v_heads
        q, k, v, beta, g = ops.gdn_prep(proj, tail0, L["conv"], L["A_log"], L["dt_bias"], b, T, cfg.lin_k_heads,
                                        cfg.lin_v_heads, b_off, a_off)
        o, s = ops.gdn_chunk_rule(q, k, v, g, beta, s0, True)  # o in the projection's type, as the norm rounds it
        qo, so = ops.gdn_gate_fp8_quant(o, proj, z_off, L["gnorm"], cfg.eps, b, T)
        out = L["out"]
        h = ops.fp8_block_gemm_residual(qo, so, out.weight, out.weight_scale, None, h2).view(b, T, D)
        n = cfg.conv - 1  # the convolution inputs the next tokens would continue from
        qkv = proj.view(b, T, -1)[..., :C]
        tail = qkv[:, T - n:] if T >= n else torch.cat([tail0.expand(b, -1, -1), qkv], 1)[:, -n:]
        return h, s, tail.contiguous()

    def _attention(self, L, h, cos, sin, pk, pv, bufs=None):
        """h + attention(rms(h)) over the prefix keys / values pk, pv [1, kv heads, P, d] (or none) and the rows'
        own tokens, causally (basal/gdn_graph.py:452-466, :578-604) -> (h, the rows' keys, values). The norms and rotary
        embedding are one kernel (basal::attn_prep), which writes the rows' keys and values after the prefix's into
        bufs (PrefixState.kv_buffers, [b, kv heads, P + T, d], the prefix's already there) or into new buffers; the
        output gate is fused with the output projection's quantiser, the residual add is in that GEMM's epilogue."""
        cfg = self.cfg
        b, T, D = h.shape
        H, Hk, d = cfg.heads, cfg.kv_heads, cfg.head_dim
        q8, s8 = ops.rms_norm_fp8_quant(h.reshape(-1, D), L["nw"], cfg.eps)
        w = L["w_qkv"]
        qkv = ops.fp8_block_gemm(q8, s8, w.weight, w.weight_scale, h.dtype)  # [b * T, (q, gate) * H | k | v]
        P = 0 if pk is None else pk.shape[2]
        if P and bufs is not None:
            kk, vv = bufs
        else:
            kk, vv = h.new_empty(b, Hk, P + T, d), h.new_empty(b, Hk, P + T, d)
            if P:
                kk[:, :, :P].copy_(pk.expand(b, -1, -1, -1))
                vv[:, :, :P].copy_(pv.expand(b, -1, -1, -1))
        # the q / k norms and rotary embedding, the rows' keys and values written after the prefix's
        q = ops.attn_prep(qkv, L["q_norm"], L["k_norm"], cfg.eps, cos, sin, cfg.rotary_dims, H, Hk, b, T, kk, vv, P)
        G = H // Hk
        own = torch.ones(T, T, dtype=torch.bool, device=h.device).tril()
        allow = torch.cat([torch.ones(T, P, dtype=torch.bool, device=h.device), own], 1)
        allow = allow[None, None, None].expand(1, 1, G, T, P + T).reshape(1, 1, G * T, P + T)
        o = F.scaled_dot_product_attention(q.reshape(b, Hk, G * T, d), kk, vv, attn_mask=allow,
                                           scale=1.0 / math.sqrt(d)).reshape(b, H, T, d)
        qa, sa = ops.attn_gate_fp8_quant(o, qkv, b, T, H)  # o * sigmoid(gate), quantised for the output projection
        out = L["o"]
        h = ops.fp8_block_gemm_residual(qa, sa, out.weight, out.weight_scale, out.bias, h.reshape(-1, D))
        return h.view(b, T, D), kk[:, :, P:], vv[:, :, P:]

    def _layers(self, ids, pos, st):
        cfg = self.cfg
        h = self.embed[ids]
        cos, sin = rope_tables(cfg, pos, h.dtype)
        kv, states = [], []
        ia = ig = 0
        for L in self.layers:
            if L["kind"] == LINEAR:
                if st is None:
                    s0 = torch.zeros(1, cfg.lin_v_heads, cfg.lin_k_dim, cfg.lin_v_dim, device=h.device)
                    c0 = torch.zeros(1, cfg.conv - 1, cfg.conv_dim, dtype=h.dtype, device=h.device)
                else:
                    s0, c0 = st.states[ig]
                h, s, tail = self._gdn(L, h, s0, c0)
                states.append((s, tail))
                ig += 1
            else:
                pk, pv = (None, None) if st is None else st.kv[ia]
                bufs = None if st is None else st.kv_buffers(ia, h.shape[0], h.shape[1])
                h, k, v = self._attention(L, h, cos, sin, pk, pv, bufs)
                kv.append((k, v))
                ia += 1
            h = self._mlp(L, h)
        return h, kv, states

    @torch.no_grad()
    def prefix(self, ids):
        """The shared prefix ids [P] from position 0 -> PrefixState (its keys, values, states, tails)."""
        ids = ids.reshape(1, -1).to(self.device)
        P = ids.shape[1]
        pos = torch.arange(P, device=self.device)[None]
        _, kv, states = self._layers(ids, pos, None)
        return PrefixState(P, kv, states)

    @torch.no_grad()
    def suffix_hidden(self, ids, st):
        """Rows ids [B, S] at positions P .. P + S - 1 after the prefix st -> final-normed hidden state of each row's
        last token [B, D]."""
        B, S = ids.shape
        pos = torch.arange(st.length, st.length + S, device=self.device)[None].expand(B, S)
        h, _, _ = self._layers(ids.to(self.device), pos, st)
        return rms(h[:, -1], self.final_norm, self.cfg.eps)

    @torch.no_grad()
    def decide(self, ids, st, readout, rows, idx, pad):
        """Option probabilities [B, k] of the rows' last tokens: the readout of readout.rows(...) = rows, idx, pad."""
        return readout.device_probs(self.suffix_hidden(ids, st), rows, idx, pad)

    def linears(self):
        """Every FP8-block linear of the model, with its name."""
        for i, L in enumerate(self.layers):
            for name, m in L.items():
                if isinstance(m, BlockFP8Linear):
                    yield f"layers.{i}.{name}", m

    def flops_per_token(self):
        """2 x the FP8 weights' multiply-adds a token (the linears; the recurrence, attention and readout excluded)."""
        return sum(2 * m.in_features * m.out_features for _, m in self.linears())
