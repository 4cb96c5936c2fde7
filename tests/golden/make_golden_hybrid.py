"""Writes tests/golden/hybrid.npz from the reference itself (rkinas/basal 2.8.1, imported read-only): the Qwen 3.5
graph forward (basal/gdn_graph.py:469-734, Qwen35Graph) of a tiny random transformers Qwen3_5 model in float32 on
the CPU, whose Gated DeltaNet layers run transformers' torch_chunk_gated_delta_rule (the reference's CPU path,
basal/gdn_graph.py:492-493):

    PYTHONPATH=<reference checkout> python tests/golden/make_golden_hybrid.py

  pass 1  Qwen35Graph.forward(prefix ids [1, P], lens, kv, st): the prefix's final-normed hidden states, and the
          buffers of its keys / values and recurrent states / convolution tails (:622-634)
  pass 2  Qwen35Graph.forward_suffix(rows [2, S] at positions P .., unit 0, plen P, kv, st): the rows' final-normed
          hidden states, each continuing the prefix (:636-656)
The model has 4 layers (3 Gated DeltaNet : 1 attention, the C5 pattern), 2 key / 4 value heads (so the keys repeat),
a partial rotary embedding, and norm weights moved off their initial values, so that every weight takes part. The
arrays hold the weights in the layout of oracle/hybrid.py (merged projections, zero rows to whole 128-row blocks),
the ids and both passes' outputs.
"""
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
SIZES = dict(layers=4, hidden=32, heads=2, kv_heads=1, head_dim=16, inter=64, vocab=64, lin_k_heads=2,
             lin_v_heads=4, lin_k_dim=8, lin_v_dim=8, conv=4, full_every=4, eps=1e-6, rotary_frac=0.5,
             rope_theta=10000.0)
P, S = 70, 37   # a prefix past one chunk of 64, a suffix of a partial chunk


def model():
    from transformers import Qwen3_5ForCausalLM, Qwen3_5TextConfig
    c = SIZES
    torch.manual_seed(0)
    m = Qwen3_5ForCausalLM(Qwen3_5TextConfig(
        vocab_size=c["vocab"], hidden_size=c["hidden"], intermediate_size=c["inter"], num_hidden_layers=c["layers"],
        layer_types=["linear_attention"] * 3 + ["full_attention"], num_attention_heads=c["heads"],
        num_key_value_heads=c["kv_heads"], head_dim=c["head_dim"], linear_num_key_heads=c["lin_k_heads"],
        linear_num_value_heads=c["lin_v_heads"], linear_key_head_dim=c["lin_k_dim"],
        linear_value_head_dim=c["lin_v_dim"], linear_conv_kernel_dim=c["conv"], rms_norm_eps=c["eps"],
        max_position_embeddings=256,
        rope_parameters={"rope_type": "default", "rope_theta": c["rope_theta"],
                         "partial_rotary_factor": c["rotary_frac"], "mrope_section": [2, 1, 1],
                         "mrope_interleaved": True})).eval()
    g = torch.Generator().manual_seed(1)
    with torch.no_grad():
        for name, p in m.named_parameters():
            if "norm" in name:  # (zeros / ones at init: move them so that their maths shows)
                p.add_(torch.randn(p.shape, generator=g) * 0.1)
            if name.endswith("dt_bias"):
                p.add_(torch.randn(p.shape, generator=g) * 0.2)
    return m


def export(m):
    """The weights in oracle/hybrid.py's layout (fp32 arrays)."""
    f = lambda t: t.detach().float().numpy().copy()  # noqa: E731
    out = {"embed": f(m.model.embed_tokens.weight), "head": f(m.lm_head.weight), "final_norm": f(m.model.norm.weight)}
    for i, lay in enumerate(m.model.layers):
        p = f"l{i}."
        out[p + "nw"] = f(lay.input_layernorm.weight)
        out[p + "mlp_nw"] = f(lay.post_attention_layernorm.weight)
        out[p + "gate_up"] = np.concatenate([f(lay.mlp.gate_proj.weight), f(lay.mlp.up_proj.weight)])
        out[p + "down"] = f(lay.mlp.down_proj.weight)
        if hasattr(lay, "linear_attn"):
            a = lay.linear_attn
            w = np.concatenate([f(a.in_proj_qkv.weight), f(a.in_proj_z.weight), f(a.in_proj_b.weight),
                                f(a.in_proj_a.weight)])
            out[p + "w_in"] = np.concatenate([w, np.zeros((-w.shape[0] % 128, w.shape[1]), np.float32)])
            out[p + "conv"] = f(a.conv1d.weight)[:, 0, :]
            out[p + "A_log"], out[p + "dt_bias"] = f(a.A_log), f(a.dt_bias)
            out[p + "gnorm"], out[p + "out"] = f(a.norm.weight), f(a.out_proj.weight)
        else:
            a = lay.self_attn
            out[p + "w_qkv"] = np.concatenate([f(a.q_proj.weight), f(a.k_proj.weight), f(a.v_proj.weight)])
            out[p + "q_norm"], out[p + "k_norm"], out[p + "o"] = f(a.q_norm.weight), f(a.k_norm.weight), f(
                a.o_proj.weight)
    return out


def main():
    from basal.gdn_graph import Qwen35Graph
    m = model()
    arrays = export(m)  # before Qwen35Graph merges the projections
    g = Qwen35Graph(m, compile=False)
    gen = torch.Generator().manual_seed(2)
    pre = torch.randint(0, SIZES["vocab"], (1, P), generator=gen)
    suf = torch.randint(0, SIZES["vocab"], (2, S), generator=gen)
    kv = [(torch.zeros(1, h, P, d), torch.zeros(1, h, P, d)) for h, d in g.kv_shapes]
    st = [(torch.zeros(1, *g.state_shape), torch.zeros(1, *g.tail_shape)) for _ in range(g.n_gdn)]
    h1 = g.forward(pre, torch.tensor([P]), kv, st)
    pos = torch.arange(P, P + S)[None].expand(2, S)
    h2 = g.forward_suffix(suf, pos, torch.zeros(2, dtype=torch.long), torch.tensor([P, P]), kv, st)
    arrays.update(prefix_ids=pre[0].numpy(), suffix_ids=suf.numpy(), prefix_hidden=h1[0].numpy(),
                  suffix_hidden=h2.numpy(), sizes=np.array(list(SIZES.items()), dtype=object))
    np.savez_compressed(os.path.join(HERE, "hybrid.npz"), **{k: v for k, v in arrays.items() if k != "sizes"})
    print({k: v.shape for k, v in arrays.items() if hasattr(v, "shape")})


if __name__ == "__main__":
    main()
