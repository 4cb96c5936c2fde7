"""Writes the golden fixtures of tests/golden/ from the reference itself (rkinas/basal 2.8.1, imported read-only).

    PYTHONPATH=<reference checkout> python tests/golden/make_golden.py

Every array here is an output of the reference's own CPU functions on seeded inputs:
  blockquant.npz  BlockFormat.act_quant_ops / quantize / reference (basal/blockquant.py:54-60, :118-135) for the FP8
                  (fp8block.FORMAT) and INT8 (int8block.FORMAT) formats, and fp8block.linear / int8block.linear on the
                  CPU (fp8block.py:74-85, blockquant.py:175-183)
  nvfp4.npz       nvfp4._act_ops, swizzle, quantize, NVFP4Linear.of + forward on the CPU (basal/nvfp4.py:49-112,
                  :197-245), the code table of tests/test_nvfp4.py:13-15
  readout.npz     CodeReadout.probs / probs_each (basal/readout.py:81-104), with and without bias and soft cap
The fixtures are small (about 2.5 MB together); the GPU box has no reference checkout, so the tests read only these files.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def bf16_exact(t):
    """fp32 values that bf16 holds exactly (the CUDA path takes bf16 activations)."""
    return t.to(torch.bfloat16).float()


def u8(t):
    return t.contiguous().view(torch.uint8).numpy().copy()


def bf16_bits(t):
    """bf16-exact fp32 values stored as their 16-bit patterns (half the bytes; the tests widen them back)."""
    return t.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def act_inputs():
    """Activations with the edge cases of the quantisers: zero groups, tiny and huge groups, groups whose values sit
    on e4m3 / int8 rounding ties, mixed magnitudes within a row."""
    g = torch.Generator().manual_seed(0)
    x = torch.randn(64, 1024, generator=g)
    x[1] = 0.0                                      # an all-zero row: every scale clamps to 1e-12 / qmax
    x[2, :128] = 0.0                                # one zero group in a live row
    x[3] *= 1e-30                                   # tiny values (fp32 subnormal range after scaling)
    x[4] *= 1e4
    x[5] = torch.randn(1024, generator=g) * torch.logspace(-6, 6, 8).repeat_interleave(128)
    ties = torch.tensor([448.0, 1.5, 2.5, -3.5, 0.5, 104.0, 232.0, -240.0])  # amax 448: x / s = x exactly
    x[6, :128] = ties.repeat(16)
    x[7, :128] = torch.tensor([127.0, 0.5, 1.5, 2.5, -0.5, -1.5, 63.5, -126.5]).repeat(16)  # int8 ties at amax 127
    x[8] = -x[8].abs()                              # all negative
    x[9, 5] = 1e6                                   # one outlier per row
    return bf16_exact(x)


def make_blockquant(bq, fp8block, int8block):
    out = {}
    x = act_inputs()
    out["x_bf16"] = bf16_bits(x)
    g = torch.Generator().manual_seed(1)
    xf = torch.randn(16, 512, generator=g) * 3.0   # fp32 activations (not bf16-exact): the fp32 input path
    out["xf"] = xf.numpy()
    w = torch.randn(256, 384, generator=g) * torch.tensor([1e-3, 1.0, 50.0]).repeat_interleave(128)[None]
    out["w"] = w.numpy()
    for name, mod in (("fp8", fp8block), ("int8", int8block)):
        f = mod.FORMAT
        q, s = f.act_quant_ops(x)
        out[f"{name}_act_q"], out[f"{name}_act_s"] = u8(q), s.numpy()
        q, s = f.act_quant_ops(xf)
        out[f"{name}_actf_q"], out[f"{name}_actf_s"] = u8(q), s.numpy()
        wq, ws = f.quantize(w)
        out[f"{name}_w_q"], out[f"{name}_w_s"] = u8(wq), ws.numpy()
    # the GEMM's maths at a small shape (the GPU tests cover tests/test_fp8block.py:134-148 against this oracle): M=37, K=512, N=256
    g = torch.Generator().manual_seed(2)
    xa = bf16_exact(torch.randn(37, 512, generator=g))
    wb = bf16_exact(torch.randn(256, 512, generator=g) / 32)
    bias = torch.randn(256, generator=g)
    out["gemm_x_bf16"], out["gemm_w_bf16"], out["gemm_bias"] = bf16_bits(xa), bf16_bits(wb), bias.numpy()
    for name, mod in (("fp8", fp8block), ("int8", int8block)):
        f = mod.FORMAT
        q, s = f.quantize(wb)
        qa, sa = f.act_quant_ops(xa)
        out[f"{name}_gemm_wq"], out[f"{name}_gemm_ws"] = u8(q), s.numpy()
        out[f"{name}_gemm_y"] = bq.reference(qa, sa, q, s, torch.float32).numpy()
        out[f"{name}_linear_y"] = mod.linear(xa, q, s, bias).numpy()            # fp32 x -> fp32 y, with bias
        out[f"{name}_linear_y_bf16"] = mod.linear(xa.bfloat16(), q, s).float().numpy()  # bf16 x -> bf16 y
    return out


def make_nvfp4(nvfp4):
    out = {}
    u = torch.tensor([0, .25, .5, .75, 1, 1.25, 1.5, 1.75, 2, 2.5, 3, 3.5, 4, 5, 6, 7, -0.75, -5])
    out["table_u"], out["table_codes"] = u.numpy(), nvfp4._codes(u).numpy()
    g = torch.Generator().manual_seed(3)
    x = torch.randn(37, 512, generator=g)
    heavy = torch.rand(37, 512, generator=g) < 0.01
    x = bf16_exact(torch.where(heavy, x * 20, x))
    x[1] = 0.0
    x[2, :16] = 1e-7  # a block whose scale rounds to an e4m3 subnormal or to 0
    xg = torch.tensor([max(float(x.abs().amax()), 1e-6) * nvfp4.MARGIN / (nvfp4.FP4_MAX * nvfp4.E4M3_MAX)])
    inv_g = (1.0 / xg).float()
    out["x_bf16"], out["inv_g"] = bf16_bits(x), inv_g.numpy()
    codes, scales = nvfp4._act_ops(x, inv_g)
    out["act_codes"], out["act_scales"] = codes.numpy(), u8(scales)
    Mp = 128
    qp = torch.zeros(Mp, 256, dtype=torch.uint8)
    qp[:37] = codes
    out["act_q_padded"], out["act_s_swizzled"] = qp.numpy(), u8(nvfp4.swizzle(scales))
    s = torch.rand(300, 52, generator=torch.Generator().manual_seed(0)).mul(400).to(nvfp4.E4M3)
    out["swz_in"], out["swz_out"] = u8(s), u8(nvfp4.swizzle(s))
    for name, (n, k, std) in {"w1": (128, 512, 0.02), "w2": (300, 192, 1.0)}.items():
        w = torch.randn(n, k, generator=g) * std
        c, sc, wg = nvfp4.quantize(w)
        out[f"{name}"], out[f"{name}_codes"], out[f"{name}_scales"], out[f"{name}_g"] = \
            w.numpy(), c.numpy(), u8(sc), wg.numpy()
    torch.manual_seed(0)
    lin = torch.nn.Linear(512, 256, bias=False)
    f = nvfp4.NVFP4Linear.of(lin, x.float().abs().amax())
    out["lin_w"] = lin.weight.detach().numpy()
    out["lin_codes"], out["lin_scales"] = f.weight.detach().numpy(), u8(f.weight_scale.detach())
    out["lin_alpha"], out["lin_inv_g"] = f.alpha.detach().numpy(), f.inv_g.detach().numpy()
    out["lin_y_bf16"] = f(x.bfloat16()).float().numpy()
    out["lin_y_f32"] = nvfp4.linear(x, f.weight, f.weight_scale, f.alpha, f.inv_g).numpy()
    return out


def make_readout(readout):
    out = {}
    g = torch.Generator().manual_seed(4)
    head = torch.nn.Linear(64, 300).to(torch.bfloat16)
    with torch.no_grad():
        head.weight.copy_(torch.randn(300, 64, generator=g) * 0.02)
        head.bias.copy_(torch.randn(300, generator=g))
    h = torch.randn(6, 64, generator=g)
    lids = [[10, 11, 12], [20, 21, 22, 23, 24], [30, 31], [40, 41, 42, 43], [10, 11, 12], [299, 0]]
    out["head_w"] = head.weight.detach().float().numpy()
    out["head_b"] = head.bias.detach().float().numpy()
    out["h"] = h.numpy()
    K = max(map(len, lids))
    out["lids"] = np.asarray([ids + [-1] * (K - len(ids)) for ids in lids], np.int64)
    for tag, cap, bias in (("cap", 30.0, True), ("plain", None, False)):
        hd = head if bias else torch.nn.Linear(64, 300, bias=False).to(torch.bfloat16)
        if not bias:
            with torch.no_grad():
                hd.weight.copy_(head.weight)
        r = readout.CodeReadout(hd, softcap=cap)
        p = r.probs(h, lids)
        out[f"probs_{tag}"] = np.asarray([row + [0.0] * (K - len(row)) for row in p], np.float32)
        pe = r.probs_each(h, lids)
        out[f"probs_each_{tag}"] = np.asarray([row + [0.0] * (K - len(row)) for row in pe], np.float32)
    return out


def main():
    from basal import blockquant, fp8block, int8block, nvfp4, readout
    for name, arrays in (("blockquant", make_blockquant(blockquant, fp8block, int8block)),
                         ("nvfp4", make_nvfp4(nvfp4)), ("readout", make_readout(readout))):
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **arrays)
        print(path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    sys.exit(main())
