"""Block-scaled FP8 linears, B200 build (the interface of basal/fp8block.py, rkinas/basal 2.8.1): weights in 128 x 128
blocks and activations in 1 x 128 tiles, e4m3 values, fp32 scales (amax / 448); the tcgen05 GEMM applies both scales
to every 128-deep slice of the reduction and adds the slices in fp32.

  quantize(w)            weight [N, K] -> (FP8 [N, K], scales [N / 128, K / 128])
  act_quant(x)           activations [M, K] -> (FP8 [M, K], scales [M, K / 128])
  gemm(q, s, w, ws, dt)  the op basal::fp8_block_gemm: [M, N] in dt
  linear(x, w, ws, b)    x [..., K] -> [..., N]: the op basal::fp8_block_linear (act_quant + GEMM + bias)
  linear_glu(x, w, ws, a) a merged [gate; up] weight -> act(gate) * up: basal::fp8_block_linear_glu (no counterpart
                         in the reference, which applies the activation after the merged linear)
  BlockFP8Linear         a linear layer holding (w, ws, bias); lean.linear runs its parameters in compiled layers

The reference's Hopper branch (flashinfer's SM90 kernel, fp8block.py:37-71) has no counterpart: sm90() is False and
every GPU runs the sm_100a kernel.
"""
import torch

from .blockquant import BLOCK, TILES, BlockFormat, BlockLinear, fits, grid  # noqa: F401  (the shared core)

E4M3 = torch.float8_e4m3fn
FP8_MAX = 448.0
CONFIG = dict(TILES, num_stages=TILES["STAGES"])
FORMAT = BlockFormat("fp8_block_gemm", E4M3, FP8_MAX, rounded=False, stages=CONFIG["num_stages"])
quantize, act_quant, gemm = FORMAT.quantize, FORMAT.act_quant, FORMAT.gemm


def sm90():
    """False: this build has no Hopper path (basal/fp8block.py:37-58)."""
    return False


def linear(x, w, ws, bias=None):
    """x [..., K] (bf16) through a block-scaled FP8 weight -> [..., N] in x's dtype."""
    return FORMAT.linear(x, w, ws, bias)


def linear_glu(x, w, ws, act="silu"):
    """x [..., K] through a merged block-FP8 [gate; up] weight [2I, K] -> act(gate) * up [..., I] in one GEMM."""
    return FORMAT.linear_glu(x, w, ws, act)


class BlockFP8Linear(BlockLinear):
    """A linear layer with a block-scaled FP8 weight (quantize) and an optional bias."""

    FORMAT = FORMAT

    def forward(self, x):
        return linear(x, self.weight, self.weight_scale, self.bias)
