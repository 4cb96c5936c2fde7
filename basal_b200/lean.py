"""The linear dispatch of compiled layers, B200 build (basal/lean.py:56-93, rkinas/basal 2.8.1): a module becomes a
parameter tuple, and linear(x, p) picks the GEMM by the tuple's length and the weight's dtype, so that a compiled layer
function runs any projection through one call.

  _params(m)   (weight, bias) | (weight, block scales, bias) of a BlockLinear | (weight, scales, alpha, inv_g, bias)
               of an NVFP4Linear
  linear(x, p) F.linear | block FP8 / INT8 (basal::fp8_block_linear / int8_block_linear) | NVFP4 (basal::nvfp4_linear)
The reference's per-tensor FP8Linear (ModelOpt checkpoints, 4-tuple) is not part of this build.
"""
import torch
import torch.nn.functional as F

from . import blockquant, fp8block, int8block, nvfp4


def _params(m):
    if isinstance(m, blockquant.BlockLinear):
        return (m.weight, m.weight_scale, m.bias)
    if isinstance(m, nvfp4.NVFP4Linear):
        return (m.weight, m.weight_scale, m.alpha, m.inv_g, m.bias)
    return (m.weight, m.bias)


def linear(x, p):
    if len(p) == 2:
        return F.linear(x, p[0], p[1])
    if len(p) == 3:
        if p[0].dtype == torch.int8:
            return int8block.linear(x, *p)
        return fp8block.linear(x, *p)
    if len(p) == 5:
        return nvfp4.linear(x, *p)
    raise NotImplementedError("per-tensor FP8 (ModelOpt FP8Linear) parameters are not part of basal_b200")
