"""Block-scaled int8 linears, B200 build (the interface of basal/int8block.py, rkinas/basal 2.8.1): the layout of
fp8block with int8 values (amax / 127, rounded half to even); the GEMM multiplies int8 by int8 into int32 for every
128-deep slice (tcgen05 kind::i8, exact), applies both scales and adds the slices in fp32.

  quantize(w), act_quant(x), gemm(q, s, w, ws, dt), linear(x, w, ws, b), Int8BlockLinear
"""
import torch

from .blockquant import BLOCK, TILES, BlockFormat, BlockLinear, fits, grid  # noqa: F401  (the shared core)

INT8_MAX = 127.0
CONFIG = TILES


def int8_refused():
    """Why --mode int8 cannot run here, None if it can: this build's int8 GEMM needs an sm_100 GPU (B200)."""
    if not torch.cuda.is_available():
        return "--mode int8 needs a CUDA GPU; this build runs on sm_100 (B200)"
    cc = torch.cuda.get_device_capability()
    if tuple(cc) != (10, 0):
        return (f"--mode int8 in this build needs an sm_100 GPU (B200); {torch.cuda.get_device_name()} is "
                f"sm_{cc[0]}{cc[1]}")
    return None


FORMAT = BlockFormat("int8_block_gemm", torch.int8, INT8_MAX, rounded=True, stages=TILES["STAGES"])
quantize, act_quant, gemm, build, linear = FORMAT.quantize, FORMAT.act_quant, FORMAT.gemm, FORMAT.build, FORMAT.linear


class Int8BlockLinear(BlockLinear):
    """A linear layer with a block-scaled int8 weight (quantize) and an optional bias."""

    FORMAT = FORMAT
