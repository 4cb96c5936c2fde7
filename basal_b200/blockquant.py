"""The block-scaled formats' shared core, B200 build: the interface of basal/blockquant.py (rkinas/basal 2.8.1) over
libbasal200's kernels.

  BLOCK, fits(lin), fuse(mods)     as basal/blockquant.py:21, :28-31, :43-51
  grid(M, N)                       the GEMM's output tiles (128 x 256 here; N % 128 != 0 refused, :34-40)
  BlockFormat(op, dtype, qmax, rounded, stages)
      .quantize(w)                 weight -> (codes, fp32 128 x 128 block scales) on the GPU, bit-exact to :126-135
      .act_quant(x)                activations -> (codes, fp32 1 x 128 scales), bit-exact to :118-124
      .gemm(q, s, w, ws, dtype)    the op basal::<op> (tcgen05 GEMM, :146-173)
      .linear(x, w, ws, bias)      act_quant + gemm + bias in one op (:175-183)
  BlockLinear(weight, scale, bias) the layer, .of(lin), .part(o, n), forward (:186-211)

Every computation runs on the GPU (sm_100a); CPU tensors are moved to the current CUDA device and the results come
back to the input's device. The reference's CPU maths lives in oracle/ (tests only).
"""
import torch

from . import ops

BLOCK = 128
# the GEMM's output tile (rows x weight rows), K slice and pipeline depth: fixed for every shape, so a row's output
# does not depend on the other rows
TILES = dict(BM=128, BN=256, BK=128, STAGES=4)


def fits(lin):
    """True for a weight a block format can hold: whole 128 x 128 blocks."""
    return all(d % BLOCK == 0 for d in lin.weight.shape)


def grid(M, N, config=TILES):
    """The number of output tiles of the block GEMM for M rows and N outputs (the persistent kernel runs
    min(tiles, SMs) CTAs over them). N must be a multiple of 128, as the reference requires."""
    if N % BLOCK:
        raise ValueError(f"block GEMM: {N} outputs, not a multiple of {BLOCK}")
    return ((M + config["BM"] - 1) // config["BM"] * ((N + config["BN"] - 1) // config["BN"]),)


def fuse(mods):
    """One weight for several linear layers that read the same input -> (merged weight, each layer's output count).
    The merged weight stacks the layers' weights by output rows; afterwards each layer's weight is a frozen view of
    its rows of it, so no second copy is held (basal/blockquant.py:43-51)."""
    sizes = [int(m.weight.shape[0]) for m in mods]
    merged = torch.cat([m.weight.detach() for m in mods], dim=0)
    start = 0
    for m, rows in zip(mods, sizes):
        m.weight = torch.nn.Parameter(merged.narrow(0, start, rows), requires_grad=False)
        start += rows
    return merged, sizes


def _on_gpu(t):
    if t.is_cuda:
        return t
    if not torch.cuda.is_available():
        raise ValueError("basal_b200 computes on CUDA tensors only (sm_100a)")
    return t.to(torch.device("cuda", torch.cuda.current_device()))


class BlockFormat:
    """One block-scaled format: values of `dtype` within +-qmax (rounded to the nearest integer, ties to even, when
    `rounded`; else saturated and cast); its GEMM the op basal::<op>. `stages` is kept for the reference's
    interface; the kernel's pipeline depth is TILES["STAGES"]."""

    def __init__(self, op, dtype, qmax, rounded, stages):
        self.op, self.dtype, self.qmax, self.rounded, self.stages = op, dtype, qmax, rounded, stages
        self.integer = not dtype.is_floating_point

    @torch.no_grad()
    def quantize(self, w):
        """[N, K] -> (values [N, K], fp32 scales [N / 128, K / 128]), on w's device."""
        q, s = ops.block_quantize(_on_gpu(w), self.integer)
        return (q, s) if w.is_cuda else (q.to(w.device), s.to(w.device))

    def act_quant(self, x):
        """[M, K] -> (values [M, K], fp32 scales [M, K / 128])."""
        f = ops.int8_act_quant if self.integer else ops.fp8_act_quant
        return f(x)

    def build(self):
        """Loads libbasal200 (the reference compiles its Triton kernel here)."""
        from . import _lib
        _lib.lib()

    def gemm(self, q, s, w, ws, dtype):
        """(q, s) [M, K] x (w, ws) [N, K]^T -> [M, N] in dtype."""
        f = ops.int8_block_gemm if self.integer else ops.fp8_block_gemm
        return f(q, s, w, ws, dtype)

    def linear(self, x, w, ws, bias=None):
        """x [..., K] through a block-scaled weight of this format -> [..., N] in x's dtype."""
        shape = x.shape
        f = ops.int8_block_linear if self.integer else ops.fp8_block_linear
        y = f(x.reshape(-1, shape[-1]), w, ws, bias)
        return y.reshape(*shape[:-1], w.shape[0])

    def linear_residual(self, x, w, ws, bias, residual):
        """residual + (x [..., K] through a block-scaled weight of this format, + bias) -> [..., N] in x's dtype, the
        sum in the GEMM's epilogue (the roundings of the linear followed by torch's addition)."""
        shape = x.shape
        f = ops.int8_block_linear_residual if self.integer else ops.fp8_block_linear_residual
        y = f(x.reshape(-1, shape[-1]), w, ws, bias, residual.reshape(-1, w.shape[0]))
        return y.reshape(*shape[:-1], w.shape[0])

    def linear_glu(self, x, w, ws, act):
        """x [..., K] through a merged [gate; up] weight of this format [2I, K] -> act(gate) * up [..., I] in x's
        dtype (act "silu" or "gelu_tanh"), the gate/up products paired in the GEMM's epilogue."""
        shape = x.shape
        f = ops.int8_block_linear_glu if self.integer else ops.fp8_block_linear_glu
        y = f(x.reshape(-1, shape[-1]), w, ws, act)
        return y.reshape(*shape[:-1], w.shape[0] // 2)


class BlockLinear(torch.nn.Module):
    """A linear layer with a block-scaled weight of a format (the subclass's FORMAT) and an optional bias.

    weight [N, K] codes and weight_scale [N / 128, K / 128] are frozen parameters; part(o, n) is a layer over output
    rows o..o + n (multiples of 128) whose tensors are views of this one's."""

    FORMAT = None

    def __init__(self, weight, scale, bias=None):
        super().__init__()
        for name, t in (("weight", weight), ("weight_scale", scale)):
            setattr(self, name, torch.nn.Parameter(t, requires_grad=False))
        self.bias = bias
        self.out_features, self.in_features = (int(d) for d in weight.shape)

    @classmethod
    def of(cls, lin):
        """The block-scaled version of a torch.nn.Linear (the bf16 weight is not kept)."""
        bias = lin.bias.detach() if lin.bias is not None else None
        return cls(*cls.FORMAT.quantize(lin.weight.detach()), bias)

    def part(self, o, n):
        rows = slice(o, o + n)
        blocks = slice(o // BLOCK, (o + n) // BLOCK)
        return type(self)(self.weight[rows], self.weight_scale[blocks], self.bias[rows] if self.bias is not None
                          else None)

    def forward(self, x):
        return self.FORMAT.linear(x, self.weight, self.weight_scale, self.bias)

    def forward_residual(self, x, residual):
        """residual + forward(x), the addition in the GEMM's epilogue (the same bits as the two steps)."""
        return self.FORMAT.linear_residual(x, self.weight, self.weight_scale, self.bias, residual)

    def glu(self, x, act="silu"):
        """For a merged [gate; up] layer (fuse): act(gate) * up of x, in one GEMM (the bias, if any, is not part of
        the gated form: None is required)."""
        if self.bias is not None:
            raise ValueError("the gated linear takes no bias")
        return self.FORMAT.linear_glu(x, self.weight, self.weight_scale, act)
