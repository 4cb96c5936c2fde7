"""NVFP4 linears, B200 build (the interface of basal/nvfp4.py, rkinas/basal 2.8.1): e2m1 values, one e4m3 scale per 16
consecutive input features (in cuBLAS's 128 x 4 tile swizzle), one fp32 global scale per tensor; the GEMM is the
tcgen05 kind::mxf4nvf4 kernel of libbasal200, the block scales applied by the tensor core, the global scales (alpha)
in its epilogue.

  quantize(w)               weight [N, K] -> (codes [N, K / 2] uint8, swizzled e4m3 scales, global scale [1])
  act_quant(x, inv_g)       activations [M, K] -> (codes [Mp, K / 2], swizzled scales); Mp = M rounded up to 128
  linear(x, w, ws, alpha, inv_g, bias)   x [..., K] -> [..., N] (the op basal::nvfp4_linear)
  NVFP4Linear               a linear layer holding them; lean.linear runs its parameters in compiled layers
  swizzle / unswizzle / pack / unpack / dequantize   the storage layout (index arithmetic on tensors, any device)

The storage layout, stated once (the reference's bytes, basal/nvfp4.py:49-68, :140-143):
  - codes: feature 2i of a row in the low nibble of byte i, feature 2i + 1 in the high nibble; a code is 3 magnitude
    bits (an index into E2M1) under a sign bit (8);
  - scales: rows are padded to a multiple of 128 and the K / 16 groups to a multiple of 4; the scale of (row r, group
    j) is byte ((r // 128) * (groups / 4) + j // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + j % 4, so every
    128 rows x 4 groups form one 512-byte tile and the rows' tiles follow each other.
"""
import torch

from . import ops
from .blockquant import _on_gpu

BLOCK = 16                        # features per e4m3 scale
E2M1 = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)   # magnitude of codes 0..7
FP4_MAX, E4M3_MAX = E2M1[-1], 448.0
E4M3 = torch.float8_e4m3fn
MARGIN = 2.0                      # an activation global scale covers MARGIN x the calibrated amax
CANDIDATES = tuple(1.0 - 0.04 * j for j in range(8))   # the weight quantiser's trial scales, x amax / 6


def _cuts():
    """Rounding to e2m1: the midpoint between codes k and k + 1, and whether a value exactly on it goes up (it goes to
    the even code: up when k is odd)."""
    return tuple((0.5 * (E2M1[k] + E2M1[k + 1]), bool(k & 1)) for k in range(len(E2M1) - 1))


CUTS = _cuts()
TILE_ROWS, TILE_GROUPS, TILE_BYTES = 128, 4, 512


def fits(lin):
    """True for a weight this module can hold: whole 64-feature scale tiles along K, N a multiple of 16."""
    n, k = lin.weight.shape
    return (k % (TILE_GROUPS * BLOCK), n % 16) == (0, 0)


def _round_up(n, m):
    return (n + m - 1) // m * m


def _values(c):
    """e2m1 codes (uint8, any shape) -> fp32 values."""
    mag = torch.tensor(E2M1, dtype=torch.float32, device=c.device)[(c & 7).long()]
    return mag * (1.0 - 2.0 * (c >> 3).float())


def scale_offsets(rows, groups, device=None):
    """int64 [rows, groups]: the byte of the swizzled layout that holds the scale of (row r, group j)."""
    r = torch.arange(rows, device=device).view(-1, 1)
    j = torch.arange(groups, device=device).view(1, -1)
    tiles_per_row_block = _round_up(groups, TILE_GROUPS) // TILE_GROUPS
    tile = (r // TILE_ROWS) * tiles_per_row_block + j // TILE_GROUPS
    return tile * TILE_BYTES + (r % 32) * 16 + (r % TILE_ROWS // 32) * 4 + j % TILE_GROUPS


def swizzled_bytes(rows, groups):
    """The size of the swizzled layout of [rows, groups] scales (padding included)."""
    return _round_up(rows, TILE_ROWS) * _round_up(groups, TILE_GROUPS)


def swizzle(s):
    """[rows, K / 16] e4m3 scales -> the swizzled layout, flattened (padding bytes 0)."""
    rows, groups = s.shape
    out = torch.zeros(swizzled_bytes(rows, groups), dtype=torch.uint8, device=s.device)
    out[scale_offsets(rows, groups, s.device).reshape(-1)] = s.contiguous().view(torch.uint8).reshape(-1)
    return out.view(E4M3)


def unswizzle(f, rows, cols):
    """The inverse of swizzle -> [rows, cols] e4m3."""
    return f.view(torch.uint8)[scale_offsets(rows, cols, f.device)].view(E4M3)


def pack(c):
    """[M, K] codes -> [M, K / 2] bytes (even feature in the low nibble)."""
    pairs = c.reshape(c.shape[0], -1, 2).to(torch.int32)
    return (pairs[..., 0] + 16 * pairs[..., 1]).to(torch.uint8)


def unpack(p):
    """[M, K / 2] bytes -> [M, K] codes."""
    shifts = torch.tensor([0, 4], dtype=torch.uint8, device=p.device)
    return ((p.unsqueeze(-1) >> shifts) & 15).reshape(p.shape[0], -1)


@torch.no_grad()
def quantize(w):
    """[N, K] -> (codes [N, K / 2] uint8, swizzled e4m3 block scales, fp32 global scale [1]), on w's device: the
    8-candidate least-squares scales of basal/nvfp4.py:75-97, bit for bit, computed on the GPU."""
    codes, scales, g = ops.nvfp4_quantize(_on_gpu(w))
    if w.is_cuda:
        return codes, scales, g
    return codes.to(w.device), scales.to(w.device), g.to(w.device)


def dequantize(codes, scales, g, N, K):
    """The weight's values as fp32 [N, K]."""
    per_group = unswizzle(scales, N, K // BLOCK).float().unsqueeze(-1)
    return (_values(unpack(codes)).reshape(N, K // BLOCK, BLOCK) * per_group).reshape(N, K) * g


def act_quant(x, inv_g):
    """[M, K] bf16 -> (codes [Mp, K / 2] uint8, swizzled scales uint8 [Mp * K / 16]); rows past M are zeros."""
    return ops.nvfp4_act_quant(x, inv_g)


def build():
    """Loads libbasal200 (the reference compiles its Triton quantiser here)."""
    from . import _lib
    _lib.lib()


def linear(x, w, ws, alpha, inv_g, bias=None):
    """x [..., K] through an NVFP4 weight (codes w [N, K / 2], swizzled scales ws, alpha = the two global scales'
    product, inv_g = 1 / the input's global scale) -> [..., N] in x's dtype."""
    lead, K = x.shape[:-1], x.shape[-1]
    if bias is None:
        y = ops.nvfp4_linear(x.reshape(-1, K), w, ws, alpha, inv_g)
    else:  # the reference's y + bias.to(y.dtype), with its roundings, inside the GEMM's epilogue
        y = ops.nvfp4_linear_bias(x.reshape(-1, K), w, ws, alpha, inv_g, bias)
    return y.reshape(*lead, w.shape[0])


def _frozen(t):
    return torch.nn.Parameter(t, requires_grad=False)


class NVFP4Linear(torch.nn.Module):
    """A linear layer with an NVFP4 weight (quantize) and a fixed input global scale xg (the weight's is wg); alpha =
    wg * xg and inv_g = 1 / xg are kept as one-element parameters for the op. part(o, n) is a view of output rows
    o..o + n (multiples of 128, so whole scale tiles)."""

    def __init__(self, weight, scale, wg, xg, bias=None, out_features=None):
        super().__init__()
        self.weight, self.weight_scale = _frozen(weight), _frozen(scale)
        self.wg, self.xg, self.bias = wg, xg, bias
        self.alpha = _frozen(torch.as_tensor(wg * xg).float().reshape(1))
        self.inv_g = _frozen((1.0 / torch.as_tensor(xg)).float().reshape(1))
        self.out_features = weight.shape[0]
        self.in_features = 2 * weight.shape[1]

    @classmethod
    def of(cls, lin, amax):
        """The NVFP4 version of a torch.nn.Linear whose inputs reached |x| <= amax in calibration: the input global
        scale spans MARGIN x amax (at least 1e-6) over the largest e2m1 value times the largest e4m3 scale."""
        codes, scales, wg = quantize(lin.weight.detach())
        span = max(float(amax), 1e-6) * MARGIN
        xg = torch.tensor([span / (FP4_MAX * E4M3_MAX)], device=codes.device)
        return cls(codes, scales, wg, xg, lin.bias.detach() if lin.bias is not None else None)

    def part(self, o, n):
        if o % TILE_ROWS or n % TILE_ROWS:  # the reference's error type (an assertion), raised explicitly
            raise AssertionError(f"NVFP4Linear.part({o}, {n}): parts are whole 128-row scale tiles")
        row_block = TILE_ROWS * _round_up(self.in_features // BLOCK, TILE_GROUPS)  # bytes of 128 rows' scales
        first, last = o // TILE_ROWS, (o + n) // TILE_ROWS
        bias = self.bias[o: o + n] if self.bias is not None else None
        return NVFP4Linear(self.weight[o: o + n], self.weight_scale[first * row_block: last * row_block], self.wg,
                           self.xg, bias)

    def forward(self, x):
        return linear(x, self.weight, self.weight_scale, self.alpha, self.inv_g, self.bias)
