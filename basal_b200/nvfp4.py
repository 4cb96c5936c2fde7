"""NVFP4 linears, B200 build (the interface of basal/nvfp4.py, rkinas/basal 2.8.1): e2m1 values, one e4m3 scale per 16
consecutive input features (in cuBLAS's 128 x 4 tile swizzle), one fp32 global scale per tensor; the GEMM is the
tcgen05 kind::mxf4nvf4 kernel of libbasal200, the block scales applied by the tensor core, the global scales (alpha)
in its epilogue.

  quantize(w)               weight [N, K] -> (codes [N, K / 2] uint8, swizzled e4m3 scales, global scale [1])
  act_quant(x, inv_g)       activations [M, K] -> (codes [Mp, K / 2], swizzled scales); Mp = M rounded up to 128
  linear(x, w, ws, alpha, inv_g, bias)   x [..., K] -> [..., N] (the op basal::nvfp4_linear)
  NVFP4Linear               a linear layer holding them; lean.linear runs its parameters in compiled layers
  swizzle / unswizzle / pack / unpack / dequantize   the storage layout (tensor reshapes, any device)
"""
import torch

from . import ops
from .blockquant import _on_gpu

BLOCK = 16
E2M1 = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
CUTS = tuple(((a + b) / 2, k % 2 == 1) for k, (a, b) in enumerate(zip(E2M1, E2M1[1:])))
FP4_MAX, E4M3_MAX = E2M1[-1], 448.0
E4M3 = torch.float8_e4m3fn
MARGIN = 2.0
CANDIDATES = tuple(1.0 - 0.04 * j for j in range(8))


def fits(lin):
    """True for a weight this module can hold: K a multiple of 64 (four scale blocks), N a multiple of 16."""
    n, k = lin.weight.shape
    return k % 64 == 0 and n % 16 == 0


def _values(c):
    v = torch.tensor(E2M1, device=c.device)[(c & 7).long()]
    return torch.where(c >= 8, -v, v)


def swizzle(s):
    """[rows, K / 16] e4m3 scales -> the 128 x 4 tiles, flattened (rows padded to 128, columns to 4, with 0)."""
    r, c = s.shape
    R, C = -(-r // 128), -(-c // 4)
    p = torch.zeros(R * 128, C * 4, dtype=torch.uint8, device=s.device)
    p[:r, :c] = s.view(torch.uint8)
    b = p.view(R, 128, C, 4).permute(0, 2, 1, 3)
    return b.reshape(-1, 4, 32, 4).transpose(1, 2).reshape(-1).view(E4M3)


def unswizzle(f, rows, cols):
    """The inverse of swizzle -> [rows, cols] e4m3."""
    R, C = -(-rows // 128), -(-cols // 4)
    b = f.view(torch.uint8).view(R * C, 32, 4, 4).transpose(1, 2).reshape(R, C, 128, 4).permute(0, 2, 1, 3)
    return b.reshape(R * 128, C * 4)[:rows, :cols].contiguous().view(E4M3)


def pack(c):
    """[M, K] codes -> [M, K / 2] bytes (even feature in the low nibble)."""
    return c[:, 0::2] | (c[:, 1::2] << 4)


def unpack(p):
    return torch.stack([p & 15, p >> 4], -1).view(p.shape[0], -1)


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
    s = unswizzle(scales, N, K // BLOCK).float()
    return (_values(unpack(codes)).view(N, K // BLOCK, BLOCK) * s[..., None]).view(N, K) * g


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
    shape = x.shape
    N = w.shape[0]
    y = ops.nvfp4_linear(x.reshape(-1, shape[-1]), w, ws, alpha, inv_g)
    if bias is not None:
        y = y + bias.to(y.dtype)
    return y.reshape(*shape[:-1], N)


class NVFP4Linear(torch.nn.Module):
    """A linear layer with an NVFP4 weight (quantize) and a fixed input global scale; part(o, n) is a view of output
    rows o..o + n (multiples of 128: whole scale tiles)."""

    def __init__(self, weight, scale, wg, xg, bias=None, out_features=None):
        super().__init__()
        self.weight = torch.nn.Parameter(weight, requires_grad=False)
        self.weight_scale = torch.nn.Parameter(scale, requires_grad=False)
        self.alpha = torch.nn.Parameter((wg * xg).float().reshape(1), requires_grad=False)
        self.inv_g = torch.nn.Parameter((1.0 / xg).float().reshape(1), requires_grad=False)
        self.wg, self.xg = wg, xg
        self.bias = bias
        self.out_features, self.in_features = weight.shape[0], weight.shape[1] * 2

    @classmethod
    def of(cls, lin, amax):
        """The NVFP4 version of a torch.nn.Linear whose inputs reached |x| <= amax in calibration."""
        q, s, wg = quantize(lin.weight.detach())
        xg = torch.tensor([max(float(amax), 1e-6) * MARGIN / (FP4_MAX * E4M3_MAX)], device=q.device)
        return cls(q, s, wg, xg, None if lin.bias is None else lin.bias.detach())

    def part(self, o, n):
        assert o % 128 == 0 and n % 128 == 0, "parts of whole scale tiles"
        cols = self.in_features // BLOCK
        C = -(-cols // 4) * 4
        return NVFP4Linear(self.weight[o: o + n], self.weight_scale[o * C: (o + n) * C], self.wg, self.xg,
                           None if self.bias is None else self.bias[o: o + n])

    def forward(self, x):
        return linear(x, self.weight, self.weight_scale, self.alpha, self.inv_g, self.bias)
