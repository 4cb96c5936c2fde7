"""Host-side pieces of the C5 model (basal_b200/hybrid.py) that need no GPU."""
import torch

from basal_b200 import hybrid


def test_rope_matches_the_rotate_half_form():
    """rope (x1 cos - x2 sin, x2 cos + x1 sin into a buffer) rounds every product and sum as the reference's
    x cos + rotate_half(x) sin (basal/gdn_graph.py:446-451): equal bit for bit in bf16, on a transposed view too."""
    g = torch.Generator().manual_seed(0)
    r = 32
    x = torch.randn(3, 37, 4, 128, generator=g).bfloat16().transpose(1, 2)  # [b, heads, T, d], not contiguous
    ang = torch.rand(3, 37, r // 2, generator=g) * 6
    cos, sin = torch.cat([ang, ang], -1).cos().bfloat16(), torch.cat([ang, ang], -1).sin().bfloat16()
    xr = x[..., :r]
    rot = torch.cat([-xr[..., r // 2:], xr[..., : r // 2]], -1)
    want = torch.cat([xr * cos[:, None] + rot * sin[:, None], x[..., r:]], -1)
    assert torch.equal(hybrid.rope(x, cos, sin, r), want)
    out = torch.empty(3, 4, 50, 128, dtype=torch.bfloat16)[:, :, 13:]
    hybrid.rope(x, cos, sin, r, out=out)
    assert torch.equal(out, want)
