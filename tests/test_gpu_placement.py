"""Token placement of temporal heads through the C ABI against the
reference's torch formulas (placement.py:6-31, :156-184, :390-401)."""
import pytest
import torch

from oracle.layout_oracle import place_reference
from pasa_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg,H,D,ctx,F_,S,dtype", [
    (2, 8, 64, 226, 11, 4080, torch.bfloat16),   # the reference test's layout (fewer heads)
    (1, 4, 128, 256, 5, 3600, torch.bfloat16),   # HunyuanVideo 720p frame size
    (1, 3, 128, 0, 21, 1560, torch.bfloat16),    # Wan-like: no text tail
    (2, 2, 64, 17, 3, 100, torch.float32),       # ragged sizes, fp32
])
def test_placement_matches_reference(cfg, H, D, ctx, F_, S, dtype, cuda_device):
    T = ctx + F_ * S
    g = torch.Generator().manual_seed(cfg * 100 + H)
    x = [torch.randn(cfg, H, T, D, generator=g).to(dtype) for _ in range(3)]
    best = torch.randint(0, 2, (cfg, H), generator=g)
    xd = [t.to(cuda_device) for t in x]
    outs = [torch.empty_like(t) for t in xd]
    ops.hunyuan_sparse_head_placement(*xd, *outs, best.to(cuda_device), ctx, F_, S)
    for src, out in zip(x, outs):
        assert torch.equal(out.cpu(), place_reference(src, best, ctx, F_, S))
    back = torch.empty_like(outs[0])
    r = ops.hunyuan_hidden_states_placement(outs[0], back, best.to(cuda_device), ctx, F_, S)
    assert r is back
    assert torch.equal(back.cpu(), x[0])  # inverse restores the frame-major layout
    assert torch.equal(back.cpu(), place_reference(outs[0].cpu(), best, ctx, F_, S, inverse=True))


def test_placement_rejects_bad_lengths(cuda_device):
    x = torch.zeros(1, 1, 100, 64, device=cuda_device, dtype=torch.bfloat16)
    with pytest.raises(AssertionError):
        ops.hunyuan_hidden_states_placement(x, torch.empty_like(x), torch.zeros(1, 1, dtype=torch.int64), 4, 3, 30)
