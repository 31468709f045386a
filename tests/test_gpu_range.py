"""pasa_forward_range (through the C ABI): the op on a range of query
blocks writes exactly those rows, equal bit for bit to pasa_forward's, and
disjoint ranges that cover all blocks rebuild pasa_forward's output."""
import pytest
import torch

from pasa_b200 import ops, synth

pytestmark = pytest.mark.gpu


def _inputs(B, H, T, D, seed, device):
    g = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(B, H, T, D, generator=g).to(torch.bfloat16).to(device) for _ in range(3))


def test_ranges_rebuild_the_full_op(cuda_device):
    B, H, T, D, density = 1, 3, 4000, 128, 0.15  # NT = 63: odd, ragged last block
    q, k, v = _inputs(B, H, T, D, 3, cuda_device)
    full = ops.pisa_pg_attention(q, k, v, density=density)
    NT = -(-T // 64)
    cuts = [0, 50, 97, 126, 127, H * NT]  # odd boundaries, inside and across heads
    out = torch.full_like(v, float("nan"))
    for b, e in zip(cuts, cuts[1:]):
        part = torch.full_like(v, float("nan"))
        ops.pisa_pg_attention_range(q, k, v, b, e, density=density, out=part)
        ops.pisa_pg_attention_range(q, k, v, b, e, density=density, out=out)
        torch.cuda.synchronize()
        rows = torch.zeros(B * H, NT * 64, dtype=torch.bool, device=cuda_device)
        rows.view(-1)[b * 64:e * 64] = True
        rows = rows[:, :T].reshape(B, H, T)
        assert torch.equal(part[rows], full[rows])
        assert torch.isnan(part[~rows].float()).all()  # every other row untouched
    assert torch.equal(out, full)


def test_shard_blocks_over_eight_ranks_rebuild_wan13b_heads(cuda_device):
    """The (head, query-block) shards bench.py gives 8 ranks for the 12
    heads of Wan2.1-1.3B, run one after another on one GPU, rebuild the op."""
    w = synth.WORKLOADS["wan1.3b-480p"]
    q, k, v = synth.make_inputs(w, range(w.heads), cuda_device)
    full = ops.pisa_pg_attention(q, k, v, density=w.density)
    out = torch.empty_like(v)
    for r in range(8):
        b, e = synth.shard_blocks(w.heads, w.NT, r, 8)
        ops.pisa_pg_attention_range(q, k, v, b, e, density=w.density, out=out)
    torch.cuda.synchronize()
    assert torch.equal(out, full)
