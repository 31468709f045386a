"""Dense attention on the tensor-core kernel (pasa_dense_attn) and the gated
layer call (schedule.AttentionGate) on the GPU."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _qkv(B, H, T, D, seed, device):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn((B, H, T, D), generator=g).to(torch.bfloat16).to(device) for _ in range(3)]


@pytest.mark.parametrize("T,D", [(1000, 128), (2500, 128), (640, 64), (64, 128), (70, 64)])
def test_dense_matches_fp32_softmax_attention(cuda_device, T, D):
    from pasa_b200 import dense_attention
    q, k, v = _qkv(1, 2, T, D, T + D, cuda_device)
    o = dense_attention(q, k, v).float()
    # fp32 reference of the same op: softmax(q k^T / sqrt(D)) v
    ref = torch.softmax(q.float() @ k.float().transpose(-1, -2) * D ** -0.5, dim=-1) @ v.float()
    err = (o - ref).abs()
    # bf16 P and bf16 output rounding: a few bf16 ulps of |o|
    assert err.max().item() < 2e-2 and err.mean().item() < 2e-3, (err.max().item(), err.mean().item())


def test_dense_equals_density_one(cuda_device):
    """Every block selected: the correction terms vanish, so the sparse op at
    density 1 gives the dense result."""
    from pasa_b200 import dense_attention, pisa_pg_attention
    q, k, v = _qkv(1, 3, 2500, 128, 7, cuda_device)
    a = dense_attention(q, k, v).float()
    b = pisa_pg_attention(q, k, v, density=1.0).float()
    assert (a - b).abs().max().item() < 1e-2


def test_dense_rejects_fp32(cuda_device):
    from pasa_b200 import dense_attention
    q = torch.zeros((1, 1, 128, 64), device=cuda_device)
    with pytest.raises(ValueError):
        dense_attention(q, q, q)


def test_gate_runs_both_branches(cuda_device):
    from pasa_b200 import dense_attention, pisa_pg_attention
    from pasa_b200 import schedule as S
    q, k, v = _qkv(1, 2, 2500, 128, 9, cuda_device)
    dens = S.build_rescaled_density(0.1, S.WAN_RESCALED_FACTORS)
    dense_gate = S.AttentionGate("wan", 0, 1, 900, dens)
    assert torch.equal(dense_gate(q, k, v, torch.tensor([890])), dense_attention(q, k, v))
    sparse_gate = S.AttentionGate("wan", 5, 1, 900, dens)
    want = pisa_pg_attention(q, k, v, density=0.1 * S.WAN_RESCALED_FACTORS[890])
    assert torch.equal(sparse_gate(q, k, v, torch.tensor([890])), want)
