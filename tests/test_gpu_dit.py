"""The DiT step with PASA self-attention on the GPU, against the same step
computed in fp32 torch with exact softmax attention (small shapes)."""
import pytest
import torch
import torch.nn.functional as F

from pasa_b200 import dit

pytestmark = pytest.mark.gpu

CFG = dit.DiTConfig(hidden=512, heads=4, ffn=1024, layers=2, text_len=16, frames=2, height=16, width=32,
                    in_channels=16, text_dim=64, freq_dim=32)


def _fp32(w: dict) -> dict:
    return {k: v.float() for k, v in w.items()}


def _setup(device):
    g = torch.Generator().manual_seed(3)
    lat = torch.randn((1, CFG.in_channels, CFG.frames, 2 * CFG.height, 2 * CFG.width), generator=g).to(device)
    txt = torch.randn((1, CFG.text_len, CFG.text_dim), generator=g).to(device)
    blocks = [dit.init_block(CFG, 20 + i, device) for i in range(CFG.layers)]
    emb = dit.init_embed(CFG, 2, device)
    return lat, txt, blocks, emb, dit.rope_table(CFG, device)


def _sdpa32(q, k, v):
    return F.scaled_dot_product_attention(q.float(), k.float(), v.float())


@pytest.mark.parametrize("fused", [True, False], ids=["fused", "torch"])
@pytest.mark.parametrize("core", ["pasa_density1", "dense"])
def test_step_matches_fp32_torch(cuda_device, core, fused):
    from pasa_b200 import dense_attention
    lat, txt, blocks, emb, rope = _setup(cuda_device)
    fn = dit.pasa_core(1.0) if core == "pasa_density1" else (lambda q, k, v: dense_attention(q, k, v))
    t = torch.tensor([700], device=cuda_device)
    got = dit.step(dit.patchify(lat), t, txt, rope, emb, blocks, CFG, fn, fused=fused).float()
    want = dit.step(dit.patchify(lat).float(), t, txt, rope, _fp32(emb), [_fp32(b) for b in blocks], CFG, _sdpa32)
    # bf16 activations through two blocks: compare against the fp32 step's scale
    err = (got - want).abs()
    ref = want.abs().max().item()
    cos = F.cosine_similarity(got.flatten(), want.flatten(), dim=0).item()
    assert err.max().item() < 3e-2 * ref and cos > 0.999, (err.max().item(), ref, cos)


def test_fused_step_matches_torch_step(cuda_device):
    """The row-kernel step against the same step in torch ops (same bf16
    weights, same PASA core): only LayerNorm/RMSNorm rounding differs."""
    lat, txt, blocks, emb, rope = _setup(cuda_device)
    t = torch.tensor([700], device=cuda_device)
    x = dit.patchify(lat)
    a = dit.step(x, t, txt, rope, emb, blocks, CFG, dit.pasa_core(0.25), fused=True).float()
    b = dit.step(x, t, txt, rope, emb, blocks, CFG, dit.pasa_core(0.25), fused=False).float()
    err = (a - b).abs().max().item()
    assert err < 2e-2 * b.abs().max().item()
    assert F.cosine_similarity(a.flatten(), b.flatten(), dim=0).item() > 0.9995


def test_sparse_step_is_close_to_dense(cuda_device):
    """At density 0.25 the correction keeps the step near the dense one."""
    from pasa_b200 import dense_attention
    lat, txt, blocks, emb, rope = _setup(cuda_device)
    t = torch.tensor([700], device=cuda_device)
    x = dit.patchify(lat)
    sparse = dit.step(x, t, txt, rope, emb, blocks, CFG, dit.pasa_core(0.25)).float()
    dense = dit.step(x, t, txt, rope, emb, blocks, CFG, lambda q, k, v: dense_attention(q, k, v)).float()
    assert torch.isfinite(sparse).all()
    assert F.cosine_similarity(sparse.flatten(), dense.flatten(), dim=0).item() > 0.99


@pytest.mark.parametrize("B,H,T,D", [(2, 3, 1000, 128), (1, 4, 2500, 64)])
def test_token_major_output_equals_head_major(cuda_device, B, H, T, D):
    """out_layout="bthd" stores the same values token-major (pasa_forward_ex)."""
    from pasa_b200 import pisa_pg_attention
    g = torch.Generator().manual_seed(T + D)
    q, k, v = (torch.randn((B, H, T, D), generator=g).to(torch.bfloat16).to(cuda_device) for _ in range(3))
    a = pisa_pg_attention(q, k, v, density=0.2)
    b = pisa_pg_attention(q, k, v, density=0.2, out_layout="bthd")
    assert b.shape == a.shape and b.transpose(1, 2).is_contiguous()
    assert torch.equal(a, b)


def test_token_major_output_needs_the_tensor_core_kernel(cuda_device):
    from pasa_b200 import pisa_pg_attention
    q = torch.randn((1, 2, 256, 64), device=cuda_device)
    with pytest.raises(ValueError):                 # fp32 runs the CUDA-core kernel: [B*H, T, D] only
        pisa_pg_attention(q, q, q, density=0.5, out_layout="bthd")
