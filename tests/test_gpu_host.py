"""pasa_forward_host (pisa_pg_attention_host): the whole op on host buffers,
pipelined over chunks of heads, must equal the device op on the same heads
bit for bit (every chunk runs the same kernels on its heads)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(B, H, T, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn((B, H, T, D), generator=g).to(dtype) for _ in range(3))
    return q, k, v


@pytest.mark.parametrize("heads_per_chunk", [1, 2, 3, 8])
def test_host_pipeline_equals_device_op(cuda_device, heads_per_chunk):
    from pasa_b200 import pisa_pg_attention, pisa_pg_attention_host
    q, k, v = _inputs(1, 5, 2500, 128, torch.bfloat16, 11)   # 5 heads: ragged last chunk for 2, 3
    ref = pisa_pg_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), density=0.15).cpu()
    qh, kh, vh = (t.pin_memory() for t in (q, k, v))
    out = pisa_pg_attention_host(qh, kh, vh, density=0.15, heads_per_chunk=heads_per_chunk)
    assert out.dtype == torch.bfloat16 and out.shape == q.shape
    assert torch.equal(out, ref)


def test_host_pipeline_f32_and_out_buffer(cuda_device):
    from pasa_b200 import pisa_pg_attention, pisa_pg_attention_host
    q, k, v = _inputs(2, 2, 700, 64, torch.float32, 12)
    ref = pisa_pg_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), density=0.25).cpu()
    out = torch.full_like(q, float("nan")).pin_memory()
    got = pisa_pg_attention_host(q.pin_memory(), k.pin_memory(), v.pin_memory(), density=0.25,
                                 heads_per_chunk=3, out=out)
    assert got.data_ptr() == out.data_ptr()
    assert torch.equal(out, ref)


def test_host_pipeline_pageable_buffers(cuda_device):
    """Pageable host memory gives the same result (the copies just do not overlap)."""
    from pasa_b200 import pisa_pg_attention, pisa_pg_attention_host
    q, k, v = _inputs(1, 3, 1000, 128, torch.bfloat16, 13)
    ref = pisa_pg_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), density=0.2).cpu()
    out = pisa_pg_attention_host(q, k, v, density=0.2, heads_per_chunk=2, out=torch.empty_like(q))
    assert torch.equal(out, ref)


def test_host_pipeline_rejects_bad_arguments(cuda_device):
    from pasa_b200 import pisa_pg_attention_host
    q, k, v = _inputs(1, 2, 640, 128, torch.bfloat16, 14)
    with pytest.raises(ValueError):
        pisa_pg_attention_host(q.to(cuda_device), k, v)          # device tensor
    with pytest.raises(ValueError):
        pisa_pg_attention_host(q, k, v, heads_per_chunk=0)       # no chunk size
    with pytest.raises(ValueError):
        pisa_pg_attention_host(q, k[:, :, :320], v)              # shape mismatch
