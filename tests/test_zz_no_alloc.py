"""pasa_forward_noalloc: the whole op with the library's built-in scratch
instead of a caller workspace, for callers that cannot allocate device
memory (hosts owning all device memory in their own pool, plugin interfaces
without an allocator, paths that cannot afford an allocation's implicit
synchronisation).

Called through the C ABI, twice in a row, and compared with pasa_forward
(the entry point with a caller workspace).  Both run the same deterministic
kernels on the same inputs, so the outputs must be equal bit for bit: a
stale or aliased scratch region cannot hide inside a tolerance.  This file
is collected last so that a run stopping at the first failure has already
run every other test; it also passes on its own in a fresh process.
"""
import numpy as np
import pytest
import torch

from pasa_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _noalloc(q, k, v, density, o):
    B, H, T, D = q.shape
    lib = _lib.load()
    return lib.pasa_forward_noalloc(torch.cuda.current_stream(q.device).cuda_stream, q.data_ptr(), k.data_ptr(),
                                    v.data_ptr(), B, H, T, D, _lib.BF16, float(density), float(D ** -0.5), 1, None,
                                    o.data_ptr(), _lib.ATTN_AUTO)


def test_no_alloc_entry_matches_workspace_entry(cuda_device):
    g = torch.Generator().manual_seed(123)
    B, H, T, D, density = 1, 3, 3000, 128, 0.15
    q, k, v = (torch.randn(B, H, T, D, generator=g).to(torch.bfloat16).to(cuda_device) for _ in range(3))
    ref = ops.pisa_pg_attention(q, k, v, density=density)  # workspace entry point (pasa_forward)
    for call in range(2):  # the scratch keeps the previous call's contents
        o = torch.full_like(v, float("nan"))
        assert _noalloc(q, k, v, density, o) == _lib.OK
        torch.cuda.synchronize()
        assert np.isfinite(o.float().cpu().numpy()).all(), call
        assert torch.equal(o, ref), call


def test_no_alloc_different_problem_after_a_larger_one(cuda_device):
    # a smaller problem after a larger one: every scratch region it reads is
    # rewritten, so the leftover contents of the first call change nothing
    g = torch.Generator().manual_seed(7)
    for (H, T, density) in ((4, 5000, 0.2), (2, 1500, 0.1)):
        q, k, v = (torch.randn(1, H, T, 128, generator=g).to(torch.bfloat16).to(cuda_device) for _ in range(3))
        o = torch.empty_like(v)
        assert _noalloc(q, k, v, density, o) == _lib.OK
        torch.cuda.synchronize()
        assert torch.equal(o, ops.pisa_pg_attention(q, k, v, density=density)), (H, T)


def test_no_alloc_rejects_problems_beyond_its_scratch(cuda_device):
    B, H, T, D = 1, 40, 75600, 128  # needs ~113 MB of scratch
    q = torch.empty(1, device=cuda_device, dtype=torch.bfloat16)
    o = torch.empty(1, device=cuda_device, dtype=torch.bfloat16)
    lib = _lib.load()
    rc = lib.pasa_forward_noalloc(torch.cuda.current_stream().cuda_stream, q.data_ptr(), q.data_ptr(), q.data_ptr(),
                                  B, H, T, D, _lib.BF16, 0.1, float(D ** -0.5), 1, None, o.data_ptr(), 0)
    assert rc == _lib.ERR_WORKSPACE
