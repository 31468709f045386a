"""pasa_forward_noalloc: the whole op with the library's built-in scratch
instead of a caller workspace, for callers that cannot allocate device
memory (hosts owning all device memory in their own pool, plugin interfaces
without an allocator, paths that cannot afford an allocation's implicit
synchronisation).

Called through the C ABI, twice in a row, and compared with pasa_forward
(the entry point with a caller workspace) under the tolerance the parity
tests use.  This file is collected last so that a run stopping at the first
failure has already run every other test; it also passes on its own in a
fresh process.
"""
import numpy as np
import pytest
import torch

from oracle import pasa_oracle as O
from pasa_b200 import _lib, ops

pytestmark = pytest.mark.gpu

TOL_ABS = 2e-2
TOL_COS = 0.999


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
        a, b = o.float().cpu().numpy(), ref.float().cpu().numpy()
        assert np.isfinite(a).all()
        assert float(np.max(np.abs(a - b))) <= TOL_ABS and O.cosine(a, b) >= TOL_COS, call


def test_no_alloc_rejects_problems_beyond_its_scratch(cuda_device):
    B, H, T, D = 1, 40, 75600, 128  # needs ~113 MB of scratch
    q = torch.empty(1, device=cuda_device, dtype=torch.bfloat16)
    o = torch.empty(1, device=cuda_device, dtype=torch.bfloat16)
    lib = _lib.load()
    rc = lib.pasa_forward_noalloc(torch.cuda.current_stream().cuda_stream, q.data_ptr(), q.data_ptr(), q.data_ptr(),
                                  B, H, T, D, _lib.BF16, 0.1, float(D ** -0.5), 1, None, o.data_ptr(), 0)
    assert rc == _lib.ERR_WORKSPACE
