"""Host-side mirror of the reference interface: argument handling that runs
before any kernel (CPU only)."""
import inspect

import pytest
import torch

import pasa_b200
from pasa_b200 import ops


def test_signature_matches_reference():
    sig = inspect.signature(pasa_b200.pisa_pg_attention)
    names = list(sig.parameters)[:12]
    assert names == ["q", "k", "v", "density", "timestep", "block_size", "group_size", "scale", "use_cov_bias",
                     "use_random", "verbose", "prompt_token_length"]
    d = {k: p.default for k, p in sig.parameters.items()}
    assert d["density"] == 0.15 and d["block_size"] == 64 and d["group_size"] == 32
    assert d["scale"] is None and d["use_cov_bias"] is True and d["use_random"] is False


def test_piecewise_alias_signature():
    sig = inspect.signature(pasa_b200.piecewise_sparse_attention)
    assert list(sig.parameters)[:6] == ["q", "k", "v", "density", "block_size", "use_random"]


def test_cpu_tensors_are_rejected_no_fallback():
    q = torch.randn(1, 1, 128, 64)
    with pytest.raises(ValueError, match="CUDA"):
        pasa_b200.pisa_pg_attention(q, q, q, density=0.5)


def test_bad_shapes_and_options_are_rejected():
    q = torch.randn(1, 1, 128, 64)
    with pytest.raises(ValueError):
        pasa_b200.pisa_pg_attention(q, q, q, block_size=128)
    with pytest.raises(ValueError):
        pasa_b200.pisa_pg_attention(q[0], q[0], q[0])
    with pytest.raises(ValueError):
        ops._dtype_code(torch.empty(1, dtype=torch.float16))
