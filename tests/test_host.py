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


def test_integer_bf16_rounding_formula():
    """The integer round-to-nearest-even the block statistics use
    ((bits + 0x7FFF + bit16) & 0xFFFF0000) equals the bf16 conversion for
    finite values, ties and subnormals included."""
    import numpy as np
    import torch
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(200000).astype(np.float32) * 10.0 ** rng.integers(-30, 30, 200000),
        np.float32([1.0, -1.0, 0.0, 1e-40, -3e-39, 3.3895314e38]),
        # exact ties: low 16 bits 0x8000 with either parity of bit 16
        (np.arange(1000, dtype=np.uint32) * np.uint32(0x10000) + np.uint32(0x3F808000)).view(np.float32),
    ]).astype(np.float32)
    b = x.view(np.uint32)
    got = ((b + np.uint32(0x7FFF) + ((b >> 16) & 1)) & np.uint32(0xFFFF0000)).view(np.float32)
    want = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(got, want)
