"""The DiT row oracle (oracle/dit_oracle.py) against golden fixtures made by
running the reference's own row kernels (Triton interpreter, fp32) and its
torch rotary path (bf16): tests/golden/make_golden_dit.py."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import dit_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"
FIX = np.load(GOLDEN / "dit_rows.npz")
META = json.loads((GOLDEN / "dit_rows.json").read_text())
EPS = 1e-6


def _row_inputs(name):
    import sys
    sys.path.insert(0, str(GOLDEN))
    import make_golden_dit as M
    m = META[name]
    t = M.row_inputs(m["rows"], m["cols"], m["seed"])
    assert M.digest(*t.values()) == m["digest"]      # same random stream as when the fixture was made
    return {k: v.numpy().reshape(m["rows"], m["cols"]) if v.dim() == 3 else v.numpy() for k, v in t.items()}


@pytest.mark.parametrize("name", ["n320", "n640"])
def test_oracle_reproduces_reference_kernels(name):
    t = _row_inputs(name)
    x = t["x"]
    ln = O.layer_norm(x, EPS, order="reference", pad_variance=True)
    assert np.array_equal(ln, FIX[f"{name}_ln"])
    assert np.array_equal(O.layer_norm(x, EPS, t["w"], t["b"], order="reference", pad_variance=True),
                          FIX[f"{name}_ln_affine"])
    assert np.array_equal(O.layer_norm(x, EPS, t["w"], None, center=False, order="reference"), FIX[f"{name}_rms"])
    assert np.array_equal(O.modulate(FIX[f"{name}_ln"], t["scale"], t["shift"]), FIX[f"{name}_modulate"])
    assert np.array_equal(O.gate_residual(x, t["add"], t["gate"]), FIX[f"{name}_gate_residual"])


@pytest.mark.parametrize("name", ["n320", "n640"])
def test_kernel_order_is_within_rounding_of_reference_order(name):
    t = _row_inputs(name)
    for pad in (False, True):
        a = O.layer_norm(t["x"], EPS, order="kernel", pad_variance=pad)
        b = O.layer_norm(t["x"], EPS, order="reference", pad_variance=pad)
        assert np.abs(a - b).max() < 4e-6


def test_padded_variance_is_the_reference_triton_quirk():
    """The Triton LayerNorm adds (P - C) * mean^2 to the variance; the torch
    LayerNorm does not.  Without the term the oracle is torch's LayerNorm."""
    t = _row_inputs("n320")
    x = t["x"]
    plain = O.layer_norm(x, EPS, order="reference")
    ref = torch.nn.functional.layer_norm(torch.from_numpy(x), (x.shape[1],), eps=EPS).numpy()
    assert np.abs(plain - ref).max() < 2e-6
    assert np.abs(plain - FIX["n320_ln"]).max() > 1e-2       # rows with mean ~0.5: visible difference


def test_rope_matches_reference_torch_path():
    c = META["rope"]
    g = torch.Generator().manual_seed(c["seed"])
    L = c["frames"] * c["height"] * c["width"]
    x = torch.randn((1, c["heads"], L, c["head_dim"]), generator=g).to(torch.bfloat16)
    cos, sin = O.rope_table(c["frames"], c["height"], c["width"], c["head_dim"])
    got = O.rope(x.float().numpy(), cos, sin)
    want = torch.from_numpy(FIX["rope_out_bits"]).view(torch.bfloat16).float().numpy()
    assert np.array_equal(got, want)


def test_rope_table_matches_the_product_table():
    from pasa_b200 import dit
    cfg = dit.DiTConfig(frames=3, height=4, width=5)
    cos, sin = dit.rope_table(cfg, "cpu")
    oc, os_ = O.rope_table(3, 4, 5, cfg.head_dim)
    assert np.allclose(cos.numpy(), oc, atol=1e-15, rtol=0) and np.allclose(sin.numpy(), os_, atol=1e-15, rtol=0)


def test_qkv_oracle_composition():
    """qkv_rope = bf16 RMSNorm, head split, rotation; v is the head split."""
    rng = np.random.default_rng(0)
    L, H, D = 12, 3, 16
    xq = O.bf16_round(rng.standard_normal((L, H * D)).astype(np.float32))
    w = (1 + 0.1 * rng.standard_normal(H * D)).astype(np.float32)
    cos, sin = O.rope_table(2, 2, 3, D)
    q, k, v = O.qkv_rope(xq, None, xq, w, None, cos, sin, H, EPS)
    n = O.bf16_round(O.layer_norm(xq, EPS, w, None, center=False)).reshape(L, H, D).transpose(1, 0, 2)
    assert np.array_equal(q, O.rope(n, cos, sin)) and k is None
    assert np.array_equal(v, xq.reshape(L, H, D).transpose(1, 0, 2))
