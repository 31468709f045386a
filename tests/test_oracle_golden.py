"""The CPU oracle against the reference's own outputs (fixtures made by
tests/golden/make_golden.py from ZHANGWENTAI/PASA run through the Triton
interpreter, fp32)."""
import numpy as np
import pytest

from conftest import golden_cases, load_golden
from oracle import pasa_oracle as O

CASES = sorted(golden_cases())


def _run(name, **kw):
    case, g, q, k, v = load_golden(name)
    noise = g.get("noise")
    r = O.pisa_pg_attention(q.numpy(), k.numpy(), v.numpy(), density=case["density"],
                            use_cov_bias=case.get("use_cov_bias", True), noise=noise, dtype="fp32",
                            return_all=True, **kw)
    return case, g, r, (q, k, v)


@pytest.mark.parametrize("name", CASES)
def test_block_stats_bit_exact(name):
    case, g, r, _ = _run(name)
    NT = g["qc"].shape[1]
    # qc / kc / vc follow the reference's row order: bit-exact
    np.testing.assert_array_equal(r["qc"], g["qc"])
    np.testing.assert_array_equal(r["kc"], g["kc"])
    np.testing.assert_array_equal(r["vc"], g["vc"])
    np.testing.assert_allclose(r["h_norm"], g["h_norm"], rtol=2e-6, atol=0)
    np.testing.assert_allclose(r["h_group"], g["h_group"], rtol=0, atol=2e-6)
    assert r["top_k"] == case["top_k"] and NT == -(-case["T"] // 64)


@pytest.mark.parametrize("name", CASES)
def test_selection_bit_exact(name):
    _, g, r, _ = _run(name)
    np.testing.assert_array_equal(r["indices"], g["indices"])


@pytest.mark.parametrize("name", CASES)
def test_output_matches_reference(name):
    case, g, r, _ = _run(name)
    np.testing.assert_allclose(r["o"], g["o"], rtol=0, atol=1e-6)


@pytest.mark.parametrize("name", CASES)
def test_attention_bit_exact_on_reference_intermediates(name):
    case, g, _, (q, k, v) = _run(name)
    B, H, T, D = q.shape
    o = O.attention(q.numpy().reshape(B * H, T, D), k.numpy().reshape(B * H, T, D), v.numpy().reshape(B * H, T, D),
                    g["kc"], g["vc"], g["h_group"], g["indices"], D ** -0.5, T, dtype="fp32")
    np.testing.assert_array_equal(o.reshape(B, H, T, D), g["o"])


def test_max_shift_case_exercises_unrescaled_denominator():
    """The reference never rescales g_l (group_pisa_attention.py:242-243).
    Plant the 'fixed' variant in the oracle: it must disagree with the
    reference on the max_shift fixture, while the faithful oracle agrees."""
    case, g, _, (q, k, v) = _run("max_shift")
    B, H, T, D = q.shape
    args = (q.numpy().reshape(B * H, T, D), k.numpy().reshape(B * H, T, D), v.numpy().reshape(B * H, T, D),
            g["kc"], g["vc"], g["h_group"], g["indices"], D ** -0.5, T)
    faithful = O.attention(*args, dtype="fp32")
    fixed = O.attention(*args, dtype="fp32", rescale_gl=True)
    np.testing.assert_array_equal(faithful.reshape(g["o"].shape), g["o"])
    assert np.max(np.abs(fixed.reshape(g["o"].shape) - g["o"])) > 1e-3


def test_bf16_rounding_helper():
    x = np.array([1.0, 1.00390625, 1.005859375, -3.1415926, 65504.0, 1e-40], np.float32)
    r = O.bf16_round(x)
    # every result is a bf16 value (low 16 bits clear) and within half an ulp
    assert np.all((r.view(np.uint32) & 0xFFFF) == 0)
    assert r[1] == np.float32(1.0)            # tie -> even
    assert r[2] == np.float32(1.0078125)      # above the tie -> up


def test_bf16_oracle_rounding_points():
    """bf16 mode: every stored intermediate is bf16-representable and the
    tree sum agrees with a float64 reduction to within bf16 accumulation."""
    rng = np.random.default_rng(0)
    q, k, v = (O.bf16_round(rng.standard_normal((2, 200, 64)).astype(np.float32)) for _ in range(3))
    qc, kc, vc, hc, hn = O.chunk_reduce(q, k, v, 64, "bf16")
    for a in (qc, kc, vc, hc):
        assert np.all((a.view(np.uint32) & 0xFFFF) == 0)
    exact = np.concatenate([v, np.zeros((2, 56, 64), np.float32)], axis=1).reshape(2, 4, 64, 64).sum(2)
    assert np.max(np.abs(vc - exact)) < 0.25
