"""Density schedule and dense/sparse gating (pasa_b200.schedule): the rules of
the reference processors' attention_core_logic and lookup_rescaled_density."""
import math

import pytest
import torch

from pasa_b200 import schedule as S


def test_tables_are_the_calibrated_ones():
    # key count, key sum and factor sum of svg/models/wan/utils.py:182-223 and
    # svg/models/hyvideo/utils.py:155-200
    assert len(S.WAN_RESCALED_FACTORS) == 40 and sum(S.WAN_RESCALED_FACTORS) == 28014
    assert math.isclose(sum(S.WAN_RESCALED_FACTORS.values()), 40.18051124970705, rel_tol=1e-15)
    assert len(S.HUNYUAN_RESCALED_FACTORS) == 44 and sum(S.HUNYUAN_RESCALED_FACTORS) == 33929
    assert math.isclose(sum(S.HUNYUAN_RESCALED_FACTORS.values()), 44.0, rel_tol=1e-12)
    assert S.WAN_RESCALED_FACTORS[952] == 0.9751290602409638
    assert S.HUNYUAN_RESCALED_FACTORS[125] == 2.2366760448475045


def test_build_rescaled_density():
    d = S.build_rescaled_density(0.1, S.HUNYUAN_RESCALED_FACTORS)
    assert d[980] == 0.1 * 1.6152366403841978
    flat = S.build_rescaled_density(0.1, S.HUNYUAN_RESCALED_FACTORS, dynamic=False)
    assert set(flat) == set(S.HUNYUAN_RESCALED_FACTORS) and all(v == 0.1 for v in flat.values())


def test_lookup_nearest_key():
    d = {100: 1.0, 200: 2.0, 300: 3.0}
    assert S.lookup_rescaled_density(d, 200) == 2.0          # exact
    assert S.lookup_rescaled_density(d, 149) == 1.0          # nearer to 100
    assert S.lookup_rescaled_density(d, 150) == 1.0          # tie goes to the lower key
    assert S.lookup_rescaled_density(d, 151) == 2.0
    assert S.lookup_rescaled_density(d, 50) == 1.0           # below the range
    assert S.lookup_rescaled_density(d, 1000) == 3.0         # above the range
    assert S.lookup_rescaled_density({}, 5) is None


def test_gate_decisions():
    dens = S.build_rescaled_density(0.1, S.WAN_RESCALED_FACTORS)
    g = S.AttentionGate("wan", layer_idx=0, first_layers_fp=1, first_times_fp=900, rescaled_density=dens)
    assert g.full_attention(torch.tensor([500]))             # an early layer runs dense
    g = S.AttentionGate("wan", layer_idx=3, first_layers_fp=1, first_times_fp=900, rescaled_density=dens)
    assert g.full_attention(torch.tensor([952]))             # an early (noisy) timestep runs dense
    assert not g.full_attention(torch.tensor([890]))
    assert g.density(torch.tensor([890])) == 0.1 * S.WAN_RESCALED_FACTORS[890]
    with pytest.raises(AssertionError):                      # Wan needs the exact calibrated timestep
        g.density(torch.tensor([891]))
    h = S.AttentionGate("hunyuan", layer_idx=3, first_layers_fp=1, first_times_fp=900,
                        rescaled_density=S.build_rescaled_density(0.1, S.HUNYUAN_RESCALED_FACTORS))
    assert h.density(torch.tensor([898])) == 0.1 * S.HUNYUAN_RESCALED_FACTORS[899]   # nearest
    with pytest.raises(ValueError):
        S.AttentionGate("flux", 0, 0, 0, {})
