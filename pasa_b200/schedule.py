"""Density schedule and dense/sparse gating of the PASA attention layers.

The model processors of the reference decide per layer and per denoising
step whether a self-attention call runs dense or through PASA, and at which
density (``attention_core_logic``, svg/models/wan/attention.py:355-390 and
svg/models/hyvideo/attention.py:649-690):

* dense when ``layer_idx < first_layers_fp`` or ``timestep > first_times_fp``;
* otherwise PASA at ``rescaled_density[timestep]``, the base density times a
  per-timestep calibration factor (svg/models/wan/inference.py:54-57,
  svg/models/hyvideo/inference.py:73-80).  Wan looks the timestep up exactly;
  Hunyuan takes the nearest calibrated timestep
  (``lookup_rescaled_density``, svg/models/hyvideo/utils.py:202-215).

The dense branch runs :func:`pasa_b200.dense_attention` (the tensor-core
kernel with every block selected) instead of the reference's SDPA/FlashInfer
call; fp32 inputs take ``pisa_pg_attention`` at density 1.
"""
from __future__ import annotations

import bisect
from typing import Optional

import torch

from . import ops

# Per-timestep density factors, calibrated by the reference for each model
# (data, kept as the reference has them: svg/models/wan/utils.py:182-223,
# svg/models/hyvideo/utils.py:155-200).
WAN_RESCALED_FACTORS = {
    952: 0.9751290602409638, 946: 0.9700656385542168, 940: 0.9650698795180721,
    934: 0.9601417831325302, 927: 0.9544778554216867, 920: 0.9489060240963856,
    913: 0.9434262891566265, 906: 0.9380386506024097, 898: 0.9319941204819276,
    890: 0.9260698795180723, 882: 0.9202659277108434, 873: 0.913880265060241,
    863: 0.9069636385542168, 854: 0.9008993734939759, 843: 0.8936942409638554,
    833: 0.887341469879518, 821: 0.8799662409638555, 809: 0.8728616626506024,
    796: 0.8654704578313253, 783: 0.8583968915662651, 768: 0.85062978313253,
    753: 0.8432855662650602, 737: 0.8359178554216867, 720: 0.8286168674698794,
    701: 0.821099734939759, 681: 0.8139199759036144, 660: 0.8071903614457832,
    636: 0.800514313253012, 611: 0.7947113012048193, 584: 0.789763469879518,
    555: 0.7859753012048193, 522: 0.7835873734939759, 487: 0.7832913493975904,
    448: 0.7856736385542169, 405: 0.7916138554216866, 356: 0.8026193734939759,
    302: 0.819974843373494, 241: 2.2507440386715194, 172: 2.7757292234192645,
    92: 3.0025936743632604,
}
HUNYUAN_RESCALED_FACTORS = {
    980: 1.6152366403841978, 977: 1.4244029491374073, 973: 1.2456681678710728,
    969: 1.1577642551524232, 965: 1.087926426180865, 961: 1.0259881680507759,
    956: 0.9882446640033729, 952: 0.998799764326042, 947: 0.976715734175757,
    942: 0.9477546592234024, 937: 1.0769424030861474, 931: 0.9294812964749741,
    925: 1.0657480013838343, 919: 0.9829626617416454, 913: 0.9267012194852744,
    906: 0.9763504224744779, 899: 0.881764156653075, 891: 0.8393725940255019,
    883: 0.8388535229660975, 875: 0.8281609252565499, 865: 0.9164300181371487,
    856: 0.8481337559091641, 846: 0.8545773921107588, 835: 0.8255081833973007,
    823: 0.8232195053020991, 810: 0.8222604824037629, 797: 0.8989242548341655,
    782: 0.8668879556184683, 767: 0.8278520354957465, 750: 0.8240282394569347,
    731: 0.8416698289227471, 710: 0.83350478810412, 688: 0.8543081007474298,
    663: 0.8488151060279007, 636: 0.859377515215382, 605: 0.88276764659049,
    571: 0.8928392386920468, 532: 0.9087985042129907, 488: 0.9239564591192239,
    437: 0.9691458885876514, 378: 1.038657955349757, 308: 1.1553916971248515,
    225: 1.4314307717394603, 125: 2.2366760448475045,
}


def build_rescaled_density(base_density: float, factors: dict, dynamic: bool = True) -> dict:
    """timestep -> density: base_density * factor, or base_density for every
    calibrated timestep when ``dynamic`` is off (Hunyuan's ``use_dynamic``;
    Wan always scales)."""
    return {int(ts): (base_density * f if dynamic else base_density) for ts, f in factors.items()}


def lookup_rescaled_density(rescaled_density: dict, ts: int) -> Optional[float]:
    """The density of timestep ``ts``: the exact key if present, else the
    nearest calibrated timestep (the lower one on a tie), clamped to the
    table's range; None for an empty table (hyvideo/utils.py:202-215)."""
    if ts in rescaled_density:
        return rescaled_density[ts]
    keys = sorted(rescaled_density)
    if not keys:
        return None
    if ts <= keys[0]:
        return rescaled_density[keys[0]]
    if ts >= keys[-1]:
        return rescaled_density[keys[-1]]
    i = bisect.bisect_left(keys, ts)
    lo, hi = keys[i - 1], keys[i]
    return rescaled_density[lo] if (ts - lo) <= (hi - ts) else rescaled_density[hi]


def _timestep_value(timestep) -> float:
    t = timestep[0] if isinstance(timestep, (torch.Tensor, list, tuple)) else timestep
    return float(t.item() if isinstance(t, torch.Tensor) else t)


class AttentionGate:
    """The per-layer decision of the reference processors.

    ``model`` is ``"wan"`` (exact timestep lookup) or ``"hunyuan"`` (nearest
    timestep).  Calling the gate with ``q, k, v`` of shape [cfg, H, T, D] and
    the step's ``timestep`` (tensor or number; its first element is used)
    returns the attention output of the same shape.
    """

    def __init__(self, model: str, layer_idx: int, first_layers_fp: int, first_times_fp: float,
                 rescaled_density: dict, use_random: bool = False):
        if model not in ("wan", "hunyuan"):
            raise ValueError("model must be 'wan' or 'hunyuan'")
        self.model, self.layer_idx = model, int(layer_idx)
        self.first_layers_fp, self.first_times_fp = first_layers_fp, first_times_fp
        self.rescaled_density, self.use_random = rescaled_density, use_random

    def full_attention(self, timestep) -> bool:
        """attention.py: layer_idx < first_layers_fp, or timestep > first_times_fp."""
        return self.layer_idx < self.first_layers_fp or _timestep_value(timestep) > self.first_times_fp

    def density(self, timestep) -> float:
        ts = int(_timestep_value(timestep))
        d = (self.rescaled_density.get(ts) if self.model == "wan"
             else lookup_rescaled_density(self.rescaled_density, ts))
        if d is None:
            raise AssertionError(f"Density is not found for timestep {ts}")
        return d

    def __call__(self, q, k, v, timestep):
        cfg, num_heads, seq_len, dim = q.shape
        if cfg != 1:
            raise AssertionError("Batch size must be 1 for kmeans block sparse attention")
        if self.full_attention(timestep):
            if q.dtype == torch.bfloat16:
                return ops.dense_attention(q, k, v)
            return ops.pisa_pg_attention(q, k, v, density=1.0)
        use_random = self.use_random if self.model == "hunyuan" else False
        return ops.piecewise_sparse_attention(q, k, v, density=self.density(timestep), block_size=64,
                                              use_random=use_random)
