"""Spatial / temporal head classification (the SVG profiling step): torch
restatement of the reference, the checker of the CUDA kernel
``pasa_sample_mse`` (``pasa_b200.classify``).

TEST INFRASTRUCTURE ONLY: imported by tests/ only, never by the product.

Restates ``sample_mse`` (svg/models/hyvideo/attention.py:381-405, Wan twin
svg/models/wan/attention.py:264-288) with the emulated masks of
``get_attention_mask`` (svg/models/hyvideo/utils.py:48-94,
svg/models/wan/utils.py:63-110).  The reference builds each mask as a dense
T x T tensor on the CPU with a Python double loop (4.3 GB at T=32760) and
then indexes the sampled rows.  Here the two masks are evaluated in closed
form for the sampled rows only:

* spatial: keys within ``thres // 128`` 128-token blocks of the query block,
  with ``thres = 1.5 * frame_size`` (HunyuanVideo) or ``2 * frame_size``
  (Wan).  HunyuanVideo keeps the trailing ``context_length`` text tokens
  fully visible in both directions.  Wan adds a first-frame sink
  (keys < frame_size).
* temporal: the spatial mask of the token-major layout.  Position
  f*S + p maps to p*F + f, from the reference's
  ``reshape(S, F, S, F).permute(1, 0, 3, 2)``.

``sample_mse`` consumes the CPU random generator exactly as the reference
does (``torch.randint(0, sample_mse_max_row, (rows,))``).  It returns the
per-head MSE of each masked softmax output against the full softmax output,
``[2, cfg, H]``.  ``classify_heads`` takes the argmin (0 spatial,
1 temporal), which is the ``best_mask_idx`` that the placement functions
consume.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

MASKS = ("spatial", "temporal")


def _band(qi: torch.Tensor, ki: torch.Tensor, frame_size: int, factor: float) -> torch.Tensor:
    """|qi//128 - ki//128| < (factor * frame_size) // 128, elementwise with broadcasting."""
    width = int((factor * frame_size) // 128)
    return (torch.div(qi, 128, rounding_mode="floor") - torch.div(ki, 128, rounding_mode="floor")).abs() < width


def emulated_mask_rows(rows: torch.Tensor, mask_name: str, model: str, context_length: int, num_frame: int,
                       frame_size: int) -> torch.Tensor:
    """Rows ``rows`` of the emulated attention mask, as a bool [R, T] tensor.

    ``model`` is "hunyuan" (text tokens at the tail, hyvideo/utils.py:48-94)
    or "wan" (no text tokens, first-frame sink, wan/utils.py:63-110)."""
    device = rows.device
    V = num_frame * frame_size
    T = V + (context_length if model == "hunyuan" else 0)
    keys = torch.arange(T, device=device)
    q = rows.to(torch.int64)[:, None]
    k = keys[None, :]

    def token_major(x):  # frame-major position f*S + p -> token-major p*F + f
        f = torch.div(x, frame_size, rounding_mode="floor")
        p = x - f * frame_size
        return p * num_frame + f

    if mask_name == "temporal":
        qm, km = token_major(torch.clamp(q, max=V - 1)), token_major(torch.clamp(k, max=V - 1))
    elif mask_name == "spatial":
        qm, km = q, k
    else:
        raise ValueError(f"unknown mask {mask_name!r}")
    if model == "hunyuan":
        m = _band(qm, km, frame_size, 1.5)
        video = (q < V) & (k < V)
        return torch.where(video, m, torch.ones_like(m))  # text rows and columns are all ones
    if model == "wan":
        return _band(qm, km, frame_size, 2.0) | (km < frame_size)  # + first-frame sink
    raise ValueError(f"unknown model {model!r}")


def sample_mse(query, key, value, *, model="hunyuan", context_length=0, num_frame=1, frame_size=None,
               num_sampled_rows=32, sample_mse_max_row=10000, masks=MASKS):
    """Per-head MSE of each emulated sparse mask against full attention on
    sampled query rows; [len(masks), cfg, H] in the query dtype."""
    n = min(num_sampled_rows, query.size(2))
    sampled_rows = torch.randint(low=0, high=sample_mse_max_row, size=(n,))  # CPU generator, like the reference
    return sample_mse_rows(query, key, value, sampled_rows, model=model, context_length=context_length,
                           num_frame=num_frame, frame_size=frame_size, masks=masks)


def sample_mse_rows(query, key, value, sampled_rows, *, model="hunyuan", context_length=0, num_frame=1,
                    frame_size=None, masks=MASKS):
    """sample_mse on the given sampled rows (the reference's steps after its
    random draw, hyvideo/attention.py:388-405), on the tensors' device."""
    cfg, num_heads, seq_len, dim = query.size()
    if frame_size is None:
        frame_size = (seq_len - (context_length if model == "hunyuan" else 0)) // num_frame
    rows_dev = sampled_rows.to(query.device)
    sampled_q = query[:, :, rows_dev, :]
    scores = torch.matmul(sampled_q, key.transpose(-2, -1)) / (dim ** 0.5)
    golden = torch.matmul(F.softmax(scores, dim=-1), value)
    out = torch.zeros(len(masks), cfg, num_heads, device=query.device, dtype=query.dtype)
    for i, name in enumerate(masks):
        m = emulated_mask_rows(rows_dev, name, model, context_length, num_frame, frame_size)
        masked = scores.masked_fill(~m, float("-inf"))
        hs = torch.matmul(F.softmax(masked, dim=-1), value)
        out[i] = torch.mean((hs - golden) ** 2, dim=(2, 3))
    return out


def classify_heads(query, key, value, **kw) -> torch.Tensor:
    """best_mask_idx [cfg, H]: 0 = spatial head, 1 = temporal head."""
    return torch.argmin(sample_mse(query, key, value, **kw), dim=0)
