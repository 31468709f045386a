"""Spatial / temporal head classification on the GPU (the SVG profiling
step that decides which heads the token placement reorders).

``sample_mse`` keeps the meaning of the reference's
``sample_mse`` (svg/models/hyvideo/attention.py:381-405; Wan twin
svg/models/wan/attention.py:264-288): for ``num_sampled_rows`` query rows
drawn with ``torch.randint(0, sample_mse_max_row, (n,))`` on the CPU
generator (the reference's own draw), the mean squared difference between
attention under each emulated mask (spatial, temporal; get_attention_mask,
svg/models/hyvideo/utils.py:48-94 and svg/models/wan/utils.py:63-110) and
full attention, per head: ``[2, cfg, H]`` in the query dtype.  The work
runs in ``pasa_sample_mse`` (csrc/classify.cu), which evaluates the masks
in closed form instead of building dense T x T tensors.  ``classify_heads``
returns the argmin, the ``best_mask_idx`` the placement functions consume
(0 spatial, 1 temporal).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .ops import _dtype_code, _stream_ptr

_MODELS = {"hunyuan": _lib.MODEL_HUNYUAN, "wan": _lib.MODEL_WAN}


def _run(query, key, value, model, context_length, num_frame, frame_size, num_sampled_rows, sample_mse_max_row,
         rows):
    for name, t in (("query", query), ("key", key), ("value", value)):
        if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dim() != 4:
            raise ValueError(f"{name} must be a [cfg, H, T, D] CUDA tensor")
    if key.shape != query.shape or value.shape != query.shape:
        raise ValueError("query, key and value must have one shape")
    if key.dtype != query.dtype or value.dtype != query.dtype:
        raise ValueError("query, key and value must have one dtype")
    if model not in _MODELS:
        raise ValueError(f"model is one of {sorted(_MODELS)}")
    query, key, value = query.contiguous(), key.contiguous(), value.contiguous()
    cfg, H, T, D = query.shape
    ctx = context_length if model == "hunyuan" else 0
    if frame_size is None:
        frame_size = (T - ctx) // num_frame
    if rows is None:
        n = min(num_sampled_rows, T)
        rows = torch.randint(low=0, high=sample_mse_max_row, size=(n,))  # CPU generator, as the reference
    rows = rows.to(device="cpu", dtype=torch.int64).contiguous()
    dcode = _dtype_code(query)
    lib = _lib.load()
    with torch.cuda.device(query.device):
        nb = ctypes.c_size_t()
        _lib.check("pasa_sample_mse_workspace_size",
                   lib.pasa_sample_mse_workspace_size(cfg * H, T, D, ctypes.byref(nb)))
        ws = torch.empty(nb.value, dtype=torch.uint8, device=query.device)
        mse = torch.empty((2, cfg, H), dtype=query.dtype, device=query.device)
        best = torch.empty((cfg, H), dtype=torch.int32, device=query.device)
        _lib.check("pasa_sample_mse", lib.pasa_sample_mse(
            _stream_ptr(query.device), query.data_ptr(), key.data_ptr(), value.data_ptr(), cfg, H, T, D, dcode,
            rows.data_ptr(), rows.numel(), _MODELS[model], ctx, num_frame, frame_size, ws.data_ptr(), nb.value,
            mse.data_ptr(), best.data_ptr()))
    return mse, best


def sample_mse(query, key, value, *, model="hunyuan", context_length=0, num_frame=1, frame_size=None,
               num_sampled_rows=32, sample_mse_max_row=10000, rows=None):
    """Per-head MSE of the spatial and temporal emulated masks against full
    attention on sampled query rows: ``[2, cfg, H]`` in the query dtype.
    ``rows`` (CPU int64, at most 32) replaces the random draw when given."""
    return _run(query, key, value, model, context_length, num_frame, frame_size, num_sampled_rows,
                sample_mse_max_row, rows)[0]


def classify_heads(query, key, value, **kw) -> torch.Tensor:
    """best_mask_idx [cfg, H] (int64, as torch.argmin): 0 spatial head, 1
    temporal head; equal MSEs pick spatial, as torch.argmin picks the first."""
    args = [kw.pop(n, d) for n, d in (("model", "hunyuan"), ("context_length", 0), ("num_frame", 1),
                                       ("frame_size", None), ("num_sampled_rows", 32),
                                       ("sample_mse_max_row", 10000), ("rows", None))]
    if kw:
        raise TypeError(f"unexpected arguments {sorted(kw)}")
    return _run(query, key, value, *args)[1].long()
