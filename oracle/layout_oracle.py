"""CPU restatements for the token-layout side of the hot path.

TEST INFRASTRUCTURE ONLY (imported by tests/ only; never by the product).

* ``dense_attention_mask`` restates ``get_attention_mask`` with its literal
  block double loop: svg/models/hyvideo/utils.py:48-94 (model="hunyuan", text
  tokens at the tail) and svg/models/wan/utils.py:63-110 (model="wan", with
  a first-frame sink).  It is used to check the closed-form masks of
  ``pasa_b200.classify``.
* ``place_reference`` restates the torch references of the placement
  kernels: ``hunyuan_token_reorder_to_token_major`` /
  ``..._to_frame_major`` and ``ref_hunyuan_sparse_head_placement`` /
  ``ref_hunyuan_hidden_states_placement``
  (svg/models/hyvideo/placement.py:6-31, :156-184, :390-401).  With
  context_length 0 the reference's ``[:-0]`` slice selects nothing; the
  kernel formula at placement.py:73-78 (no text tail) is used instead.
"""
from __future__ import annotations

import math

import torch


def dense_attention_mask(mask_name, context_length, num_frame, frame_size, model="hunyuan"):
    V = num_frame * frame_size
    if model == "hunyuan":
        T = context_length + V
        attention_mask = torch.zeros((T, T))
        pixel = torch.zeros((V, V), dtype=torch.bool)
        block_size, block_thres = 128, frame_size * 1.5
        num_block = math.ceil(V / block_size)
        for i in range(num_block):
            for j in range(num_block):
                if abs(i - j) < block_thres // block_size:
                    pixel[i * block_size:(i + 1) * block_size, j * block_size:(j + 1) * block_size] = 1
        if mask_name != "spatial":
            pixel = pixel.reshape(frame_size, num_frame, frame_size, num_frame).permute(1, 0, 3, 2).reshape(V, V)
        attention_mask[:V, :V] = pixel
        attention_mask[V:, :] = 1
        attention_mask[:, V:] = 1
        return attention_mask.bool()
    # wan
    pixel = torch.zeros((V, V), dtype=torch.bool)
    pixel[:, :frame_size] = 1  # first-frame sink
    block_size, block_thres = 128, frame_size * 2
    num_block = math.ceil(V / block_size)
    for i in range(num_block):
        for j in range(num_block):
            if abs(i - j) < block_thres // block_size:
                pixel[i * block_size:(i + 1) * block_size, j * block_size:(j + 1) * block_size] = 1
    if mask_name != "spatial":
        pixel = pixel.reshape(frame_size, num_frame, frame_size, num_frame).permute(1, 0, 3, 2).reshape(V, V)
    return pixel


def place_reference(x, best_mask_idx, context_length, num_frame, frame_size, inverse=False):
    """Placement of [cfg, H, T, D] by the reference's torch formulas."""
    out = x.clone()
    V = num_frame * frame_size
    for c in range(x.shape[0]):
        for h in range(x.shape[1]):
            if int(best_mask_idx[c, h]) != 1:
                continue
            video = x[c, h, :V]
            if not inverse:  # frame-major -> token-major
                out[c, h, :V] = video.reshape(num_frame, frame_size, -1).transpose(0, 1).reshape(V, -1)
            else:            # token-major -> frame-major
                out[c, h, :V] = video.reshape(frame_size, num_frame, -1).transpose(0, 1).reshape(V, -1)
    return out
