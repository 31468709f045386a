"""CPU restatement of the DiT row ops around the attention op.

TEST INFRASTRUCTURE ONLY.  This module checks the CUDA row kernels
(``pasa_dit_row_norm``, ``pasa_dit_qkv_rope``); only ``tests/`` may import it,
and the product path never calls it.

Restated from ZHANGWENTAI/PASA:

* LayerNorm without / with affine: ``_layer_norm_noparam_fwd_fused``
  (svg/kernels/triton/layernorm.py:113-155) and ``_layer_norm_param_fwd_fused``
  (:13-58): ``mean = sum(x) / N``, ``var = sum((x - mean)^2) / N``,
  ``rstd = 1 / sqrt(var + eps)``, ``(x - mean) * rstd [* w + b]``, fp32;
* RMSNorm: ``_rms_norm_fwd_fused`` (rmsnorm.py:8-48): ``var = sum(x*x) / N``,
  ``x * rstd * w``, stored in the input dtype;
* modulation ``x * (1 + scale) + shift`` (modulate.py:12-42) and gated
  residual ``r + x * gate`` (modulate.py:90-122), fp32, cast to the output
  dtype;
* the Wan block's chaining and casts (svg/models/wan/custom_models.py:24-113);
* the rotary embedding's torch path (svg/models/wan/attention.py:49-57): bf16
  -> float64 pairs times ``cos + i sin`` -> the input dtype (torch casts
  float64 to bf16 through float32).

Every fp32 operation is a separate, correctly rounded numpy float32
operation (no fused multiply-add).  Sums run in one of two orders:

* ``order="kernel"``: the CUDA kernels' order -- a 128-thread CTA per row,
  thread t adding the 8 elements of each of its 16-byte vectors
  j = t, t + 128, ... in sequence, an xor butterfly over each warp of 32, then
  the four warp sums in order.  Results then match the GPU bit for bit.
* ``order="reference"``: the Triton interpreter's order -- the row padded with
  zeros to the next power of two and reduced by ``np.sum`` (what ``tl.sum``
  becomes under ``TRITON_INTERPRET=1``).  This is the order of the golden
  fixtures in ``tests/golden/dit_rows.npz``, made by running the reference's
  kernels.
"""
from __future__ import annotations

import numpy as np

from .pasa_oracle import bf16_round

ROW_THREADS = 128
F32 = np.float32


def _sum_kernel_order(vals: np.ndarray) -> np.ndarray:
    """vals [rows, C] float32 -> [rows] float32, the CUDA kernels' order."""
    rows, C = vals.shape
    assert C % 8 == 0
    nvec = C // 8
    V = -(-nvec // ROW_THREADS)
    acc = np.zeros((rows, ROW_THREADS), dtype=F32)
    vecs = vals.reshape(rows, nvec, 8)
    for i in range(V):
        js = np.arange(ROW_THREADS) + i * ROW_THREADS
        live = js < nvec
        for e in range(8):
            add = np.zeros((rows, ROW_THREADS), dtype=F32)
            add[:, live] = vecs[:, js[live], e]
            # threads whose vector is past the row add nothing (x + 0 == x
            # for the finite sums here)
            acc = np.where(live[None, :], (acc + add).astype(F32), acc)
    lanes = acc.reshape(rows, ROW_THREADS // 32, 32)
    idx = np.arange(32)
    for off in (16, 8, 4, 2, 1):
        lanes = (lanes + lanes[:, :, idx ^ off]).astype(F32)
    warp = lanes[:, :, 0]
    t = warp[:, 0].copy()
    for w in range(1, ROW_THREADS // 32):
        t = (t + warp[:, w]).astype(F32)
    return t


def _sum_reference_order(vals: np.ndarray) -> np.ndarray:
    rows, C = vals.shape
    n2 = 1 << max(0, (C - 1).bit_length())
    pad = np.zeros((rows, n2), dtype=F32)
    pad[:, :C] = vals
    return np.sum(pad, axis=1, dtype=F32)


def row_sum(vals: np.ndarray, order: str) -> np.ndarray:
    vals = np.ascontiguousarray(vals, dtype=F32)
    if order == "kernel":
        return _sum_kernel_order(vals)
    if order == "reference":
        return _sum_reference_order(vals)
    raise ValueError(order)


def _rstd(var: np.ndarray, eps: float) -> np.ndarray:
    return (F32(1.0) / np.sqrt((var + F32(eps)).astype(F32))).astype(F32)


def padded_cols(C: int) -> int:
    """Columns of the reference's Triton row programs: C padded to a power of two."""
    return 1 << max(0, (C - 1).bit_length())


def layer_norm(x, eps, weight=None, bias=None, center=True, order="kernel", pad_variance=False):
    """Normalised rows of float32 ``x`` [rows, C] (LayerNorm, or RMSNorm when
    ``center`` is False), affine when given; float32 out, unrounded.

    ``pad_variance`` reproduces the reference's Triton LayerNorm
    (layernorm.py:40-42, :138-140): its rows are padded with zeros to
    ``padded_cols(C)`` columns and the padding's ``(0 - mean)^2`` is summed into
    the variance, which is still divided by C.  The torch LayerNorm the block
    falls back to (custom_models.py:45, FP32LayerNorm) has no such term."""
    x = np.asarray(x, dtype=F32)
    rows, C = x.shape
    if center:
        mean = (row_sum(x, order) / F32(C)).astype(F32)[:, None]
    else:
        mean = np.zeros((rows, 1), dtype=F32)
    d = (x - mean).astype(F32)
    pad = padded_cols(C) - C if (pad_variance and center) else 0
    if pad and order == "reference":
        dp = np.concatenate([d, np.broadcast_to((F32(0) - mean).astype(F32), (rows, pad))], axis=1)
        var = (np.sum((dp * dp).astype(F32), axis=1, dtype=F32) / F32(C)).astype(F32)
    else:
        ssq = row_sum((d * d).astype(F32), order)
        if pad:
            m = mean[:, 0]
            ssq = (ssq + (F32(pad) * (m * m).astype(F32)).astype(F32)).astype(F32)
        var = (ssq / F32(C)).astype(F32)
    y = (d * _rstd(var, eps)[:, None]).astype(F32)
    if weight is not None:
        y = (y * np.asarray(weight, F32)[None, :]).astype(F32)
    if bias is not None:
        y = (y + np.asarray(bias, F32)[None, :]).astype(F32)
    return y


def modulate(x, scale, shift):
    """x * (1 + scale) + shift, float32 (modulate.py:37)."""
    one = (F32(1.0) + np.asarray(scale, F32)).astype(F32)
    return ((x * one).astype(F32) + np.asarray(shift, F32)).astype(F32)


def gate_residual(r, x, gate):
    """r + x * gate, float32 (modulate.py:117)."""
    return (np.asarray(r, F32) + (np.asarray(x, F32) * np.asarray(gate, F32)).astype(F32)).astype(F32)


def row_norm(x, eps, *, add=None, gate=None, weight=None, bias=None, scale=None, shift=None, center=True,
             order="kernel", pad_variance=False):
    """What pasa_dit_row_norm computes on bf16-valued float32 rows [rows, C]:
    returns (x', y), both bf16-valued float32."""
    x = np.asarray(x, F32)
    if add is not None:
        if gate is not None:
            x = bf16_round(gate_residual(x, add, gate))
        else:
            x = bf16_round((x + np.asarray(add, F32)).astype(F32))
    y = layer_norm(x, eps, weight, bias, center, order, pad_variance)
    if scale is not None:
        y = modulate(y, scale, shift)
    return x, bf16_round(y)


def rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Rotate the (2i, 2i+1) pairs of bf16-valued ``x`` [..., L, D] by float64
    ``cos``/``sin`` [L, D/2]: float64 complex multiply, then float64 ->
    float32 -> bf16 (attention.py:49-57 with torch's cast)."""
    xf = np.asarray(x, np.float64)
    a, b = xf[..., 0::2], xf[..., 1::2]
    re = a * cos - b * sin
    im = a * sin + b * cos
    out = np.empty_like(xf)
    out[..., 0::2], out[..., 1::2] = re, im
    return bf16_round(out.astype(F32))


def qkv_rope(xq, xk, xv, wq, wk, cos, sin, heads: int, eps: float, order="kernel"):
    """What pasa_dit_qkv_rope computes: xq/xk/xv bf16-valued [L, C] of one
    batch entry -> q, k, v [heads, L, D] (RMSNorm rounded to bf16, rotary in
    float64, bf16 out)."""
    L, C = xq.shape
    D = C // heads

    def norm(x, w):
        n = bf16_round(layer_norm(x, eps, w, None, center=False, order=order))
        n = n.reshape(L, heads, D).transpose(1, 0, 2)
        return rope(n, cos, sin) if cos is not None else n

    q = norm(xq, wq)
    k = norm(xk, wk) if xk is not None else None
    v = np.asarray(xv, F32).reshape(L, heads, D).transpose(1, 0, 2).copy() if xv is not None else None
    return q, k, v


def rope_table(frames: int, height: int, width: int, head_dim: int, theta: float = 10000.0):
    """float64 cos, sin [frames*height*width, head_dim/2] of the Wan 3D rotary
    embedding: the pairs split over (frame, row, column) as
    head_dim - 4*(head_dim//6), 2*(head_dim//6), 2*(head_dim//6) channels, each
    axis with frequencies theta^(-2i/d) (diffusers' WanRotaryPosEmbed with
    float64 frequencies, which the reference model calls at
    custom_models.py:143; diffusers is not vendored in the reference)."""
    dims = [head_dim - 4 * (head_dim // 6), 2 * (head_dim // 6), 2 * (head_dim // 6)]
    f, h, w = np.meshgrid(np.arange(frames), np.arange(height), np.arange(width), indexing="ij")
    angles = []
    for pos, d in zip((f, h, w), dims):
        inv = 1.0 / theta ** (np.arange(0, d, 2, dtype=np.float64) / d)
        angles.append(pos.reshape(-1, 1).astype(np.float64) * inv[None, :])
    ang = np.concatenate(angles, axis=1)
    return np.cos(ang), np.sin(ang)
