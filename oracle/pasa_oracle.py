"""CPU restatement of the reference PASA forward (``pisa_pg_attention``).

TEST INFRASTRUCTURE ONLY.  This module is the parity checker for the CUDA
path in ``pasa_b200``.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it; the
product path never calls it and has no CPU fallback.

Every function restates one piece of ``svg/kernels/triton/group_pisa_attention.py``
(ZHANGWENTAI/PASA) with numpy, keeping the reference's rounding points:

* values travel as float32 arrays; for ``dtype="bf16"`` every place where the
  reference stores or casts to bfloat16 applies :func:`bf16_round`
  (round-to-nearest-even), so the arrays hold exactly representable bf16 values;
* matrix products accumulate in float32 (the reference's ``tl.dot`` with an
  fp32 accumulator and ``torch.einsum`` on bf16, which cuBLAS accumulates in
  fp32 and rounds once);
* ``tl.sum`` over block rows: in fp32 the reference's CPU run (Triton
  interpreter, ``np.sum`` over axis 0) adds the 64 rows in order, which is
  what :func:`_block_row_sum` does for fp32.  For bf16 Triton 3.x adds in
  the element type (``triton/language/standard.py:_pick_sum_dtype`` does not
  widen floats), every partial sum rounded to bf16, in an order the
  reference leaves to the compiler; the CUDA path and this oracle both fix
  it to the halving tree ``x[r] + x[r + n/2]``.

Parity pinning: the fp32 path is checked against the reference itself (run
through the Triton interpreter on CPU, fixtures in ``tests/golden/``).  The
reference's bf16 path cannot run on CPU (the interpreter stores bf16 as raw
uint16 and sums bit patterns), so bf16 rounding points are restated from the
source lines cited below.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

LOG2E = 1.44269504  # group_pisa_attention.py:162 (sm_scale = scale * 1.44269504)


# ---------------------------------------------------------------------------
# rounding helpers
# ---------------------------------------------------------------------------
def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even); float32 out."""
    a = np.ascontiguousarray(x, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    bias = np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))
    r = ((u + bias) & np.uint64(0xFFFF0000)).astype(np.uint32)
    # NaN stays NaN (not produced by this path, kept for safety)
    r = np.where(np.isnan(a), np.uint32(0x7FC00000), r)
    return r.view(np.float32).reshape(a.shape)


def to_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    return bf16_round(x) if dtype == "bf16" else x


def _f32(x) -> np.float32:
    return np.float32(x)


# ---------------------------------------------------------------------------
# shapes
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class Geometry:
    """Derived sizes, as in group_pisa_attention.py:341-347 and :373."""

    B: int
    H: int
    T: int
    D: int
    block: int = 64
    group: int = 32

    @property
    def NT(self) -> int:  # triton.cdiv(T, block_size)  (:345)
        return -(-self.T // self.block)

    @property
    def NG(self) -> int:  # compute_h_group: ceil(NT / group)  (:294-299)
        return -(-self.NT // self.group)

    @property
    def last_len(self) -> int:  # last_chunk_len  (:191)
        return self.T - (self.NT - 1) * self.block

    def top_k(self, density: float) -> int:  # :373
        return min(max(1, int(density * self.NT)), self.NT)


def _blocks(x: np.ndarray, block: int) -> np.ndarray:
    """[BH, T, D] -> [BH, NT, block, D] with zero rows past T (TMA zero fill)."""
    BH, T, D = x.shape
    NT = -(-T // block)
    pad = NT * block - T
    if pad:
        x = np.concatenate([x, np.zeros((BH, pad, D), np.float32)], axis=1)
    return x.reshape(BH, NT, block, D)


def _block_row_sum(xb: np.ndarray, dtype: str) -> np.ndarray:
    """tl.sum(b_x, axis=0) over the block rows (group_pisa_attention.py:101-103).

    fp32: sequential row order (the reference's interpreter run).
    bf16: halving tree, each partial sum rounded to bf16.
    """
    if dtype == "fp32":
        acc = xb[..., 0, :].astype(np.float32).copy()
        for r in range(1, xb.shape[-2]):
            acc = (acc + xb[..., r, :]).astype(np.float32)
        return acc
    y = xb.astype(np.float32)
    n = y.shape[-2]
    while n > 1:
        h = n // 2
        y = bf16_round(y[..., :h, :] + y[..., h:n, :])
        n = h
    return y[..., 0, :]


# ---------------------------------------------------------------------------
# K1: fused_chunk_reduce  (group_pisa_attention.py:75-129, :268-288)
# ---------------------------------------------------------------------------
def chunk_reduce(q, k, v, block: int = 64, dtype: str = "bf16"):
    """Per (bh, block): qc, kc (means), vc (sum), hc, h_norm.

    q, k, v: [BH, T, D] float32 arrays holding values of ``dtype``.
    Returns qc, kc, vc [BH, NT, D]; hc [BH, NT, D, D]; h_norm [BH, NT] (fp32).
    """
    BH, T, D = q.shape
    qb, kb, vb = (_blocks(np.asarray(a, np.float32), block) for a in (q, k, v))
    NT = qb.shape[1]
    lens = np.minimum(block, T - np.arange(NT) * block).astype(np.float32)  # BLOCK_SIZE (:91)

    sq = _block_row_sum(qb, dtype)
    sk = _block_row_sum(kb, dtype)
    sv = _block_row_sum(vb, dtype)
    qc_f = (sq / lens[None, :, None]).astype(np.float32)  # bf16/int -> fp32 divide (:101)
    kc_f = (sk / lens[None, :, None]).astype(np.float32)  # (:102)
    qc = to_dtype(qc_f, dtype)  # store in q dtype (:117)
    kc = to_dtype(kc_f, dtype)  # (:118)
    vc = to_dtype(sv, dtype)  # (:119), sum kept in v dtype

    # hc = k^T v (fp32 accumulate) - kc (fp32) outer vc   (:106-107)
    ktv = np.matmul(np.swapaxes(kb, -1, -2), vb).astype(np.float32)
    hc_f = (ktv - kc_f[..., :, None] * sv[..., None, :]).astype(np.float32)
    norm_sq = np.sum((hc_f * hc_f).reshape(BH, NT, D * D), axis=-1, dtype=np.float32)  # (:110)
    h_norm = np.sqrt(norm_sq).astype(np.float32)  # (:287)
    hc = to_dtype(hc_f, dtype)  # (:125)
    return qc, kc, vc, hc, h_norm


def group_mean(hc: np.ndarray, group: int = 32, dtype: str = "bf16") -> np.ndarray:
    """compute_h_group (group_pisa_attention.py:291-301): zero-pad NT to a
    multiple of ``group`` and take the mean over each run of ``group`` blocks
    (the divisor is always ``group``).  torch's mean accumulates bf16 in fp32
    and rounds once."""
    BH, NT, D, E = hc.shape
    pad = (group - NT % group) % group
    if pad:
        hc = np.concatenate([hc, np.zeros((BH, pad, D, E), np.float32)], axis=1)
    NG = hc.shape[1] // group
    s = hc.reshape(BH, NG, group, D, E).astype(np.float64).sum(axis=2)
    return to_dtype((s / group).astype(np.float32), dtype)


# ---------------------------------------------------------------------------
# covariance-aware top-k selection  (group_pisa_attention.py:365-375)
# ---------------------------------------------------------------------------
def block_scores(qc, kc, h_norm, scale: float, dtype: str = "bf16",
                 use_cov_bias: bool = True, noise=None) -> np.ndarray:
    """score[bh, i, j] in float32 (bf16-valued when use_cov_bias is False)."""
    kcs = to_dtype(kc * _f32(scale), dtype)  # kc * scale in the tensor dtype (:365)
    dots = np.matmul(qc, np.swapaxes(kcs, -1, -2)).astype(np.float32)
    score = to_dtype(dots, dtype)  # einsum output in the input dtype
    if use_cov_bias:
        log_bias = np.log((h_norm + _f32(1e-6)).astype(np.float32)).astype(np.float32)  # (:368)
        if noise is not None:
            log_bias = (log_bias + noise).astype(np.float32)  # (:370)
        score = (score + log_bias[:, None, :]).astype(np.float32)  # (:371)
    return score


def topk_desc(score: np.ndarray, k: int) -> np.ndarray:
    """torch.topk(score, k, dim=-1).indices (sorted, largest first).

    Equal scores are ordered by ascending block index (torch leaves the order
    of exact ties unspecified)."""
    NTk = score.shape[-1]
    idx = np.broadcast_to(np.arange(NTk), score.shape)
    order = np.lexsort((idx, -score.astype(np.float64)), axis=-1)
    return order[..., :k].astype(np.int32)


def select_blocks(qc, kc, h_norm, scale, top_k, dtype="bf16", use_cov_bias=True, noise=None):
    score = block_scores(qc, kc, h_norm, scale, dtype, use_cov_bias, noise)
    return topk_desc(score, top_k), score


# ---------------------------------------------------------------------------
# K2: pisa_pg_fwd_kernel  (group_pisa_attention.py:136-262)
# ---------------------------------------------------------------------------
def attention(q, k, v, kc, vc, h_group, indices, scale: float, T: int,
              block: int = 64, group: int = 32, dtype: str = "bf16",
              qblocks=None, rescale_gl: bool = False, first_order: str = "reference") -> np.ndarray:
    """Exact attention over the selected blocks, zero-order + per-group
    first-order correction over the rest, one online-softmax pass.

    All query blocks of a head advance together (vectorised over the query
    block axis); each query block follows the reference's own loop order.
    ``qblocks`` optionally restricts the computation to a subset of query
    block indices (used for bounded CPU timing samples); rows of other blocks
    are returned as zeros.  ``rescale_gl=True`` is a deliberately WRONG
    variant (g_l rescaled with the running max) used only by tests to show
    that a fixture exercises the reference's unrescaled g_l.
    ``first_order="rounded_operand"`` is a measuring variant, not the
    reference: it forms the first-order term the way the tensor-core kernel
    does, as bf16(q * bf16(w)) times H_g with w = scale * (sum of the group's
    probabilities), instead of (q H_g) * w in fp32 (:251-253); tests use it
    to size that rounding against the tolerance.
    """
    BH, _, D = q.shape
    qb, kb, vb = (_blocks(np.asarray(a, np.float32), block) for a in (q, k, v))
    NT = qb.shape[1]
    NS = indices.shape[-1]
    NG = h_group.shape[1]
    last_len = T - (NT - 1) * block
    scale32 = _f32(scale)
    sm_scale = _f32(scale32 * _f32(LOG2E))  # :162
    sel_q = np.arange(NT) if qblocks is None else np.asarray(qblocks)
    nq = len(sel_q)
    out = np.zeros((BH, NT, block, D), np.float32)

    key_valid = (np.arange(NT * block) < T).reshape(NT, block)
    lens_all = np.full(NG * group, block, np.float32)
    lens_all[NT - 1] = last_len  # :220
    pad_rows = NG * group - NT

    for bh in range(BH):
        Q = qb[bh, sel_q]  # [nq, 64, D]
        idx = indices[bh, sel_q].astype(np.int64)  # [nq, NS]
        acc = np.zeros((nq, block, D), np.float32)
        l_i = np.zeros((nq, block), np.float32)
        m_i = np.full((nq, block), -np.inf, np.float32)

        # Phase 1: exact attention (:170-186)
        for i in range(NS):
            j = idx[:, i]
            Kj = kb[bh, j]  # [nq, 64, D]
            Vj = vb[bh, j]
            s = (np.matmul(Q, np.swapaxes(Kj, -1, -2)).astype(np.float32) * sm_scale).astype(np.float32)
            s = np.where(key_valid[j][:, None, :], s, np.float32(-np.inf))
            new_m = np.maximum(m_i, s.max(axis=-1))
            alpha = np.exp2(m_i - new_m).astype(np.float32)
            p = np.exp2(s - new_m[..., None]).astype(np.float32)
            l_i = (l_i * alpha + p.sum(axis=-1, dtype=np.float32)).astype(np.float32)
            pv = np.matmul(to_dtype(p, dtype), Vj).astype(np.float32)
            acc = (acc * alpha[..., None] + pv).astype(np.float32)
            m_i = new_m

        # Phase 2: zero-order + per-group first-order (:191-253)
        selected = np.zeros((nq, NG * group), bool)
        np.put_along_axis(selected, idx, True, axis=1)
        kcp = np.concatenate([kc[bh], np.zeros((pad_rows, D), np.float32)], axis=0)
        vcp = np.concatenate([vc[bh], np.zeros((pad_rows, D), np.float32)], axis=0)
        g_l = np.zeros((nq, block), np.float32)
        for g in range(NG):
            cols = slice(g * group, (g + 1) * group)
            s = (np.matmul(Q, kcp[cols].T).astype(np.float32) * sm_scale).astype(np.float32)
            valid = (np.arange(g * group, (g + 1) * group) < NT)[None, :] & ~selected[:, cols]
            s = np.where(valid[:, None, :], s, np.float32(-np.inf))
            new_m = np.maximum(m_i, s.max(axis=-1))
            alpha = np.exp2(m_i - new_m).astype(np.float32)
            acc = (acc * alpha[..., None]).astype(np.float32)
            l_i = (l_i * alpha).astype(np.float32)
            if rescale_gl:
                g_l = (g_l * alpha).astype(np.float32)
            m_i = new_m
            p = np.exp2(s - m_i[..., None]).astype(np.float32)
            acc = (acc + np.matmul(to_dtype(p, dtype), vcp[cols]).astype(np.float32)).astype(np.float32)
            # g_l is accumulated without the alpha rescale, exactly as :242-243
            g_l = (g_l + (p * lens_all[cols]).sum(axis=-1, dtype=np.float32)).astype(np.float32)
            gps = p.sum(axis=-1, dtype=np.float32)  # :252
            if first_order == "rounded_operand":
                w = to_dtype((gps * scale32).astype(np.float32), "bf16")
                u = to_dtype((Q * w[..., None]).astype(np.float32), "bf16")
                acc = (acc + np.matmul(u, h_group[bh, g]).astype(np.float32)).astype(np.float32)
            else:
                r = np.matmul(Q, h_group[bh, g]).astype(np.float32)  # :251
                acc = (acc + r * (gps * scale32)[..., None]).astype(np.float32)  # :253

        # Final (:258-262)
        l_i = (l_i + g_l).astype(np.float32)
        out[bh, sel_q] = to_dtype(acc / l_i[..., None], dtype)

    return out.reshape(BH, NT * block, D)[:, :T]


# ---------------------------------------------------------------------------
# the whole op  (pisa_pg_attention, group_pisa_attention.py:307-398)
# ---------------------------------------------------------------------------
def pisa_pg_attention(q, k, v, density=0.15, block_size=64, group_size=32, scale=None,
                      use_cov_bias=True, noise=None, dtype="bf16", return_all=False):
    """q, k, v: [B, H, T, D] float32 arrays holding ``dtype`` values.

    ``noise`` stands in for ``torch.randn_like(log_bias)`` when the caller
    asked for ``use_random`` ([B*H, NT] float32)."""
    B, H, T, D = q.shape
    geo = Geometry(B, H, T, D, block_size, group_size)
    scale = D ** -0.5 if scale is None else scale
    qf, kf, vf = (np.asarray(a, np.float32).reshape(B * H, T, D) for a in (q, k, v))
    qc, kc, vc, hc, h_norm = chunk_reduce(qf, kf, vf, block_size, dtype)
    h_group = group_mean(hc, group_size, dtype)
    top_k = geo.top_k(density)
    indices, score = select_blocks(qc, kc, h_norm, scale, top_k, dtype, use_cov_bias, noise)
    o = attention(qf, kf, vf, kc, vc, h_group, indices, scale, T, block_size, group_size, dtype)
    o = o.reshape(B, H, T, D)
    if return_all:
        return dict(o=o, qc=qc, kc=kc, vc=vc, hc=hc, h_norm=h_norm, h_group=h_group,
                    indices=indices, score=score, top_k=top_k)
    return o


def exact_flops(geo: Geometry, top_k: int) -> float:
    """F_exact = 4 * B*H * NT * NS * block^2 * D (selected 64x64 blocks only)."""
    return 4.0 * geo.B * geo.H * geo.NT * top_k * geo.block * geo.block * geo.D


def corr_flops(geo: Geometry) -> float:
    """Phase-2 work: B*H*NT*NG*(4*block*group*D + 2*block*D^2)."""
    return float(geo.B * geo.H * geo.NT * geo.NG) * (
        4 * geo.block * geo.group * geo.D + 2 * geo.block * geo.D * geo.D)


def cosine(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (math.sqrt(a @ a) * math.sqrt(b @ b) + 1e-300))
