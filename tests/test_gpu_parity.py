"""Parity of the CUDA path (through the C ABI) with the reference and the
CPU oracle.

fp32: against the reference's own outputs (tests/golden, bit-exact for block
statistics and block indices).  bf16: against the oracle's restatement of the
reference's bf16 rounding points — block statistics and indices bit-exact,
outputs within the north-star tolerance (max-abs 2e-2, cosine >= 0.999).
"""
import numpy as np
import pytest
import torch

from conftest import golden_cases, load_golden
from oracle import pasa_oracle as O
from pasa_b200 import _lib, ops

pytestmark = pytest.mark.gpu

CASES = sorted(golden_cases())
TOL_ABS = 2e-2   # north star: bf16 output max-abs error
TOL_COS = 0.999  # north star: cosine similarity


def _pad_rows(a, ntp):
    a = np.asarray(a, np.float32)
    pad = ntp - a.shape[1]
    if pad:
        a = np.concatenate([a, np.zeros((a.shape[0], pad) + a.shape[2:], np.float32)], axis=1)
    return a


def _dev(a, dtype, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device=device, dtype=dtype)


def _np(t):
    return t.detach().float().cpu().numpy()


def _stages_for(q, st_like=None):
    B, H, T, D = q.shape
    return st_like


# ---------------------------------------------------------------------------
# fp32: the reference's own outputs
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("name", CASES)
def test_fp32_stages_against_reference(name, cuda_device):
    case, g, q, k, v = load_golden(name)
    B, H, T, D = q.shape
    qd, kd, vd = (t.to(cuda_device) for t in (q, k, v))
    noise = _dev(g["noise"], torch.float32, cuda_device) if "noise" in g else None
    o, st = ops.run_stages(qd, kd, vd, density=case["density"], use_cov_bias=case.get("use_cov_bias", True),
                           noise=noise)
    torch.cuda.synchronize()
    NT = st.NT
    # block statistics: bit-exact (the reference adds block rows in order)
    np.testing.assert_array_equal(_np(st.qc)[:, :NT], g["qc"])
    np.testing.assert_array_equal(_np(st.kc)[:, :NT], g["kc"])
    np.testing.assert_array_equal(_np(st.vc)[:, :NT], g["vc"])
    assert not _np(st.qc)[:, NT:].any() and not _np(st.vc)[:, NT:].any()
    np.testing.assert_allclose(_np(st.h_norm), g["h_norm"], rtol=1e-5)
    np.testing.assert_allclose(_np(st.h_group), g["h_group"], rtol=0, atol=1e-5)
    # top-k indices, in order: bit-exact
    np.testing.assert_array_equal(st.indices.cpu().numpy(), g["indices"])
    np.testing.assert_allclose(_np(o), g["o"], rtol=0, atol=2e-5)
    ops.check_device_errors(st)


@pytest.mark.parametrize("name", CASES)
def test_fp32_select_on_reference_inputs(name, cuda_device):
    """The selection kernel fed the reference's own qc, kc, h_norm."""
    case, g, q, k, v = load_golden(name)
    B, H, T, D = q.shape
    NT, NG, NS = _lib.derive(T, case["density"])
    st = ops.Stages(B, H, T, D, NT, NG, NS, torch.float32, cuda_device)
    qc = _dev(_pad_rows(g["qc"], NG * 32), torch.float32, cuda_device)
    kc = _dev(_pad_rows(g["kc"], NG * 32), torch.float32, cuda_device)
    hn = _dev(g["h_norm"], torch.float32, cuda_device)
    noise = _dev(g["noise"], torch.float32, cuda_device) if "noise" in g else None
    ops.select(st, D, _lib.F32, D ** -0.5, case.get("use_cov_bias", True), noise, qc=qc, kc=kc, h_norm=hn)
    np.testing.assert_array_equal(st.indices.cpu().numpy(), g["indices"])
    # the bitmask agrees with the index lists
    mask = st.sel_mask.cpu().numpy().view(np.uint32)
    for bh in range(B * H):
        for i in range(NT):
            bits = {w * 32 + b for w in range(NG) for b in range(32) if (mask[bh, i, w] >> b) & 1}
            assert bits == set(g["indices"][bh, i].tolist())


@pytest.mark.parametrize("name", CASES)
def test_fp32_attention_on_reference_intermediates(name, cuda_device):
    case, g, q, k, v = load_golden(name)
    B, H, T, D = q.shape
    NT, NG, NS = _lib.derive(T, case["density"])
    st = ops.Stages(B, H, T, D, NT, NG, NS, torch.float32, cuda_device)
    st.kc.copy_(_dev(_pad_rows(g["kc"], NG * 32), torch.float32, cuda_device))
    st.vc.copy_(_dev(_pad_rows(g["vc"], NG * 32), torch.float32, cuda_device))
    st.h_group.copy_(_dev(g["h_group"], torch.float32, cuda_device))
    st.indices.copy_(torch.from_numpy(g["indices"]))
    mask = np.zeros((B * H, NT, NG), np.uint32)
    for bh in range(B * H):
        for i in range(NT):
            for j in g["indices"][bh, i]:
                mask[bh, i, j // 32] |= np.uint32(1 << (j % 32))
    st.sel_mask.copy_(torch.from_numpy(mask.view(np.int32)))
    qd, kd, vd = (t.to(cuda_device) for t in (q, k, v))
    o = torch.empty_like(vd)
    ops.attn(qd, kd, vd, st, D ** -0.5, o, _lib.ATTN_SIMT)
    np.testing.assert_allclose(_np(o), g["o"], rtol=0, atol=2e-5)


# ---------------------------------------------------------------------------
# bf16: the oracle's restatement of the reference's bf16 rounding points
# ---------------------------------------------------------------------------
def _bf16_inputs(B, H, T, D, seed, kind="normal", scale=1.0):
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(B, H, T, D, generator=g) * scale for _ in range(3))
    if kind == "max_shift":
        e = torch.randn(D, generator=g)
        e = e / e.norm() * D ** 0.5
        nt = -(-T // 64)
        for j in range(33, nt, 2):
            rows = slice(j * 64, min(T, (j + 1) * 64))
            k[:, :, rows] = (2.0 + 3.0 * torch.rand(1, generator=g).item()) * e + 0.01 * k[:, :, rows]
    return tuple(t.to(torch.bfloat16) for t in (q, k, v))


BF16_CASES = [
    # B, H, T, D, density, seed, kind
    (1, 2, 2500, 128, 0.15, 11, "normal"),   # partial last group, 4-token last block
    (1, 1, 1050, 128, 0.25, 12, "normal"),   # NT = 17: last pair has one query block
    (2, 1, 1000, 64, 0.3, 13, "normal"),     # head_dim 64, ragged last block
    (1, 1, 2200, 128, 0.25, 14, "max_shift"),  # running max grows in the correction phase
    (1, 1, 640, 128, 0.01, 15, "normal"),    # NS = 1
    (1, 1, 700, 128, 1.0, 16, "normal"),     # NS = NT (no corrected blocks)
    (1, 3, 4160, 128, 0.1, 17, "normal"),    # NG = 3
    (1, 2, 2049, 128, 0.2, 18, "normal"),    # a one-token last block alone in the last group
    (1, 1, 50, 128, 0.5, 19, "normal"),      # one partial block: NT = NS = 1, no pair partner
    (1, 2, 130, 128, 0.5, 20, "normal"),     # NT = 3: a full pair and a lone 2-token block
]


def _oracle_bf16(q, k, v, density, st=None):
    """Oracle in bf16 mode; when ``st`` is given, selection and attention
    use the GPU's own block statistics (so that the indices comparison is
    about the selection alone)."""
    B, H, T, D = q.shape
    qf, kf, vf = (t.float().reshape(B * H, T, D).numpy() for t in (q, k, v))
    qc, kc, vc, hc, hn = O.chunk_reduce(qf, kf, vf, 64, "bf16")
    hg = O.group_mean(hc, 32, "bf16")
    NS = O.Geometry(B, H, T, D).top_k(density)
    if st is not None:
        NT = qc.shape[1]
        qc, kc, vc = (_np(x)[:, :NT] for x in (st.qc, st.kc, st.vc))
        hn, hg = _np(st.h_norm), _np(st.h_group)
    idx, _ = O.select_blocks(qc, kc, hn, D ** -0.5, NS, "bf16")
    o = O.attention(qf, kf, vf, kc, vc, hg, idx, D ** -0.5, T, dtype="bf16")
    return dict(qc=qc, kc=kc, vc=vc, h_norm=hn, h_group=hg, hc=hc, indices=idx, o=o.reshape(B, H, T, D))


def _close(o, ref):
    o = np.asarray(o, np.float64)
    ref = np.asarray(ref, np.float64)
    err = float(np.max(np.abs(o - ref)))
    cos = O.cosine(o, ref)
    return err, cos


@pytest.mark.parametrize("B,H,T,D,density,seed,kind", BF16_CASES)
def test_bf16_block_stats_bit_exact(B, H, T, D, density, seed, kind, cuda_device):
    q, k, v = _bf16_inputs(B, H, T, D, seed, kind)
    ref = _oracle_bf16(q, k, v, density)
    _, st = ops.run_stages(*(t.to(cuda_device) for t in (q, k, v)), density=density)
    torch.cuda.synchronize()
    NT = st.NT
    np.testing.assert_array_equal(_np(st.qc)[:, :NT], ref["qc"])
    np.testing.assert_array_equal(_np(st.kc)[:, :NT], ref["kc"])
    np.testing.assert_array_equal(_np(st.vc)[:, :NT], ref["vc"])
    np.testing.assert_allclose(_np(st.h_norm), ref["h_norm"], rtol=1e-5)
    # h_group = bf16(mean_j bf16(hc_j)): a different fp32 summation order of
    # k^T v may move a bf16(hc_j) by one bf16 step (at most 2^-7 |hc_j|), and
    # the mean is rounded once more; bound the difference elementwise by that
    hg, rg = _np(st.h_group), ref["h_group"]
    hc = ref["hc"]
    BH, NTb = hc.shape[:2]
    pad = (32 - NTb % 32) % 32
    hcp = np.concatenate([np.abs(hc), np.zeros((BH, pad) + hc.shape[2:], np.float32)], axis=1)
    step = hcp.reshape(BH, -1, 32, D, D).sum(axis=2) / 32 * 2.0 ** -7
    assert np.all(np.abs(hg - rg) <= np.abs(rg) * 2.0 ** -7 + step + 1e-30)
    assert np.mean(hg == rg) > 0.99


@pytest.mark.parametrize("B,H,T,D,density,seed,kind", BF16_CASES)
def test_bf16_selection_bit_exact(B, H, T, D, density, seed, kind, cuda_device):
    q, k, v = _bf16_inputs(B, H, T, D, seed, kind)
    _, st = ops.run_stages(*(t.to(cuda_device) for t in (q, k, v)), density=density)
    torch.cuda.synchronize()
    ref = _oracle_bf16(q, k, v, density, st=st)
    np.testing.assert_array_equal(st.indices.cpu().numpy(), ref["indices"])


@pytest.mark.parametrize("kernel", [_lib.ATTN_TCGEN05, _lib.ATTN_SIMT])
@pytest.mark.parametrize("B,H,T,D,density,seed,kind", BF16_CASES)
def test_bf16_output_within_tolerance(B, H, T, D, density, seed, kind, kernel, cuda_device):
    q, k, v = _bf16_inputs(B, H, T, D, seed, kind)
    o, st = ops.run_stages(*(t.to(cuda_device) for t in (q, k, v)), density=density, kernel=kernel)
    torch.cuda.synchronize()
    ops.check_device_errors(st)
    ref = _oracle_bf16(q, k, v, density, st=st)
    err, cos = _close(_np(o), ref["o"])
    assert np.isfinite(_np(o)).all()
    assert err <= TOL_ABS and cos >= TOL_COS, (err, cos)


def test_tcgen05_matches_cuda_core_kernel(cuda_device):
    """Both attention kernels on identical intermediates (bf16, 14B-like
    head_dim and density, AR(1) keys)."""
    q, k, v = _bf16_inputs(1, 2, 8000, 128, 21)
    qd, kd, vd = (t.to(cuda_device) for t in (q, k, v))
    o_tc, st = ops.run_stages(qd, kd, vd, density=0.1, kernel=_lib.ATTN_TCGEN05)
    o_ref = torch.empty_like(o_tc)
    ops.attn(qd, kd, vd, st, 128 ** -0.5, o_ref, _lib.ATTN_SIMT)
    torch.cuda.synchronize()
    ops.check_device_errors(st)
    err, cos = _close(_np(o_tc), _np(o_ref))
    assert err <= TOL_ABS and cos >= 0.9999, (err, cos)


def test_forward_entry_point_matches_stages(cuda_device):
    q, k, v = (t.to(cuda_device) for t in _bf16_inputs(1, 2, 3000, 128, 31))
    o1 = ops.pisa_pg_attention(q, k, v, density=0.2)
    o2, _ = ops.run_stages(q, k, v, density=0.2)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)


def test_deterministic(cuda_device):
    q, k, v = (t.to(cuda_device) for t in _bf16_inputs(1, 2, 3000, 128, 41))
    a = ops.pisa_pg_attention(q, k, v, density=0.15)
    b = ops.pisa_pg_attention(q, k, v, density=0.15)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_use_random_consumes_the_cuda_generator_like_the_reference(cuda_device):
    q, k, v = (t.to(cuda_device) for t in _bf16_inputs(1, 2, 2048, 128, 51))
    B, H, T, D = q.shape
    NT = T // 64
    torch.manual_seed(7)
    o = ops.pisa_pg_attention(q, k, v, density=0.2, use_random=True)
    torch.manual_seed(7)
    noise = torch.randn_like(torch.zeros(B, H, NT, device=cuda_device))  # the reference's draw (:370)
    o2, _ = ops.run_stages(q, k, v, density=0.2, noise=noise)
    torch.cuda.synchronize()
    assert torch.equal(o, o2)


def test_full_op_against_oracle_end_to_end(cuda_device):
    """pisa_pg_attention alone (its own statistics and selection) against the
    oracle's own end-to-end result."""
    q, k, v = _bf16_inputs(1, 2, 3000, 128, 61)
    o = ops.pisa_pg_attention(*(t.to(cuda_device) for t in (q, k, v)), density=0.15)
    ref = _oracle_bf16(q, k, v, 0.15)
    err, cos = _close(_np(o), ref["o"])
    assert err <= TOL_ABS and cos >= TOL_COS, (err, cos)


def test_piecewise_alias(cuda_device):
    q, k, v = (t.to(cuda_device) for t in _bf16_inputs(1, 1, 1024, 128, 71))
    a = ops.piecewise_sparse_attention(q, k, v, density=0.25, block_size=64, use_random=False)
    b = ops.pisa_pg_attention(q, k, v, density=0.25)
    assert torch.equal(a, b)


def test_running_max_jumps_in_early_steps(cuda_device):
    """Keys repeated across the frames of a patch (a temporal head after the
    token placement) give each query block a few keys with logits ~60 (log2
    units) above the rest, met a few steps into the walk: the running maximum
    jumps at steps 2 and 3 of a tile, and the output accumulator is rescaled
    while the tensor core may still be adding earlier steps into it.  Forty
    calls (with the allocator churned in between) must all give the same
    output, within the tolerance of the oracle."""
    from oracle.layout_oracle import place_reference

    H, ctx, F_, S, D, density = 4, 64, 4, 512, 128, 0.2
    T = ctx + F_ * S
    g = torch.Generator().manual_seed(21)
    q, k, v = (torch.randn(1, H, T, D, generator=g).to(torch.bfloat16) for _ in range(3))
    for h in (1, 3):
        base = torch.randn(S, D, generator=g) * 2
        k[0, h, :F_ * S] = base.repeat(F_, 1).to(torch.bfloat16)
        q[0, h, :F_ * S] = (base.repeat(F_, 1) + 0.2 * torch.randn(F_ * S, D, generator=g)).to(torch.bfloat16)
    temporal = torch.tensor([[0, 1, 1, 1]])
    q, k, v = (place_reference(t.float(), temporal, ctx, F_, S).to(torch.bfloat16) for t in (q, k, v))
    ref = O.pisa_pg_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), density=density,
                              dtype="bf16")
    qd, kd, vd = (t.to(cuda_device) for t in (q, k, v))
    first = None
    for it in range(40):
        junk = torch.full((64 << 20,), it % 251, dtype=torch.uint8, device=cuda_device)
        del junk
        o = ops.pisa_pg_attention(qd, kd, vd, density=density)
        torch.cuda.synchronize()
        if first is None:
            first = o.clone()
            err, cos = _close(_np(o), ref)
            assert err <= TOL_ABS and cos >= TOL_COS, (err, cos)
        assert torch.equal(o, first), it
