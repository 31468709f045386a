"""Head classification on the GPU (pasa_sample_mse, through the C ABI)
against the torch restatement of the reference's sample_mse
(oracle/classify_oracle.py, whose closed-form masks the CPU tests pin to the
reference's dense mask loops), and the SVG layout chain around the PASA op.

The restatement runs the reference's own torch ops (matmul, softmax, mean
in the input dtype) on the same device and the same sampled rows.  The
kernel reproduces the reference's roundings but sums in its own fixed
order, so in bf16 a probability may round to the neighbouring bf16 value
now and then: the MSEs are compared within 2% relative, and the class
(argmin) must match wherever the restatement's two MSEs are more than 2%
apart.  fp32 inputs are compared within 1e-4 relative.
"""
import numpy as np
import pytest
import torch

from oracle import classify_oracle as CO
from oracle import pasa_oracle as O
from oracle.layout_oracle import place_reference
from pasa_b200 import classify, ops

pytestmark = pytest.mark.gpu

CASES = [
    # model, cfg, H, ctx, F, S, D, dtype
    ("hunyuan", 1, 4, 64, 4, 512, 128, torch.bfloat16),
    ("hunyuan", 2, 3, 0, 3, 384, 64, torch.bfloat16),
    ("wan", 1, 4, 0, 5, 640, 128, torch.bfloat16),
    ("hunyuan", 1, 3, 256, 6, 1024, 128, torch.float32),
    ("wan", 2, 2, 0, 4, 512, 64, torch.float32),
]


def _inputs(cfg, H, T, D, dtype, seed, device):
    g = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(cfg, H, T, D, generator=g).to(dtype).to(device) for _ in range(3))


def _compare(got, ref, dtype):
    got, ref = got.float().cpu(), ref.float().cpu()
    rtol = 2e-2 if dtype == torch.bfloat16 else 1e-4
    assert torch.isfinite(got).all()
    # an MSE below 1e-30 means the masked and full outputs agree to the last
    # bit in all but a few elements; such values are bf16 subnormals, whose
    # flushing differs between libraries
    torch.testing.assert_close(got, ref, rtol=rtol, atol=1e-30)
    # the class: argmin of the two masks, unless the reference's MSEs are within the tolerance
    clear = (ref[0] - ref[1]).abs() > rtol * torch.maximum(ref[0], ref[1]) + 1e-30
    return clear


@pytest.mark.parametrize("model,cfg,H,ctx,F_,S,D,dtype", CASES)
def test_sample_mse_matches_torch_restatement(model, cfg, H, ctx, F_, S, D, dtype, cuda_device):
    T = ctx + F_ * S
    q, k, v = _inputs(cfg, H, T, D, dtype, 5, cuda_device)
    rows = torch.randint(0, T, (32,), generator=torch.Generator().manual_seed(9))
    got = classify.sample_mse(q, k, v, model=model, context_length=ctx, num_frame=F_, frame_size=S, rows=rows)
    ref = CO.sample_mse_rows(q, k, v, rows, model=model, context_length=ctx, num_frame=F_, frame_size=S)
    clear = _compare(got, ref, dtype)
    best = classify.classify_heads(q, k, v, model=model, context_length=ctx, num_frame=F_, frame_size=S, rows=rows)
    ref_best = torch.argmin(ref.float().cpu(), dim=0)
    assert best.dtype == torch.int64 and best.shape == (cfg, H)
    assert torch.equal(best.cpu()[clear], ref_best[clear])


def test_sample_mse_draws_rows_like_the_reference(cuda_device):
    """Without ``rows`` the op draws torch.randint(0, sample_mse_max_row, (32,))
    on the CPU generator, exactly the reference's draw."""
    model, ctx, F_, S, D = "hunyuan", 32, 4, 256, 64
    T = ctx + F_ * S
    q, k, v = _inputs(1, 2, T, D, torch.float32, 6, cuda_device)
    torch.manual_seed(123)
    got = classify.sample_mse(q, k, v, model=model, context_length=ctx, num_frame=F_, frame_size=S,
                              sample_mse_max_row=T)
    torch.manual_seed(123)
    rows = torch.randint(low=0, high=T, size=(32,))
    ref = CO.sample_mse_rows(q, k, v, rows, model=model, context_length=ctx, num_frame=F_, frame_size=S)
    _compare(got, ref, torch.float32)


def test_sample_mse_at_hunyuan_720p_shape(cuda_device):
    """HunyuanVideo 720p x 129 frames: 24 heads, 33 x 3600 video tokens and
    256 text tokens (the reference samples rows below sample_mse_max_row)."""
    cfg, H, ctx, F_, S, D = 1, 24, 256, 33, 3600, 128
    T = ctx + F_ * S
    q, k, v = _inputs(cfg, H, T, D, torch.bfloat16, 7, cuda_device)
    rows = torch.randint(0, 10000, (32,), generator=torch.Generator().manual_seed(11))
    got = classify.sample_mse(q, k, v, model="hunyuan", context_length=ctx, num_frame=F_, frame_size=S, rows=rows)
    ref = CO.sample_mse_rows(q, k, v, rows, model="hunyuan", context_length=ctx, num_frame=F_, frame_size=S)
    _compare(got, ref, torch.bfloat16)


def test_temporal_head_is_detected(cuda_device):
    """Keys that repeat per patch across frames (pure temporal correlation)
    make a temporal head."""
    F_, S, D = 4, 512, 64
    T = F_ * S
    g = torch.Generator().manual_seed(0)
    base = torch.randn(S, D, generator=g) * 3
    k_t = base.repeat(F_, 1)
    q_t = k_t + 0.1 * torch.randn(T, D, generator=g)
    v_t = torch.randn(T, D, generator=g)
    q, k, v = (t[None, None].to(torch.bfloat16).to(cuda_device) for t in (q_t, k_t, v_t))
    torch.manual_seed(0)
    best = classify.classify_heads(q, k, v, model="wan", num_frame=F_, frame_size=S, sample_mse_max_row=T)
    assert int(best[0, 0]) == 1


def test_rejects_bad_shapes(cuda_device):
    q = torch.zeros(1, 1, 1000, 64, device=cuda_device)
    with pytest.raises(ValueError):  # T != ctx + F * S
        classify.sample_mse(q, q, q, model="hunyuan", context_length=8, num_frame=3, frame_size=300)
    with pytest.raises(ValueError):  # sampled row outside the sequence
        classify.sample_mse(q, q, q, model="wan", num_frame=2, frame_size=500, rows=torch.tensor([5, 1000]))


def test_svg_chain_classify_place_pasa_unplace(cuda_device):
    """The SVG profiling-and-layout chain around the attention op
    (svg/models/hyvideo/attention.py:478-530: sample_mse -> argmin ->
    hunyuan_sparse_head_placement -> sparse attention ->
    hunyuan_hidden_states_placement), with PASA as the sparse attention, on
    the GPU against the same chain on the CPU oracles."""
    cfg, H, ctx, F_, S, D, density = 1, 4, 64, 4, 512, 128, 0.2
    T = ctx + F_ * S
    g = torch.Generator().manual_seed(21)
    q, k, v = (torch.randn(cfg, H, T, D, generator=g).to(torch.bfloat16) for _ in range(3))
    # make heads 1 and 3 temporal: their keys repeat per patch across frames
    for h in (1, 3):
        base = torch.randn(S, D, generator=g) * 2
        k[0, h, :F_ * S] = base.repeat(F_, 1).to(torch.bfloat16)
        q[0, h, :F_ * S] = (base.repeat(F_, 1) + 0.2 * torch.randn(F_ * S, D, generator=g)).to(torch.bfloat16)
    rows = torch.randint(0, T, (32,), generator=torch.Generator().manual_seed(22))
    qd, kd, vd = (t.to(cuda_device) for t in (q, k, v))

    # GPU chain
    best = classify.classify_heads(qd, kd, vd, model="hunyuan", context_length=ctx, num_frame=F_, frame_size=S,
                                   rows=rows)
    qo, ko, vo = torch.empty_like(qd), torch.empty_like(kd), torch.empty_like(vd)
    ops.hunyuan_sparse_head_placement(qd, kd, vd, qo, ko, vo, best, ctx, F_, S)
    o_perm = ops.pisa_pg_attention(qo, ko, vo, density=density)
    out = torch.empty_like(o_perm)
    ops.hunyuan_hidden_states_placement(o_perm, out, best, ctx, F_, S)
    torch.cuda.synchronize()

    # the classes: the torch restatement (the reference's ops, same device
    # and rows) must agree wherever its two MSEs are clearly apart; the
    # temporal heads must come out temporal
    ref_mse = CO.sample_mse_rows(qd, kd, vd, rows, model="hunyuan", context_length=ctx, num_frame=F_, frame_size=S)
    clear = _compare(classify.sample_mse(qd, kd, vd, model="hunyuan", context_length=ctx, num_frame=F_,
                                         frame_size=S, rows=rows), ref_mse, torch.bfloat16)
    ref_best = torch.argmin(ref_mse.float().cpu(), dim=0)
    assert torch.equal(best.cpu()[clear], ref_best[clear])
    assert best[0, 1] == 1 and best[0, 3] == 1

    # the rest of the chain on the CPU oracles, with the same classes
    best_c = best.cpu()
    qp, kp, vp = (place_reference(t.float(), best_c, ctx, F_, S) for t in (q, k, v))
    o_ref = O.pisa_pg_attention(qp.numpy(), kp.numpy(), vp.numpy(), density=density, dtype="bf16")
    o_ref = place_reference(torch.from_numpy(o_ref), best_c, ctx, F_, S, inverse=True).numpy()
    got = out.float().cpu().numpy()
    err = float(np.max(np.abs(got - o_ref)))
    assert err <= 2e-2 and O.cosine(got, o_ref) >= 0.999, err
