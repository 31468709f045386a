"""Head classification (closed-form emulated masks) against the literal
restatement of the reference's mask construction (CPU)."""
import pytest
import torch
import torch.nn.functional as F

from oracle.layout_oracle import dense_attention_mask
from oracle import classify_oracle as classify


@pytest.mark.parametrize("model,ctx,F_,S", [("hunyuan", 16, 3, 256), ("hunyuan", 40, 5, 384), ("wan", 0, 4, 256),
                                            ("wan", 0, 3, 512), ("hunyuan", 0, 2, 640)])
@pytest.mark.parametrize("name", ["spatial", "temporal"])
def test_closed_form_masks_match_reference_loops(model, ctx, F_, S, name):
    dense = dense_attention_mask(name, ctx, F_, S, model)
    T = dense.shape[0]
    rows = torch.arange(T)
    got = classify.emulated_mask_rows(rows, name, model, ctx, F_, S)
    assert got.shape == dense.shape
    assert torch.equal(got, dense)


def _reference_sample_mse(q, k, v, masks_dense, rows):
    """sample_mse of hyvideo/attention.py:381-405 with given sampled rows."""
    dim = q.shape[-1]
    sq = q[:, :, rows, :]
    scores = torch.matmul(sq, k.transpose(-2, -1)) / (dim ** 0.5)
    golden = torch.matmul(F.softmax(scores, dim=-1), v)
    out = []
    for m in masks_dense:
        s = scores.masked_fill(m[rows, :] == 0, float("-inf"))
        out.append(torch.mean((torch.matmul(F.softmax(s, dim=-1), v) - golden) ** 2, dim=(2, 3)))
    return torch.stack(out)


@pytest.mark.parametrize("model,ctx,F_,S", [("hunyuan", 32, 4, 256), ("wan", 0, 4, 256)])
def test_sample_mse_and_rng_match_reference(model, ctx, F_, S):
    g = torch.Generator().manual_seed(3)
    T = ctx + F_ * S if model == "hunyuan" else F_ * S
    q, k, v = (torch.randn(2, 3, T, 64, generator=g) for _ in range(3))
    dense = [dense_attention_mask(n, ctx, F_, S, model) for n in ("spatial", "temporal")]
    torch.manual_seed(11)
    got = classify.sample_mse(q, k, v, model=model, context_length=ctx, num_frame=F_, frame_size=S,
                              num_sampled_rows=32, sample_mse_max_row=T)
    torch.manual_seed(11)
    rows = torch.randint(low=0, high=T, size=(32,))  # the reference's draw
    ref = _reference_sample_mse(q, k, v, dense, rows)
    torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-7)
    idx = classify.classify_heads(q, k, v, model=model, context_length=ctx, num_frame=F_, frame_size=S,
                                  sample_mse_max_row=T)
    assert idx.shape == (2, 3) and set(idx.unique().tolist()) <= {0, 1}


def test_temporal_head_is_detected():
    """A head whose keys repeat per patch across frames (pure temporal
    correlation) is classified temporal; an i.i.d. head spatial-or-temporal
    by MSE, whichever is smaller."""
    ctx, F_, S, D = 0, 4, 512, 64
    T = F_ * S
    g = torch.Generator().manual_seed(0)
    base = torch.randn(S, D, generator=g) * 3
    k_t = base.repeat(F_, 1)                    # token f*S + p has key base[p]
    q_t = k_t + 0.1 * torch.randn(T, D, generator=g)
    v_t = torch.randn(T, D, generator=g)
    q = q_t[None, None]; k = k_t[None, None]; v = v_t[None, None]
    torch.manual_seed(0)
    idx = classify.classify_heads(q, k, v, model="wan", context_length=ctx, num_frame=F_, frame_size=S,
                                  sample_mse_max_row=T)
    assert int(idx[0, 0]) == 1
