"""DiT row kernels (pasa_dit_row_norm, pasa_dit_qkv_rope) on the GPU against
the CPU oracle: bit-exact, the oracle summing in the kernels' order."""
import numpy as np
import pytest
import torch

from oracle import dit_oracle as O

pytestmark = pytest.mark.gpu

EPS = 1e-6


def _bf16(shape, g, scale=1.0, offset=0.0):
    return (torch.randn(shape, generator=g) * scale + offset).to(torch.bfloat16)


def _np(t):
    return t.float().cpu().numpy()


def _vec(n, g, scale=0.2, offset=0.0):
    return torch.randn((n,), generator=g) * scale + offset


ROW_CASES = [
    # name, batch, rows, cols, add, gate, affine, modulate, norm
    ("ln_mod_5120", 1, 37, 5120, False, False, False, True, 1),
    ("gate_res_ln_mod_5120", 1, 41, 5120, True, True, False, True, 1),
    ("res_ln_affine_640", 1, 29, 640, True, False, True, False, 1),
    ("rms_w_64", 1, 17, 64, False, False, True, False, 0),
    ("ln_padded_5120", 1, 23, 5120, True, True, False, True, 2),
    ("ln_8192", 1, 9, 8192, True, True, True, True, 1),
    ("batch2_1024", 2, 19, 1024, True, True, False, True, 1),
]


@pytest.mark.parametrize("case", ROW_CASES, ids=[c[0] for c in ROW_CASES])
def test_row_norm_bit_exact(cuda_device, case):
    from pasa_b200 import ops
    name, B, L, C, use_add, use_gate, affine, modulate, norm = case
    g = torch.Generator().manual_seed(sum(map(ord, name)))
    x = _bf16((B, L, C), g, 2.0, 0.3)
    add = _bf16((B, L, C), g) if use_add else None
    gate = torch.stack([_vec(C, g, 1.0) for _ in range(B)])[:, None] if use_gate else None
    w = _vec(C, g, 0.1, 1.0) if affine else None
    b = _vec(C, g, 0.1) if affine else None
    scale = torch.stack([_vec(C, g) for _ in range(B)])[:, None] if modulate else None
    shift = torch.stack([_vec(C, g) for _ in range(B)])[:, None] if modulate else None
    dev = lambda t: None if t is None else t.to(cuda_device)
    xd = dev(x).contiguous()
    x_out = torch.empty_like(xd) if use_add else None
    y = ops.dit_row_norm(xd, add=dev(add), gate=dev(gate), x_out=x_out, weight=dev(w), bias=dev(b),
                         scale=dev(scale), shift=dev(shift), eps=EPS, norm=norm)
    for bi in range(B):
        xo, yo = O.row_norm(_np(x[bi]), EPS, add=None if add is None else _np(add[bi]),
                            gate=None if gate is None else gate[bi, 0].numpy(),
                            weight=None if w is None else w.numpy(), bias=None if b is None else b.numpy(),
                            scale=None if scale is None else scale[bi, 0].numpy(),
                            shift=None if shift is None else shift[bi, 0].numpy(),
                            center=norm != 0, pad_variance=norm == 2, order="kernel")
        assert np.array_equal(_np(y[bi]), yo), (name, np.abs(_np(y[bi]) - yo).max())
        if use_add:
            assert np.array_equal(_np(x_out[bi]), xo)


def test_row_norm_in_place_residual(cuda_device):
    """x_out aliasing x: the residual stream is updated in place."""
    from pasa_b200 import ops
    g = torch.Generator().manual_seed(5)
    x = _bf16((1, 33, 5120), g)
    add = _bf16((1, 33, 5120), g)
    gate = _vec(5120, g, 1.0)
    xd = x.to(cuda_device)
    ops.dit_row_norm(xd, add=add.to(cuda_device), gate=gate.to(cuda_device), x_out=xd, eps=EPS)
    xo, _ = O.row_norm(_np(x[0]), EPS, add=_np(add[0]), gate=gate.numpy())
    assert np.array_equal(_np(xd[0]), xo)


QKV_CASES = [
    # name, batch, tokens, heads, head_dim, rope, head_major, with_k, with_v
    ("wan_5120_rope", 2, 24, 40, 128, True, True, True, True),
    ("d64_rope", 1, 30, 8, 64, True, True, True, True),
    ("rms_only_rows", 1, 30, 8, 64, False, False, False, False),
    ("rope_rows_k", 1, 12, 4, 128, True, False, True, False),
]


@pytest.mark.parametrize("case", QKV_CASES, ids=[c[0] for c in QKV_CASES])
def test_qkv_rope_bit_exact(cuda_device, case):
    from pasa_b200 import ops
    name, B, L, H, D, use_rope, head_major, with_k, with_v = case
    C = H * D
    g = torch.Generator().manual_seed(len(name) * 7 + L)
    xq, xk, xv = (_bf16((B, L, C), g, 1.5) for _ in range(3))
    wq, wk = _vec(C, g, 0.1, 1.0), _vec(C, g, 0.1, 1.0)
    frames = 2
    cos = sin = None
    if use_rope:
        cos, sin = O.rope_table(frames, 1, L // frames, D)
    dev = lambda t: t.to(cuda_device)
    q, k, v = ops.dit_qkv_rope(dev(xq), dev(xk) if with_k else None, dev(xv) if with_v else None, dev(wq),
                               dev(wk), None if cos is None else torch.from_numpy(cos).to(cuda_device),
                               None if sin is None else torch.from_numpy(sin).to(cuda_device), H, EPS,
                               head_major=head_major)
    for bi in range(B):
        qo, ko, vo = O.qkv_rope(_np(xq[bi]), _np(xk[bi]) if with_k else None, _np(xv[bi]) if with_v else None,
                                wq.numpy(), wk.numpy(), cos, sin, H, EPS)
        back = (lambda a: a) if head_major else (lambda a: a.transpose(1, 0, 2).reshape(L, C))
        assert np.array_equal(_np(q[bi]), back(qo))
        if with_k:
            assert np.array_equal(_np(k[bi]), back(ko))
        if with_v:
            assert np.array_equal(_np(v[bi]), back(vo))
    if not with_k:
        assert k is None


def test_qkv_rope_matches_reference_torch_path(cuda_device):
    """Against the reference's own torch ops on the GPU (rmsnorm restated in
    fp32, rotary as attention.py:49-53 in complex128): equal up to the
    RMSNorm's reduction order (at most one bf16 step on a few elements)."""
    from pasa_b200 import ops
    g = torch.Generator().manual_seed(3)
    B, L, H, D = 1, 40, 40, 128
    C = H * D
    x = _bf16((B, L, C), g, 1.5).to(cuda_device)
    w = _vec(C, g, 0.1, 1.0).to(cuda_device)
    cos, sin = O.rope_table(2, 4, 5, D)
    cos_t, sin_t = torch.from_numpy(cos).to(cuda_device), torch.from_numpy(sin).to(cuda_device)
    q = ops.dit_qkv_rope(x, None, None, w, None, cos_t, sin_t, H, EPS)[0]
    xf = x.float()
    n = (xf * (1.0 / torch.sqrt(xf.pow(2).mean(-1, keepdim=True) + EPS)) * w).to(torch.bfloat16)
    n = n.unflatten(2, (H, D)).transpose(1, 2)
    rot = torch.view_as_complex(n.to(torch.float64).unflatten(3, (-1, 2)).contiguous())
    ref = torch.view_as_real(rot * torch.complex(cos_t, sin_t)).flatten(3, 4).type_as(n)
    diff = (q.float() - ref.float()).abs()
    assert (diff > 0).float().mean().item() < 0.01
    assert (diff <= ref.float().abs() * 2 ** -7 + 1e-6).all()
