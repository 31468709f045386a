"""Host-side mirror of the reference's PASA operator interface.

``pisa_pg_attention`` keeps the signature, argument meaning and error
behaviour of ZHANGWENTAI/PASA ``svg/kernels/triton/group_pisa_attention.py:
307-398`` and runs on the B200 through the C ABI of ``libpasa_b200.so``
(``include/pasa_b200.h``).  PyTorch only provides device memory, the current
stream and the random draw of ``use_random``; there is no CPU or Triton path.
"""
from __future__ import annotations

import ctypes

from typing import Optional

import torch

from . import _lib

_DTYPES = {torch.bfloat16: _lib.BF16, torch.float32: _lib.F32}


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise ValueError(f"pasa_b200 supports bfloat16 and float32 inputs, got {t.dtype}") from None


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _check_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if t.dim() != 4:
            raise ValueError(f"{name} must be [B, H, T, D], got shape {tuple(t.shape)}")
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor (pasa_b200 has no CPU path)")
    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError(f"q, k, v must share one shape, got {tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("q, k, v must share one dtype")
    if q.device != k.device or q.device != v.device:
        raise ValueError("q, k, v must be on one device")
    _dtype_code(q)


class Stages:
    """Intermediates of one call, allocated by torch (used for verbose output
    and parity tests)."""

    def __init__(self, B, H, T, D, NT, NG, NS, dtype, device):
        NTP = NG * 32
        self.qc = torch.empty(B * H, NTP, D, dtype=dtype, device=device)
        self.kc = torch.empty_like(self.qc)
        self.vc = torch.empty_like(self.qc)
        self.h_norm = torch.empty(B * H, NT, dtype=torch.float32, device=device)
        self.h_group = torch.empty(B * H, NG, D, D, dtype=dtype, device=device)
        self.indices = torch.empty(B * H, NT, NS, dtype=torch.int32, device=device)
        self.sel_mask = torch.empty(B * H, NT, NG, dtype=torch.int32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.NT, self.NG, self.NS = NT, NG, NS


def prep(q, k, v, st: Stages):
    B, H, T, D = q.shape
    lib = _lib.load()
    _lib.check("pasa_prep", lib.pasa_prep(_stream_ptr(q.device), q.data_ptr(), k.data_ptr(), v.data_ptr(), B, H, T,
                                          D, _dtype_code(q), 64, 32, st.qc.data_ptr(), st.kc.data_ptr(),
                                          st.vc.data_ptr(), st.h_norm.data_ptr(), st.h_group.data_ptr()))


def select(st: Stages, D: int, dtype_code: int, scale: float, use_cov_bias: bool, noise=None,
           device=None, qc=None, kc=None, h_norm=None):
    lib = _lib.load()
    qc = st.qc if qc is None else qc
    kc = st.kc if kc is None else kc
    h_norm = st.h_norm if h_norm is None else h_norm
    _lib.check("pasa_select", lib.pasa_select(_stream_ptr(device or qc.device), qc.data_ptr(), kc.data_ptr(),
                                              h_norm.data_ptr(), _ptr(noise), st.indices.shape[0], st.NT, D,
                                              dtype_code, float(scale), int(bool(use_cov_bias)), st.NS,
                                              st.indices.data_ptr(), st.sel_mask.data_ptr()))


def attn(q, k, v, st: Stages, scale: float, o: torch.Tensor, kernel: int = _lib.ATTN_AUTO,
         kc=None, vc=None, h_group=None, indices=None, sel_mask=None):
    B, H, T, D = q.shape
    lib = _lib.load()
    kc = st.kc if kc is None else kc
    vc = st.vc if vc is None else vc
    h_group = st.h_group if h_group is None else h_group
    indices = st.indices if indices is None else indices
    sel_mask = st.sel_mask if sel_mask is None else sel_mask
    _lib.check("pasa_attn", lib.pasa_attn(_stream_ptr(q.device), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                          kc.data_ptr(), vc.data_ptr(), h_group.data_ptr(), indices.data_ptr(),
                                          sel_mask.data_ptr(), B * H, T, D, _dtype_code(q), float(scale), st.NS,
                                          o.data_ptr(), st.err.data_ptr(), int(kernel)))


def check_device_errors(st: Stages) -> None:
    """Raise if a kernel reported a bounded-wait timeout (synchronises)."""
    flags = int(st.err.item())
    if flags & _lib.DEVERR_WAIT_TIMEOUT:
        raise RuntimeError("pasa_b200: a device-side barrier wait timed out (error word %#x)" % flags)


def run_stages(q, k, v, density=0.15, scale=None, use_cov_bias=True, noise=None, kernel=_lib.ATTN_AUTO):
    """The op as three separate C-ABI calls; returns (o, Stages)."""
    _check_qkv(q, k, v)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    B, H, T, D = q.shape
    scale = D ** -0.5 if scale is None else scale
    NT, NG, NS = _lib.derive(T, density)
    with torch.cuda.device(q.device):
        st = Stages(B, H, T, D, NT, NG, NS, q.dtype, q.device)
        prep(q, k, v, st)
        select(st, D, _dtype_code(q), scale, use_cov_bias, noise)
        o = torch.empty_like(v)
        attn(q, k, v, st, scale, o, kernel)
    return o, st


def pisa_pg_attention(
    q, k, v,
    density=0.15,
    timestep=0,
    block_size=64,
    group_size=32,
    scale=None,
    use_cov_bias=True,
    use_random=False,
    verbose=False,
    prompt_token_length: Optional[int] = None,
    *,
    kernel: int = _lib.ATTN_AUTO,
    out_layout: str = "bhtd",
):
    """PASA forward: exact attention on the covariance-aware top-k blocks,
    zero-order + per-group first-order correction on the rest.

    Same arguments as the reference (group_pisa_attention.py:307-318):
    q, k, v [B, H, T, D] CUDA tensors (bf16 or fp32); ``density`` is the
    fraction of 64-token blocks attended exactly; ``scale`` defaults to
    D**-0.5; ``use_cov_bias`` adds log(h_norm + 1e-6) to the block score;
    ``use_random`` adds ``torch.randn_like`` noise to that bias (drawn here,
    on the current CUDA generator, exactly as the reference draws it).
    ``timestep`` and ``prompt_token_length`` are accepted and unused, as in
    the reference.  Returns a new [B, H, T, D] tensor like ``v``; with
    ``out_layout="bthd"`` (bf16, tensor-core kernel) its storage is
    token-major [B, T, H, D] and the result is the transposed view, so a
    following ``o.transpose(1, 2).flatten(2, 3)`` costs no copy.
    """
    del timestep, prompt_token_length  # unused by the reference as well
    if out_layout not in ("bhtd", "bthd"):
        raise ValueError("out_layout is 'bhtd' or 'bthd'")
    if block_size != 64 or group_size != 32:
        raise ValueError("pasa_b200 supports block_size=64 and group_size=32 (the reference's defaults)")
    _check_qkv(q, k, v)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    B, H, T, K = q.shape
    scale = K ** -0.5 if scale is None else scale
    NT, NG, NS = _lib.derive(T, density, block_size, group_size)
    noise = None
    if use_cov_bias and use_random:
        # torch.randn_like(log_bias), log_bias: [B, H, NT] fp32 (:368-370)
        noise = torch.randn((B, H, NT), dtype=torch.float32, device=q.device)

    if verbose and out_layout == "bhtd":
        o, st = run_stages(q, k, v, density, scale, use_cov_bias, noise, kernel)
        hn = st.h_norm
        print(f"NT={NT}, N_GROUPS={NG}, GROUP_SIZE={group_size}")
        print(f"h_norm: mean={hn.mean():.2f}, max={hn.max():.2f}")
        print(f"h_group: {tuple(st.h_group.shape)}")
        print(f"top_k={NS}, density={density}")
        return o

    dcode = _dtype_code(q)
    lib = _lib.load()
    with torch.cuda.device(q.device):
        ws_bytes = _lib.workspace_size(B, H, T, K, dcode, NS, block_size, group_size)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
        if out_layout == "bthd":
            o_store = torch.empty((B, T, H, K), dtype=v.dtype, device=v.device)
            o = o_store.transpose(1, 2)
        else:
            o_store = o = torch.empty_like(v)
        _lib.check("pasa_forward_ex", lib.pasa_forward_ex(
            _stream_ptr(q.device), q.data_ptr(), k.data_ptr(), v.data_ptr(), B, H, T, K, dcode, float(density),
            float(scale), int(bool(use_cov_bias)), _ptr(noise), ws.data_ptr(), ws_bytes, o_store.data_ptr(),
            int(kernel), _lib.O_BTHD if out_layout == "bthd" else _lib.O_BHTD))
    return o


def pisa_pg_attention_range(q, k, v, block_begin: int, block_end: int, density=0.15, scale=None,
                            use_cov_bias=True, noise=None, out=None):
    """The op on the query blocks [block_begin, block_end) of q's B*H*NT
    blocks (numbered head by head; pasa_forward_range): only their rows of
    ``out`` ([B, H, T, D] like v, allocated when None) are written.  For
    splitting one call over several GPUs finer than by heads.  bf16 only
    (tensor-core kernel).  No counterpart in the reference."""
    _check_qkv(q, k, v)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    B, H, T, K = q.shape
    scale = K ** -0.5 if scale is None else scale
    dcode = _dtype_code(q)
    lib = _lib.load()
    if out is None:
        out = torch.empty_like(v)
    elif out.shape != v.shape or out.dtype != v.dtype or not out.is_contiguous() or out.device != v.device:
        raise ValueError("out must be a contiguous tensor like v")
    with torch.cuda.device(q.device):
        n = ctypes.c_size_t()
        _lib.check("pasa_forward_range_workspace_size", lib.pasa_forward_range_workspace_size(
            B, H, T, K, dcode, float(density), int(block_begin), int(block_end), ctypes.byref(n)))
        ws = torch.empty(n.value, dtype=torch.uint8, device=q.device)
        _lib.check("pasa_forward_range", lib.pasa_forward_range(
            _stream_ptr(q.device), q.data_ptr(), k.data_ptr(), v.data_ptr(), B, H, T, K, dcode, float(density),
            float(scale), int(bool(use_cov_bias)), _ptr(noise), ws.data_ptr(), n.value, out.data_ptr(),
            _lib.ATTN_AUTO, int(block_begin), int(block_end)))
    return out


def pisa_pg_attention_host(
    q, k, v,
    density=0.15,
    scale=None,
    use_cov_bias=True,
    use_random=False,
    *,
    heads_per_chunk: int = 4,
    out: Optional[torch.Tensor] = None,
    device=None,
    kernel: int = _lib.ATTN_AUTO,
):
    """The same op on host-resident tensors: q, k, v are [B, H, T, D] CPU
    tensors (page-locked for the copies to overlap the compute) and the
    result is a CPU tensor like ``v`` (``out`` if given).  The heads go
    through the GPU in chunks of ``heads_per_chunk``: chunk i is computed
    while chunk i+1 is copied in and chunk i-1 copied out
    (``pasa_forward_host``).  No counterpart in the reference, whose op takes
    CUDA tensors; the result equals ``pisa_pg_attention`` on the same heads.
    Synchronous: returns when the result is in host memory.
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not isinstance(t, torch.Tensor) or t.device.type != "cpu":
            raise ValueError(f"{name} must be a CPU tensor")
        if t.dim() != 4:
            raise ValueError(f"{name} must be [B, H, T, D]")
    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError("q, k and v must have the same shape")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("q, k and v must have the same dtype")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    B, H, T, K = q.shape
    dcode = _dtype_code(q)
    scale = K ** -0.5 if scale is None else scale
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    NT, NG, NS = _lib.derive(T, density)
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    elif out.shape != q.shape or out.dtype != q.dtype or out.device.type != "cpu" or not out.is_contiguous():
        raise ValueError("out must be a contiguous CPU tensor like q")
    lib = _lib.load()
    with torch.cuda.device(dev):
        noise = None
        if use_cov_bias and use_random:
            noise = torch.randn((B, H, NT), dtype=torch.float32, device=dev).cpu()
        n = ctypes.c_size_t()
        _lib.check("pasa_forward_host_workspace_size", lib.pasa_forward_host_workspace_size(
            B, H, T, K, dcode, float(density), int(heads_per_chunk), ctypes.byref(n)))
        ws = torch.empty(n.value, dtype=torch.uint8, device=dev)
        err = ctypes.c_uint32(0)
        _lib.check("pasa_forward_host", lib.pasa_forward_host(
            _stream_ptr(dev), q.data_ptr(), k.data_ptr(), v.data_ptr(), B, H, T, K, dcode, float(density),
            float(scale), int(bool(use_cov_bias)), _ptr(noise), ws.data_ptr(), n.value, int(heads_per_chunk),
            out.data_ptr(), ctypes.byref(err), int(kernel)))
    if err.value & _lib.DEVERR_WAIT_TIMEOUT:
        raise RuntimeError("pasa_forward_host: a kernel gave up waiting on a barrier (device error word)")
    return out


def dense_attention(q, k, v, scale=None):
    """Dense attention softmax(q k^T scale) v for [B, H, T, D] bf16 CUDA tensors
    on the tensor-core kernel (pasa_dense_attn): the branch the models take for
    their dense layers and timesteps (SDPA in the reference,
    svg/models/wan/attention.py:299-301).  Returns a new tensor like ``v``.
    """
    _check_qkv(q, k, v)
    if q.dtype != torch.bfloat16:
        raise ValueError("dense_attention runs the bf16 tensor-core kernel; q, k, v must be bf16")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    B, H, T, K = q.shape
    scale = K ** -0.5 if scale is None else scale
    lib = _lib.load()
    with torch.cuda.device(q.device):
        o = torch.empty_like(v)
        err = torch.zeros(1, dtype=torch.int32, device=q.device)
        _lib.check("pasa_dense_attn", lib.pasa_dense_attn(
            _stream_ptr(q.device), q.data_ptr(), k.data_ptr(), v.data_ptr(), B * H, T, K, _dtype_code(q),
            float(scale), o.data_ptr(), err.data_ptr()))
    return o


# ---------------------------------------------------------------------------
# DiT row kernels around the attention op (pasa_dit_row_norm, pasa_dit_qkv_rope)
# ---------------------------------------------------------------------------
def _vec(t: Optional[torch.Tensor], cols: int, name: str) -> Optional[torch.Tensor]:
    if t is None:
        return None
    if t.dtype != torch.float32 or not t.is_cuda or t.shape[-1] != cols:
        raise ValueError(f"{name} must be an fp32 CUDA tensor with last dimension {cols}")
    return t.contiguous()


DIT_RMSNORM, DIT_LAYERNORM, DIT_LAYERNORM_PADDED = 0, 1, 2

def dit_row_norm(x, *, add=None, gate=None, x_out=None, weight=None, bias=None, scale=None, shift=None,
                 eps: float = 1e-6, norm: int = DIT_LAYERNORM, out=None):
    """Gated residual + LayerNorm / RMSNorm + affine + modulation over the last
    dimension of bf16 ``x`` [B, L, C] in one pass (pasa_dit_row_norm):

        x' = x + add * gate  (or x + add; x when add is None), written to x_out
        y  = ((x' - mean) * rstd) [* weight] [+ bias] [* (1 + scale) + shift]

    ``norm``: DIT_LAYERNORM (the torch LayerNorm), DIT_RMSNORM (mean 0), or
    DIT_LAYERNORM_PADDED (the reference's Triton LayerNorm, whose zero padding
    to a power of two adds (P - C) * mean^2 to the variance).

    ``gate``, ``scale``, ``shift`` are fp32 [B, 1, C] or [C] (one vector per
    batch entry), ``weight`` and ``bias`` fp32 [C].  Returns y (bf16, like x).
    """
    if x.dtype != torch.bfloat16 or not x.is_cuda or not x.is_contiguous():
        raise ValueError("x must be a contiguous bf16 CUDA tensor")
    C = x.shape[-1]
    rows = x.numel() // C
    batch = x.shape[0] if x.dim() == 3 else 1
    for t, n in ((add, "add"), (x_out, "x_out")):
        if t is not None and (t.shape != x.shape or t.dtype != x.dtype or not t.is_contiguous()):
            raise ValueError(f"{n} must be a contiguous bf16 tensor shaped like x")
    per_batch = []
    for t, n in ((gate, "gate"), (scale, "scale"), (shift, "shift")):
        t = _vec(t, C, n)
        if t is not None and t.numel() not in (C, batch * C):
            raise ValueError(f"{n} must hold one [C] vector per batch entry")
        if t is not None and t.numel() == C and batch > 1:
            t = t.reshape(1, C).expand(batch, C).contiguous()
        per_batch.append(t)
    gate, scale, shift = per_batch
    weight, bias = _vec(weight, C, "weight"), _vec(bias, C, "bias")
    y = torch.empty_like(x) if out is None else out
    lib = _lib.load()
    with torch.cuda.device(x.device):
        _lib.check("pasa_dit_row_norm", lib.pasa_dit_row_norm(
            _stream_ptr(x.device), x.data_ptr(), _ptr(add), _ptr(gate), _ptr(x_out), _ptr(weight), _ptr(bias),
            _ptr(scale), _ptr(shift), rows, rows // batch, C, float(eps), int(norm), y.data_ptr()))
    return y


def dit_qkv_rope(xq, xk, xv, wq, wk, cos, sin, heads: int, eps: float = 1e-6, head_major: bool = True):
    """Self-attention producer (pasa_dit_qkv_rope): RMSNorm of the bf16 q and k
    projections [B, L, H*D] with fp32 weights [H*D], fp64 rotary embedding
    (``cos``, ``sin`` [L, D/2] float64, or None) and the transpose to
    [B, H, L, D] (``head_major``); v is transposed.  ``xk`` / ``xv`` may be
    None.  Returns (q, k, v) with None for the skipped ones."""
    for t, n in ((xq, "xq"), (xk, "xk"), (xv, "xv")):
        if t is not None and (t.dtype != torch.bfloat16 or not t.is_cuda or not t.is_contiguous() or t.dim() != 3
                              or t.shape != xq.shape):
            raise ValueError(f"{n} must be a contiguous bf16 CUDA tensor [B, L, C] like xq")
    B, L, C = xq.shape
    if C % heads:
        raise ValueError("hidden size is not a multiple of heads")
    D = C // heads
    wq, wk = _vec(wq, C, "wq"), _vec(wk, C, "wk")
    if (cos is None) != (sin is None):
        raise ValueError("cos and sin are given together")
    if cos is not None:
        if cos.dtype != torch.float64 or sin.dtype != torch.float64 or cos.shape != (L, D // 2) \
                or sin.shape != (L, D // 2):
            raise ValueError(f"cos, sin must be float64 [{L}, {D // 2}]")
        cos, sin = cos.contiguous(), sin.contiguous()
    shape = (B, heads, L, D) if head_major else (B, L, C)
    outs = [torch.empty(shape, dtype=torch.bfloat16, device=xq.device) if t is not None else None
            for t in (xq, xk, xv)]
    lib = _lib.load()
    with torch.cuda.device(xq.device):
        _lib.check("pasa_dit_qkv_rope", lib.pasa_dit_qkv_rope(
            _stream_ptr(xq.device), xq.data_ptr(), _ptr(xk), _ptr(xv), wq.data_ptr(), _ptr(wk), _ptr(cos),
            _ptr(sin), B, L, heads, D, float(eps), int(bool(head_major)), *(_ptr(t) for t in outs)))
    return tuple(outs)


def piecewise_sparse_attention(q, k, v, density=0.15, block_size=64, use_random=False, **kwargs):
    """The name the model processors call (svg/models/wan/attention.py:384,
    svg/models/hyvideo/attention.py:640, :682); its source is not in the
    reference tree, and the processors pass the arguments of
    ``pisa_pg_attention``, so it is the same op."""
    return pisa_pg_attention(q, k, v, density=density, block_size=block_size, use_random=use_random, **kwargs)


# ---------------------------------------------------------------------------
# token-layout permutation (svg/models/hyvideo/placement.py)
# ---------------------------------------------------------------------------
def _place(src, dst, best_mask_idx, context_length, num_frame, frame_size, inverse):
    if src.dim() != 4 or dst.shape != src.shape:
        raise ValueError("placement expects [cfg, H, T, D] tensors of one shape")
    if not (src.is_cuda and dst.is_cuda):
        raise ValueError("placement tensors must be CUDA tensors")
    if not (src.is_contiguous() and dst.is_contiguous()):
        raise ValueError("placement tensors must be contiguous")
    cfg, H, T, D = src.shape
    if T != context_length + num_frame * frame_size:  # placement.py:128, :366
        raise AssertionError("seq_len must equal context_length + num_frame * frame_size")
    idx = best_mask_idx.to(device=src.device, dtype=torch.int32).contiguous()
    if idx.shape != (cfg, H):
        raise ValueError(f"best_mask_idx must be [cfg, H] = {(cfg, H)}, got {tuple(idx.shape)}")
    lib = _lib.load()
    with torch.cuda.device(src.device):
        _lib.check("pasa_place", lib.pasa_place(_stream_ptr(src.device), src.data_ptr(), dst.data_ptr(),
                                                idx.data_ptr(), cfg, H, T, D, _dtype_code(src),
                                                int(context_length), int(num_frame), int(frame_size),
                                                int(inverse)))


def hunyuan_sparse_head_placement(query, key, value, query_out, key_out, value_out, best_mask_idx,
                                  context_length, num_frame, frame_size):
    """Frame-major -> token-major for temporal heads (best_mask_idx == 1),
    copy for spatial heads; writes the caller's outputs
    (placement.py:124-153)."""
    for src, dst in ((query, query_out), (key, key_out), (value, value_out)):
        _place(src, dst, best_mask_idx, context_length, num_frame, frame_size, inverse=0)


def hunyuan_hidden_states_placement(hidden_states, hidden_states_out, best_mask_idx, context_length, num_frame,
                                    frame_size):
    """Token-major -> frame-major for temporal heads (placement.py:360-387)."""
    _place(hidden_states, hidden_states_out, best_mask_idx, context_length, num_frame, frame_size, inverse=1)
    return hidden_states_out
