"""Wan2.1-style DiT denoising step with PASA self-attention and Ulysses
sequence parallelism (the full-step benchmark configuration).

One block follows the op sequence of the reference's
``WanTransformerBlock_Sparse.forward`` (svg/models/wan/custom_models.py:24-113)
and its attention processor (svg/models/wan/attention.py:166-225):

1. AdaLN: ``shift, scale, gate, c_shift, c_scale, c_gate =
   (scale_shift_table + temb).chunk(6)``; fp32 LayerNorm (no affine),
   ``x * (1 + scale) + shift``.
2. Self-attention: q, k, v projections, RMSNorm of q and k over the hidden
   dimension, split into heads, 3D rotary embedding, the attention core
   (PASA), output projection; ``x = x + attn * gate`` in fp32.
3. Cross-attention over the text tokens: LayerNorm with affine, q from x,
   k and v from the text, RMSNorm of q and k, SDPA, output projection,
   ``x = x + attn``.
4. Feed-forward: LayerNorm, ``(1 + c_scale)`` / ``c_shift`` modulation,
   Linear -> GELU(tanh) -> Linear, ``x = x + ffn * c_gate``.

The model-level parts of a step (patch embedding, timestep and text
embedders, output norm and projection) follow
``WanTransformer3DModel_Sparse.forward`` (custom_models.py:115-200).
Weights are random (seeded); there are no checkpoints.

Two implementations of the same step:

* ``fused=True`` (the B200 path): the elementwise work between the GEMMs runs
  in the library's row kernels -- ``pasa_dit_row_norm`` folds each residual
  update into the LayerNorm + modulation that reads it (the FFN residual of
  block i into block i+1's first norm), ``pasa_dit_qkv_rope`` does q/k
  RMSNorm, the rotary embedding and the head-major transpose in one pass.
  GEMMs are cuBLAS (torch), cross-attention is torch SDPA, self-attention is
  the attention core passed in (PASA).
* ``fused=False``: the same step in plain torch ops, with the casts of the
  reference's torch path (LayerNorm, modulation and residuals in fp32,
  rotary embedding in float64).  It runs on any device and is the comparison
  for the fused path.

With a process group of P ranks each rank holds T/P consecutive tokens
(Ulysses): q, k, v go sequence-sharded -> head-sharded with one all-to-all
each, the attention core runs on H/P heads over all T tokens, and one
all-to-all brings the output back; everything else is token-local.
"""
from __future__ import annotations

import dataclasses
import math
from typing import Callable, List, Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import ops


@dataclasses.dataclass(frozen=True)
class DiTConfig:
    hidden: int = 5120
    heads: int = 40
    ffn: int = 13824
    layers: int = 40
    text_len: int = 512
    frames: int = 21          # latent frames x height x width patches: 21 x 45 x 80 = 75600 tokens
    height: int = 45
    width: int = 80
    eps: float = 1e-6
    density: float = 0.10
    in_channels: int = 16     # latent channels; a 1 x 2 x 2 patch is 64 features
    text_dim: int = 4096
    freq_dim: int = 256

    @property
    def tokens(self) -> int:
        return self.frames * self.height * self.width

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


WAN14B_720P = DiTConfig()

# per-channel vectors the row kernels read as fp32
_F32_VECTORS = ("norm_q", "norm_k", "cnorm_q", "cnorm_k")


def init_block(cfg: DiTConfig, seed: int, device, dtype=torch.bfloat16) -> dict:
    """Random weights of one block (std 0.02 projections, small random norms).
    Norm weights are kept in ``dtype`` like the model's parameters, with fp32
    copies (``<name>_f``) for the row kernels."""
    g = torch.Generator(device=device).manual_seed(seed)
    C, Fd = cfg.hidden, cfg.ffn

    def lin(out_f, in_f):
        return (torch.randn((out_f, in_f), generator=g, device=device, dtype=torch.float32) * 0.02).to(dtype)

    def vec(n, mean=0.0, std=0.02):
        return (mean + std * torch.randn((n,), generator=g, device=device, dtype=torch.float32)).to(dtype)

    w = {
        "scale_shift_table": torch.randn((1, 6, C), generator=g, device=device, dtype=torch.float32) / C ** 0.5,
        "q": lin(C, C), "q_b": vec(C), "k": lin(C, C), "k_b": vec(C), "v": lin(C, C), "v_b": vec(C),
        "o": lin(C, C), "o_b": vec(C), "norm_q": vec(C, 1.0), "norm_k": vec(C, 1.0),
        "norm2_w": vec(C, 1.0).float(), "norm2_b": vec(C).float(),
        "cq": lin(C, C), "cq_b": vec(C), "ck": lin(C, C), "ck_b": vec(C), "cv": lin(C, C), "cv_b": vec(C),
        "co": lin(C, C), "co_b": vec(C), "cnorm_q": vec(C, 1.0), "cnorm_k": vec(C, 1.0),
        "ffn1": lin(Fd, C), "ffn1_b": vec(Fd), "ffn2": lin(C, Fd), "ffn2_b": vec(C),
    }
    for n in _F32_VECTORS:
        w[n + "_f"] = w[n].float()
    return w


def rope_table(cfg: DiTConfig, device, theta: float = 10000.0):
    """float64 cos, sin [T, D/2] of the 3D rotary embedding: the head
    dimension's pairs split over (frame, row, column) as D - 4*(D//6),
    2*(D//6), 2*(D//6), axis frequencies theta^(-2i/d) in float64 (the table
    diffusers' WanRotaryPosEmbed builds; the reference's complex ``freqs`` is
    cos + i sin)."""
    D = cfg.head_dim
    dims = [D - 4 * (D // 6), 2 * (D // 6), 2 * (D // 6)]
    angles = []
    grids = torch.meshgrid(torch.arange(cfg.frames, device=device), torch.arange(cfg.height, device=device),
                           torch.arange(cfg.width, device=device), indexing="ij")
    for pos, d in zip(grids, dims):
        inv = 1.0 / theta ** (torch.arange(0, d, 2, device=device, dtype=torch.float64) / d)
        angles.append(pos.reshape(-1, 1).double() * inv[None, :])
    ang = torch.cat(angles, dim=1)                       # [T, D/2]
    return torch.cos(ang), torch.sin(ang)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [B, H, L, D]; rotates the pairs (2i, 2i+1) by the angles of its L
    tokens in float64 and casts back (attention.py:49-53)."""
    xf = x.double().unflatten(-1, (-1, 2))
    a, b = xf[..., 0], xf[..., 1]
    c, s = cos.double(), sin.double()
    out = torch.stack((a * c - b * s, a * s + b * c), dim=-1).flatten(-2)
    return out.to(x.dtype)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """x * rstd * w in fp32, rounded once (rmsnorm.py:30-45)."""
    xf = x.float()
    return (xf / torch.sqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


def seq_to_head(t: torch.Tensor, group) -> torch.Tensor:
    """[B, H, L/P, D] on every rank (its tokens, all heads) -> [B, H/P, L, D]
    (all tokens, its heads), one all-to-all."""
    P = dist.get_world_size(group)
    B, H, Ll, D = t.shape
    send = t.reshape(B, P, H // P, Ll, D).permute(1, 0, 2, 3, 4).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)         # recv[src] = src's tokens of my heads
    return recv.permute(1, 2, 0, 3, 4).reshape(B, H // P, P * Ll, D)


def head_to_seq(t: torch.Tensor, group) -> torch.Tensor:
    """Inverse of seq_to_head: [B, H/P, L, D] -> [B, H, L/P, D]."""
    P = dist.get_world_size(group)
    B, Hl, L, D = t.shape
    send = t.reshape(B, Hl, P, L // P, D).permute(2, 0, 1, 3, 4).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)         # recv[src] = my tokens of src's heads
    return recv.permute(1, 0, 2, 3, 4).reshape(B, P * Hl, L // P, D)


def head_to_tokens(t: torch.Tensor, group) -> torch.Tensor:
    """head_to_seq followed by the token-major flatten the output projection
    reads: [B, H/P, L, D] -> [B, L/P, H*D] with one copy after the all-to-all."""
    P = dist.get_world_size(group)
    B, Hl, L, D = t.shape
    send = t.reshape(B, Hl, P, L // P, D).permute(2, 0, 1, 3, 4).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)         # recv[src] = my tokens of src's heads
    return recv.permute(1, 3, 0, 2, 4).reshape(B, L // P, P * Hl * D)


def pasa_core(density: float) -> Callable:
    """PASA as the self-attention core; its output is stored token-major so
    the output projection reads it without a transpose copy."""
    def core(q, k, v):
        return ops.pisa_pg_attention(q, k, v, density=density, out_layout="bthd")
    return core


def _self_attention(q, k, v, w, attn_core, group):
    """Head-major q, k, v of this rank's tokens -> the projected attention
    output [B, L_local, C]."""
    if group is not None:
        q, k, v = (seq_to_head(t, group) for t in (q, k, v))
    o = attn_core(q.contiguous(), k.contiguous(), v.contiguous())
    o = head_to_tokens(o, group) if group is not None else o.transpose(1, 2).flatten(2, 3)
    return F.linear(o, w["o"], w["o_b"])


def _cross_attention(cq, text, w, cfg, fused: bool):
    """cq [B, L, C] normalised queries -> the projected cross-attention output."""
    H, D = cfg.heads, cfg.head_dim
    if fused:
        ck = ops.dit_qkv_rope(F.linear(text, w["ck"], w["ck_b"]), None, None, w["cnorm_k_f"], None, None, None,
                              H, cfg.eps, head_major=False)[0]
    else:
        ck = rms_norm(F.linear(text, w["ck"], w["ck_b"]), w["cnorm_k"], cfg.eps)
    cv = F.linear(text, w["cv"], w["cv_b"])
    heads = lambda t: t.unflatten(2, (H, D)).transpose(1, 2)
    co = F.scaled_dot_product_attention(heads(cq), heads(ck), heads(cv))
    return F.linear(co.transpose(1, 2).flatten(2, 3), w["co"], w["co_b"])


def block_forward(x: torch.Tensor, text: torch.Tensor, temb: torch.Tensor, rope, w: dict, cfg: DiTConfig,
                  attn_core: Callable, group=None) -> torch.Tensor:
    """One block in torch ops on this rank's tokens.  x [B, L_local, C], text
    [B, Lt, C], temb [B, 6, C] fp32, rope = float64 (cos, sin) of this rank's
    tokens."""
    B, Ll, C = x.shape
    H, D = cfg.heads, cfg.head_dim
    shift, scale, gate, c_shift, c_scale, c_gate = (w["scale_shift_table"] + temb.float()).chunk(6, dim=1)

    # 1. self-attention
    h = F.layer_norm(x.float(), (C,), eps=cfg.eps)
    h = (h * (1 + scale) + shift).to(x.dtype)
    q = rms_norm(F.linear(h, w["q"], w["q_b"]), w["norm_q"], cfg.eps)
    k = rms_norm(F.linear(h, w["k"], w["k_b"]), w["norm_k"], cfg.eps)
    v = F.linear(h, w["v"], w["v_b"])
    q, k, v = (t.unflatten(2, (H, D)).transpose(1, 2).contiguous() for t in (q, k, v))
    q, k = apply_rope(q, *rope), apply_rope(k, *rope)
    o = _self_attention(q, k, v, w, attn_core, group)
    x = (x.float() + o.float() * gate).to(x.dtype)

    # 2. cross-attention over the text tokens
    h = F.layer_norm(x.float(), (C,), w["norm2_w"], w["norm2_b"], eps=cfg.eps).to(x.dtype)
    cq = rms_norm(F.linear(h, w["cq"], w["cq_b"]), w["cnorm_q"], cfg.eps)
    x = x + _cross_attention(cq, text, w, cfg, fused=False)

    # 3. feed-forward
    h = F.layer_norm(x.float(), (C,), eps=cfg.eps)
    h = (h * (1 + c_scale) + c_shift).to(x.dtype)
    f = F.linear(F.gelu(F.linear(h, w["ffn1"], w["ffn1_b"]), approximate="tanh"), w["ffn2"], w["ffn2_b"])
    return (x.float() + f.float() * c_gate).to(x.dtype)


Pending = Optional[Tuple[torch.Tensor, torch.Tensor]]


def block_forward_fused(x: torch.Tensor, pending: Pending, text: torch.Tensor, temb: torch.Tensor, rope, w: dict,
                        cfg: DiTConfig, attn_core: Callable, group=None, exchange=None) -> Tuple[torch.Tensor, Pending]:
    """One block with the row kernels; ``x`` (bf16, contiguous) is updated in
    place.  ``pending`` = (ffn output, its gate) of the previous block, whose
    residual update is folded into this block's first norm; the block returns
    its own pending pair.  With ``exchange`` (a ``UlyssesPeerExchange``) the
    sequence<->head exchange is done by the producer and the attention
    kernels themselves over peer memory, and PASA runs at ``cfg.density``."""
    mods = (w["scale_shift_table"] + temb.float()).chunk(6, dim=1)
    shift, scale, gate, c_shift, c_scale, c_gate = (m.contiguous() for m in mods)
    add, add_gate = pending if pending is not None else (None, None)

    # 1. (previous FFN residual) + LayerNorm + modulation -> self-attention
    h = ops.dit_row_norm(x, add=add, gate=add_gate, x_out=x if add is not None else None, scale=scale,
                         shift=shift, eps=cfg.eps)
    xq, xk, xv = F.linear(h, w["q"], w["q_b"]), F.linear(h, w["k"], w["k_b"]), F.linear(h, w["v"], w["v_b"])
    if exchange is not None:
        q, k, v = exchange.scatter_qkv(xq, xk, xv, w["norm_q_f"], w["norm_k_f"], rope[0], rope[1], cfg.eps)
        o = F.linear(exchange.attention(q, k, v, cfg.density), w["o"], w["o_b"])
    else:
        q, k, v = ops.dit_qkv_rope(xq, xk, xv, w["norm_q_f"], w["norm_k_f"], rope[0], rope[1], cfg.heads, cfg.eps,
                                   head_major=True)
        o = _self_attention(q, k, v, w, attn_core, group)

    # 2. gated residual + affine LayerNorm -> cross-attention
    h = ops.dit_row_norm(x, add=o, gate=gate, x_out=x, weight=w["norm2_w"], bias=w["norm2_b"], eps=cfg.eps)
    cq = ops.dit_qkv_rope(F.linear(h, w["cq"], w["cq_b"]), None, None, w["cnorm_q_f"], None, None, None,
                          cfg.heads, cfg.eps, head_major=False)[0]
    co = _cross_attention(cq, text, w, cfg, fused=True)

    # 3. residual + LayerNorm + modulation -> FFN (its residual goes to the next norm)
    h = ops.dit_row_norm(x, add=co, x_out=x, scale=c_scale, shift=c_shift, eps=cfg.eps)
    f = F.linear(F.gelu(F.linear(h, w["ffn1"], w["ffn1_b"]), approximate="tanh"), w["ffn2"], w["ffn2_b"])
    return x, (f, c_gate)


def init_embed(cfg: DiTConfig, seed: int, device, dtype=torch.bfloat16) -> dict:
    """Random weights of the patch embedding, the condition embedder and the
    output head (the model-level parts of one step)."""
    g = torch.Generator(device=device).manual_seed(seed)
    C = cfg.hidden

    def lin(out_f, in_f):
        return (torch.randn((out_f, in_f), generator=g, device=device, dtype=torch.float32) * 0.02).to(dtype)

    def vec(n):
        return (0.02 * torch.randn((n,), generator=g, device=device, dtype=torch.float32)).to(dtype)

    pin = cfg.in_channels * 4                       # one 1 x 2 x 2 latent patch
    return {
        "patch": lin(C, pin), "patch_b": vec(C),
        "t1": lin(C, cfg.freq_dim), "t1_b": vec(C), "t2": lin(C, C), "t2_b": vec(C),
        "tproj": lin(6 * C, C), "tproj_b": vec(6 * C),
        "x1": lin(C, cfg.text_dim), "x1_b": vec(C), "x2": lin(C, C), "x2_b": vec(C),
        "out_table": torch.randn((1, 2, C), generator=g, device=device, dtype=torch.float32) / C ** 0.5,
        "proj_out": lin(pin, C), "proj_out_b": vec(pin),
    }


def patchify(latents: torch.Tensor) -> torch.Tensor:
    """[B, c, F, 2h, 2w] -> [B, F*h*w, c*4] patches, token order (frame, row,
    column) and features (channel, dy, dx) as a stride-(1,2,2) convolution sees them."""
    B, c, Fr, H2, W2 = latents.shape
    t = latents.reshape(B, c, Fr, H2 // 2, 2, W2 // 2, 2)
    return t.permute(0, 2, 3, 5, 1, 4, 6).reshape(B, Fr * (H2 // 2) * (W2 // 2), c * 4)


def unpatchify(tokens: torch.Tensor, cfg: DiTConfig) -> torch.Tensor:
    """Inverse of patchify: [B, F*h*w, c*4] -> [B, c, F, 2h, 2w]."""
    B = tokens.shape[0]
    t = tokens.reshape(B, cfg.frames, cfg.height, cfg.width, cfg.in_channels, 2, 2)
    return t.permute(0, 4, 1, 2, 5, 3, 6).reshape(B, cfg.in_channels, cfg.frames, 2 * cfg.height, 2 * cfg.width)


def timestep_features(t: torch.Tensor, dim: int) -> torch.Tensor:
    """Sinusoidal timestep features [B, dim], cosines first."""
    half = dim // 2
    freqs = torch.exp(-math.log(10000.0) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
    ang = t.float().reshape(-1, 1) * freqs[None, :]
    return torch.cat((torch.cos(ang), torch.sin(ang)), dim=1)


def condition(e: dict, timestep: torch.Tensor, text_embed: torch.Tensor):
    """temb [B, C] fp32, the blocks' modulation [B, 6, C] fp32 and the
    projected text [B, Lt, C]."""
    dt = e["t1"].dtype
    f = timestep_features(timestep, e["t1"].shape[1]).to(dt)
    temb = F.linear(F.silu(F.linear(f, e["t1"], e["t1_b"])), e["t2"], e["t2_b"])
    tproj = F.linear(F.silu(temb), e["tproj"], e["tproj_b"])
    text = F.linear(F.gelu(F.linear(text_embed.to(dt), e["x1"], e["x1_b"]), approximate="tanh"), e["x2"], e["x2_b"])
    return temb.float(), tproj.float().unflatten(1, (6, -1)), text


def step(latents_local: torch.Tensor, timestep: torch.Tensor, text_embed: torch.Tensor, rope, embed: dict,
         blocks: List[dict], cfg: DiTConfig, attn_core: Callable, group=None, fused: bool = False,
         exchange=None) -> torch.Tensor:
    """One denoising step (the transformer forward of the reference's
    WanTransformer3DModel_Sparse.forward, svg/models/wan/custom_models.py:115-200)
    on this rank's tokens: patch embedding, condition embedder, every block,
    output norm and projection.  ``latents_local`` holds this rank's patches
    [B, L_local, c*4]; returns the predicted patches [B, L_local, c*4].
    ``fused`` selects the row-kernel path (bf16 CUDA tensors); ``exchange``
    (with ``fused``) replaces the NCCL all-to-alls by the peer-memory scatter."""
    temb, tproj, text = condition(embed, timestep, text_embed)
    x = F.linear(latents_local.to(embed["patch"].dtype), embed["patch"], embed["patch_b"])
    shift, scale = (embed["out_table"] + temb.unsqueeze(1)).chunk(2, dim=1)
    if fused:
        x = x.contiguous()
        pending: Pending = None
        for w in blocks:
            x, pending = block_forward_fused(x, pending, text, tproj, rope, w, cfg, attn_core, group, exchange)
        add, add_gate = pending if pending is not None else (None, None)
        h = ops.dit_row_norm(x, add=add, gate=add_gate, x_out=x if add is not None else None,
                             scale=scale.contiguous(), shift=shift.contiguous(), eps=cfg.eps)
    else:
        for w in blocks:
            x = block_forward(x, text, tproj, rope, w, cfg, attn_core, group)
        h = (F.layer_norm(x.float(), (cfg.hidden,), eps=cfg.eps) * (1 + scale) + shift).to(x.dtype)
    return F.linear(h, embed["proj_out"], embed["proj_out_b"])


def local_slice(cfg: DiTConfig, rank: int, world: int):
    """Token range [t0, t1) of a rank (T divisible by the world size)."""
    if cfg.tokens % world:
        raise ValueError(f"{cfg.tokens} tokens do not split over {world} ranks")
    n = cfg.tokens // world
    return rank * n, (rank + 1) * n
