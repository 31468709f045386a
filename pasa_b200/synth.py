"""Seeded synthetic inputs with the shapes and value distributions of the
op configurations the PASA north star names (no public dataset or model
checkpoint is involved: inputs are random, generated on the device).

Every head has its own generator seeded with ``seed * 1000 + head``, so a
head gets identical data whichever GPU (or how many GPUs) it is placed on.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    heads: int
    T: int
    D: int
    density: float
    dtype: torch.dtype
    kind: str            # "normal", "scaled", "ar1"
    frames: int = 1
    frame_tokens: int = 0
    text_tokens: int = 0

    @property
    def dtype_name(self) -> str:
        return "bf16" if self.dtype == torch.bfloat16 else "fp32"

    @property
    def NT(self) -> int:
        return -(-self.T // 64)

    @property
    def NS(self) -> int:
        return min(max(1, int(self.density * self.NT)), self.NT)

    @property
    def NG(self) -> int:
        return -(-self.NT // 32)

    def exact_flops(self, heads=None) -> float:
        """F_exact = 4 * H * NT * NS * 64^2 * D (selected 64x64 blocks)."""
        h = self.heads if heads is None else heads
        return 4.0 * h * self.NT * self.NS * 64 * 64 * self.D

    def corr_flops(self, heads=None) -> float:
        """Correction-phase work: H * NT * NG * (4*64*32*D + 2*64*D^2)."""
        h = self.heads if heads is None else heads
        return float(h * self.NT * self.NG) * (4 * 64 * 32 * self.D + 2 * 64 * self.D * self.D)


WORKLOADS = {
    # 1 x 4 x 1024 x 64, fp32, top-25% blocks
    "tiny": Workload("tiny", 4, 1024, 64, 0.25, torch.float32, "normal"),
    # Wan2.1-1.3B 480p, 21 x 30 x 52 latent, N(0,1)/sqrt(128)
    "wan1.3b-480p": Workload("wan1.3b-480p", 12, 32760, 128, 0.15, torch.bfloat16, "scaled", 21, 1560),
    # Wan2.1-14B 720p, 21 x 45 x 80 latent, AR(1) keys across frames
    "wan14b-720p": Workload("wan14b-720p", 40, 75600, 128, 0.10, torch.bfloat16, "ar1", 21, 3600),
    # HunyuanVideo 720p x 129 frames, 33 x 45 x 80 video + 256 text tokens
    "hunyuan-720p": Workload("hunyuan-720p", 24, 119056, 128, 0.10, torch.bfloat16, "normal", 33, 3600, 256),
}


def head_qkv(w: Workload, head: int, device, seed: int = 0):
    """q, k, v of one head, each [T, D] in the workload dtype."""
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1000 + head)
    shape = (w.T, w.D)
    q = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    v = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    if w.kind == "ar1":
        # k_f = 0.9 k_{f-1} + sqrt(1 - 0.81) eps_f over the frames, k_0 = eps_0
        eps = torch.randn((w.frames, w.frame_tokens, w.D), generator=g, device=device, dtype=torch.float32)
        k = torch.empty_like(eps)
        k[0] = eps[0]
        for f in range(1, w.frames):
            k[f] = 0.9 * k[f - 1] + (1.0 - 0.81) ** 0.5 * eps[f]
        k = k.reshape(shape)
    else:
        k = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    if w.kind == "scaled":
        s = w.D ** -0.5
        q, k, v = q * s, k * s, v * s
    return q.to(w.dtype), k.to(w.dtype), v.to(w.dtype)


def make_inputs(w: Workload, heads: range, device, seed: int = 0):
    """q, k, v of shape [1, len(heads), T, D] on ``device``."""
    qs, ks, vs = [], [], []
    for h in heads:
        q, k, v = head_qkv(w, h, device, seed)
        qs.append(q); ks.append(k); vs.append(v)
    stack = lambda xs: torch.stack(xs, 0).unsqueeze(0).contiguous()
    return stack(qs), stack(ks), stack(vs)


def shard_heads(total: int, rank: int, world: int) -> range:
    """Contiguous head range of one rank (sizes differ by at most one)."""
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def shard_blocks(heads: int, NT: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous range [begin, end) of the heads * NT query blocks (numbered
    head by head) of one rank, for head counts the world size does not
    divide: the ranks' block counts differ by at most three, and every
    boundary inside a head is even, so no pair of query blocks (one tile of
    the tensor-core kernel) is split between ranks."""
    total = heads * NT

    def cut(r):
        if r <= 0:
            return 0
        if r >= world:
            return total
        b = (r * total) // world
        h, j = divmod(b, NT)
        j -= j & 1  # even within the head
        return h * NT + j

    return cut(rank), cut(rank + 1)
