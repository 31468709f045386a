"""Host-side helpers for running the op head-sharded over several ranks.

Heads are independent, so each rank owns a contiguous head range and runs
the op on it alone; torch.distributed is used only to line ranks up and to
take the slowest rank's time.  Works with the nccl (GPU) and gloo (CPU)
backends.
"""
from __future__ import annotations

import torch

from .synth import shard_heads  # noqa: F401  (re-exported: the head partition)


def _device_for_backend():
    import torch.distributed as dist

    return torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else torch.device("cpu")


def max_over_ranks(x: float) -> float:
    """The maximum of a per-rank scalar (e.g. a time) over all ranks."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=_device_for_backend())
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier() -> None:
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()
