"""Host-side helpers for running the op head-sharded over several ranks.

Heads are independent, so each rank owns a contiguous head range and runs
the op on it alone; torch.distributed is used only to line ranks up and to
take the slowest rank's time.  Works with the nccl (GPU) and gloo (CPU)
backends.
"""
from __future__ import annotations

import torch

from .synth import shard_blocks, shard_heads  # noqa: F401  (re-exported: the partitions)


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


def _parse_cpulist(text: str) -> set:
    cpus = set()
    for part in text.strip().split(","):
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-")
            cpus.update(range(int(a), int(b) + 1))
        else:
            cpus.add(int(part))
    return cpus


def gpu_numa_node(device_index: int, sysfs: str = "/sys") -> int:
    """NUMA node of a GPU's PCI device (-1 when the system does not say)."""
    props = torch.cuda.get_device_properties(device_index)
    bus = f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
    try:
        with open(f"{sysfs}/bus/pci/devices/{bus}/numa_node") as f:
            return int(f.read().strip())
    except (OSError, ValueError):
        return -1


def pin_to_gpu_numa(device_index: int, sysfs: str = "/sys") -> int:
    """Restrict this process to the CPU cores of its GPU's NUMA node, so that
    page-locked host buffers it allocates and touches afterwards live in the
    memory next to the GPU's PCIe root (first-touch placement) and host
    copies of several ranks do not all cross the socket interconnect.
    Returns the node, or -1 (and changes nothing) when it is unknown."""
    import os

    node = gpu_numa_node(device_index, sysfs)
    if node < 0:
        return -1
    try:
        with open(f"{sysfs}/devices/system/node/node{node}/cpulist") as f:
            cpus = _parse_cpulist(f.read()) & os.sched_getaffinity(0)
    except OSError:
        return -1
    if cpus:
        os.sched_setaffinity(0, cpus)
    return node
