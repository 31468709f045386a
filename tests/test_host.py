"""Host-side mirror of the reference interface: argument handling that runs
before any kernel (CPU only)."""
import inspect

import pytest
import torch

import pasa_b200
from pasa_b200 import ops


def test_signature_matches_reference():
    sig = inspect.signature(pasa_b200.pisa_pg_attention)
    names = list(sig.parameters)[:12]
    assert names == ["q", "k", "v", "density", "timestep", "block_size", "group_size", "scale", "use_cov_bias",
                     "use_random", "verbose", "prompt_token_length"]
    d = {k: p.default for k, p in sig.parameters.items()}
    assert d["density"] == 0.15 and d["block_size"] == 64 and d["group_size"] == 32
    assert d["scale"] is None and d["use_cov_bias"] is True and d["use_random"] is False


def test_piecewise_alias_signature():
    sig = inspect.signature(pasa_b200.piecewise_sparse_attention)
    assert list(sig.parameters)[:6] == ["q", "k", "v", "density", "block_size", "use_random"]


def test_cpu_tensors_are_rejected_no_fallback():
    q = torch.randn(1, 1, 128, 64)
    with pytest.raises(ValueError, match="CUDA"):
        pasa_b200.pisa_pg_attention(q, q, q, density=0.5)


def test_bad_shapes_and_options_are_rejected():
    q = torch.randn(1, 1, 128, 64)
    with pytest.raises(ValueError):
        pasa_b200.pisa_pg_attention(q, q, q, block_size=128)
    with pytest.raises(ValueError):
        pasa_b200.pisa_pg_attention(q[0], q[0], q[0])
    with pytest.raises(ValueError):
        ops._dtype_code(torch.empty(1, dtype=torch.float16))


def test_numa_pinning_reads_sysfs(tmp_path, monkeypatch):
    """pin_to_gpu_numa: the GPU's PCI device's numa_node and that node's CPU
    list, intersected with the allowed CPUs (a fake sysfs tree)."""
    import os
    import types

    from pasa_b200 import dist as pdist

    props = types.SimpleNamespace(pci_domain_id=0, pci_bus_id=0x1b, pci_device_id=0)
    monkeypatch.setattr(pdist.torch.cuda, "get_device_properties", lambda i: props)
    dev = tmp_path / "bus" / "pci" / "devices" / "0000:1b:00.0"
    dev.mkdir(parents=True)
    (dev / "numa_node").write_text("1\n")
    node = tmp_path / "devices" / "system" / "node" / "node1"
    node.mkdir(parents=True)
    allowed = sorted(os.sched_getaffinity(0))
    (node / "cpulist").write_text(f"{allowed[0]}-{allowed[0]},{allowed[-1]}\n")
    seen = {}
    monkeypatch.setattr(os, "sched_setaffinity", lambda pid, cpus: seen.setdefault("cpus", set(cpus)))
    assert pdist.gpu_numa_node(0, str(tmp_path)) == 1
    assert pdist.pin_to_gpu_numa(0, str(tmp_path)) == 1
    assert seen["cpus"] == {allowed[0], allowed[-1]}
    (dev / "numa_node").write_text("-1\n")
    assert pdist.pin_to_gpu_numa(0, str(tmp_path)) == -1
