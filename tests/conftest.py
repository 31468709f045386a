"""Shared pytest set-up: the ``gpu`` marker and golden-fixture helpers."""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(GOLDEN))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built CUDA library")


def golden_cases():
    return json.loads((GOLDEN / "manifest.json").read_text())


def load_golden(name):
    """(case dict, npz arrays, q, k, v as float32 torch CPU tensors)."""
    from make_golden import case_inputs, input_digest

    case = golden_cases()[name]
    q, k, v = case_inputs(case)
    assert input_digest(q, k, v) == case["digest"], "torch CPU random stream changed; regenerate the fixtures"
    arr = dict(np.load(GOLDEN / f"{name}.npz"))
    return case, arr, q, k, v


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability()
    if major != 10:
        pytest.skip("needs an sm_100 GPU")
    return torch.device("cuda:0")
