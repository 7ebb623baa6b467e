"""Shared pytest setup: the `gpu` marker, import paths and common helpers."""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line(
        "markers", "gpu: needs a B200 (sm_100a) GPU and the built libkvm_sm100.so")


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device for GPU tests; fails (not skips) when there is none."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu-marked test run without a CUDA device")
    return torch.device("cuda:0")


def rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    """||got - ref||_2 / ||ref||_2 in float64."""
    g = np.asarray(got, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    den = np.linalg.norm(r)
    return float(np.linalg.norm(g - r) / (den if den > 0 else 1.0))


def to_bits(t):
    """bf16 torch tensor -> numpy uint16 bit patterns (host copy)."""
    import torch
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def from_bits(a: np.ndarray, device):
    """numpy uint16 bf16 bit patterns -> bf16 torch tensor on `device`."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a).view(np.int16))
    return t.view(torch.bfloat16).to(device)
