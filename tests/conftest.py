"""Shared pytest setup: the `gpu` marker, import paths and golden-fixture helpers."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "mla-cuda_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_golden(name: str):
    return np.load(GOLDEN / name)


def checksum(*ts) -> np.ndarray:
    """Same input checksum as tests/golden/make_golden.py."""
    return np.array([float(t.double().sum()) for t in ts] + [float(t.double().abs().sum()) for t in ts])


def rel_l2(a, b) -> float:
    a = torch.as_tensor(a).double().reshape(-1)
    b = torch.as_tensor(b).double().reshape(-1)
    return float((a - b).norm() / b.norm().clamp_min(1e-300))


def sampled(t: torch.Tensor, idx: np.ndarray) -> np.ndarray:
    return t.detach().double().reshape(-1).cpu().numpy()[idx]
