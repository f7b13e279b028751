"""Test configuration: import paths, the ``gpu`` marker, golden fixtures.

``-m "not gpu"`` runs on any machine (oracle vs golden vectors, host logic,
ABI loading); ``-m gpu`` needs a B200 and compares the CUDA path with the
oracle through the C ABI.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "vllm-ascend-quantized-kv-cache-hust_b200"
GOLDEN = ROOT / "tests" / "golden"
for p in (str(PKG), str(ROOT / "oracle"), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100 GPU (B200)")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    """name -> loaded npz of tests/golden/."""
    cache: dict[str, dict] = {}

    def load(name: str) -> dict:
        if name not in cache:
            with np.load(GOLDEN / f"{name}.npz") as f:
                cache[name] = {k: f[k] for k in f.files}
        return cache[name]

    return load


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)
