"""Shared fixtures and the ``gpu`` marker.

Tests marked ``gpu`` need a CUDA device and the built ``libb200asr.so``; they are
skipped when no device is present, so ``pytest -m "not gpu"`` runs anywhere.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device and the built extension")
    config.addinivalue_line("markers", "slow: long-running")


def _has_gpu() -> bool:
    try:
        import torch
    except ImportError:
        return False
    return torch.cuda.is_available()


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="needs a CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 values."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def load_npz(name: str) -> dict:
    with np.load(GOLDEN / name) as data:
        return {k: data[k] for k in data.files}


def load_json(name: str):
    return json.loads((GOLDEN / name).read_text())


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN
