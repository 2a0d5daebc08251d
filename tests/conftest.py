"""Shared test setup: the ``gpu`` marker, package import by path, seeded inputs."""
from __future__ import annotations

import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PKG = "26mlsys-ae-ghostserve_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def pkg(sub: str = ""):
    """Import the engine package (or a submodule) by its directory name."""
    return importlib.import_module(PKG + ("." + sub if sub else ""))


def bf16_bits(rng: np.random.Generator, shape) -> np.ndarray:
    """Seeded bf16 N(0,1) bit patterns as uint16 (the KV the configs specify)."""
    x = rng.standard_normal(shape, dtype=np.float32)
    return (x.view(np.uint32) >> 16).astype(np.uint16)


def fp16_bits(rng: np.random.Generator, shape) -> np.ndarray:
    return rng.standard_normal(shape).astype(np.float16).view(np.uint16)


def rand_bytes(rng: np.random.Generator, n: int) -> np.ndarray:
    return rng.integers(0, 256, size=n, dtype=np.uint8)


@pytest.fixture
def rng():
    return np.random.default_rng(1234)
