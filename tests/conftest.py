"""Shared test setup.

Markers: ``gpu`` tests need a CUDA device and call the engine through its C ABI
(libtie_b200.so); everything else runs on the CPU (the oracle against the golden
vectors, host-side logic, and that the library loads and exports its ABI).
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "transformer-inference-engine_b200")
for p in (PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libtie_b200.so")


def _have_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


HAVE_GPU = _have_gpu()


def pytest_collection_modifyitems(config, items):
    if HAVE_GPU:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


def golden(name: str):
    """The committed fixture tests/golden/<name>.npz and its metadata, or a skip."""
    import json
    path = os.path.join(GOLDEN, f"{name}.npz")
    if not os.path.exists(path):
        pytest.skip(f"golden fixture {name} not generated")
    with open(os.path.join(GOLDEN, f"{name}.json")) as f:
        meta = json.load(f)
    return dict(np.load(path)), meta


@pytest.fixture(scope="session")
def tiny_paths():
    from tie_b200 import synth
    return synth.ensure_model("tiny", seed=7, ln_affine="random")


@pytest.fixture(scope="session")
def mini_paths():
    from tie_b200 import synth
    return synth.ensure_model("mini", seed=7, ln_affine="random")


@pytest.fixture(scope="session")
def small_paths():
    from tie_b200 import synth
    return synth.ensure_model("small", seed=1234, ln_affine="unit")
