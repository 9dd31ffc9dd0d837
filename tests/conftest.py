"""Shared test set-up: markers, golden fixtures, CUDA helpers.

Tests marked `gpu` run on a B200 (`pytest -m gpu`) and call the kernels through
the C ABI (ctypes) or the `deepseekrpc_cuda` extension; everything else runs on
CPU (`pytest -m "not gpu"`).
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built sm_100a library")


def load_golden(name: str):
    if name.endswith(".json"):
        return json.loads((GOLDEN / name).read_text())
    with np.load(GOLDEN / f"{name}.npz") as data:
        return {k: data[k] for k in data.files}


@pytest.fixture
def golden():
    return load_golden


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device; fails (does not skip) when the native library is absent."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from deepseekrpc_b200 import _native
    _native.library()  # raises ImportError when the library was not built
    assert _native.library().dsr_device_check() == 0, _native.last_error()
    return torch.device("cuda", torch.cuda.current_device())
