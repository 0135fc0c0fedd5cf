"""Shared test helpers: the ``gpu`` marker and golden-fixture loading."""

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(ROOT), str(Path(__file__).resolve().parent)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")


def golden(name: str):
    return np.load(GOLDEN / f"{name}.npz")


def have_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda():
    """The CUDA library, loaded; GPU tests fail (not skip) if it cannot load on a GPU box."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU in this process")
    from latent_b200 import _lib
    return _lib.lib()
