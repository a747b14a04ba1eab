"""Shared test setup: paths, the `gpu` marker, golden fixtures and a per-session GPU context."""

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "moa-workspace_b200"))
GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) and the built libg4b200.so")


@pytest.fixture(scope="session")
def golden_runs():
    return np.load(GOLDEN / "reference_runs.npz")


@pytest.fixture(scope="session")
def golden_boundary():
    return np.load(GOLDEN / "qkv_boundary.npz")


@pytest.fixture(scope="session")
def golden_stress():
    return np.load(GOLDEN / "ffn_stress.npz")


@pytest.fixture(scope="session")
def golden_attention():
    return np.load(GOLDEN / "attention_sdpa.npz")


@pytest.fixture(scope="session")
def device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from g4b200 import ops

    dev = ops.Device(0)
    yield dev
    dev.close()
