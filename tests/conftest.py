import gzip
import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
PKG = REPO / "faster-rl-training_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(PKG), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device; runs the kernels through the C ABI")


def gpu_available() -> bool:
    import torch

    return torch.cuda.is_available()


@pytest.fixture(scope="session")
def golden_traces():
    with gzip.open(GOLDEN / "cache_traces.json.gz", "rt") as f:
        return json.load(f)


@pytest.fixture(scope="session")
def golden_rollouts():
    arrays = np.load(GOLDEN / "rollouts.npz")
    meta = json.loads((GOLDEN / "rollouts.json").read_text())
    return arrays, meta


@pytest.fixture(scope="session")
def golden_tinylm():
    return np.load(GOLDEN / "tinylm.npz")


@pytest.fixture(scope="session")
def golden_rope():
    return np.load(GOLDEN / "rope.npz")


@pytest.fixture(scope="session")
def golden_evicted_at():
    return np.load(GOLDEN / "evicted_at.npz")
