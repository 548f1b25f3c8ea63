"""Shared test setup: the `gpu` marker, repo-root import path, fixture loader."""
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name: str) -> dict:
    """Fixture `name` from tests/golden as a dict of numpy arrays / python scalars."""
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        out = {}
        for k in z.files:
            v = z[k]
            out[k] = v.item() if v.ndim == 0 else v
        return out


@pytest.fixture
def golden():
    return load_golden
