"""Shared pytest setup.

`-m "not gpu"` runs the oracle, fixture, ABI-export and host-logic tests on
CPU; `-m gpu` runs the CUDA parity tests (they need a B200 and the built
libtle_attn.so, and fail loudly without them).
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", "tinyllama-engine_b200"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


def load_golden(name):
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    import tle  # noqa: F401  (raises if libtle_attn.so is missing)
    return torch.device("cuda:0")
