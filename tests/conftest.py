"""Test configuration: the `gpu` marker (tests that need a B200 and the built CUDA library), and helpers shared by
the test files (golden fixtures, bf16 widening)."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a) and the built libbasal200.so")


def golden(name):
    """The arrays of tests/golden/<name>.npz (written by tests/golden/make_golden.py from the reference)."""
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        return {k: z[k] for k in z.files}


def widen_bf16(bits):
    """uint16 bf16 patterns -> fp32 values."""
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


@pytest.fixture
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
