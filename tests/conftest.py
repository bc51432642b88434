"""Shared test configuration: the ``gpu`` marker and fixture loaders."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line(
        "markers", "gpu: needs a CUDA device (B200, sm_100a) and the built "
        "libamass_b200.so")


def bits_to_f32(a):
    """bf16 stored as int16 bits -> float32."""
    a = np.ascontiguousarray(a).view(np.uint16).astype(np.uint32) << 16
    return a.view(np.float32)


def load_golden(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"), allow_pickle=False)
    return {k: z[k] for k in z.files}


@pytest.fixture
def golden():
    return load_golden
