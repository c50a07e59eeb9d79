"""Shared fixtures. Tests marked ``gpu`` need a CUDA device and the built library; the rest
run on CPU. GPU tests never skip silently: without a device they fail."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libmmfree_cuda.so")
    config.addinivalue_line("markers", "slow: writes a multi-GB blob or runs a long decode")


def golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, name)) as z:
        return {k: z[k] for k in z.files}


def bits_equal(a, b) -> bool:
    """Bit equality of float arrays, with every NaN equal to every NaN."""
    a, b = np.asarray(a), np.asarray(b)
    if a.shape != b.shape:
        return False
    if a.dtype != np.float32:
        return np.array_equal(a, b)
    na, nb = np.isnan(a), np.isnan(b)
    return bool(np.array_equal(na, nb) and
                np.array_equal(a[~na].view(np.uint32), b[~nb].view(np.uint32)))


@pytest.fixture(scope="session")
def orc():
    import oracle
    return oracle.Oracle()


@pytest.fixture(scope="session")
def blob_cache():
    d = os.environ.get("MMFREE_BLOB_CACHE", "/tmp/mmfree_blobs")
    os.makedirs(d, exist_ok=True)
    return d


@pytest.fixture(scope="session")
def cuda():
    import torch
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    from matmulfreellmcpu_b200 import _lib
    _lib.lib()  # the native library must load; no fallback exists
    return torch.device("cuda:0")
