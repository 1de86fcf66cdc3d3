"""Shared test setup.

Markers: ``gpu`` tests need a B200 (run with ``-m gpu``); everything else
runs on CPU (``-m "not gpu"``).  GPU tests fail, rather than skip, when no
CUDA device is visible, so that a broken box cannot pass silently.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def cuda():
    import torch
    assert torch.cuda.is_available(), "GPU test run without a visible CUDA device"
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def gdsq(cuda):
    """The C-ABI helpers (gdsllm_b200.capi) with the library loaded."""
    from gdsllm_b200 import capi
    return capi


@pytest.fixture(scope="session")
def ext(cuda):
    import gdsllm_b200
    return gdsllm_b200.ext()


def assert_f16_bitexact(a, b, what=""):
    """fp16 arrays equal bit for bit, except that NaN only has to match NaN."""
    a = np.asarray(a).view(np.uint16).reshape(-1)
    b = np.asarray(b).view(np.uint16).reshape(-1)
    assert a.shape == b.shape, (what, a.shape, b.shape)
    nan_a = ((a & 0x7C00) == 0x7C00) & ((a & 0x3FF) != 0)
    nan_b = ((b & 0x7C00) == 0x7C00) & ((b & 0x3FF) != 0)
    assert np.array_equal(nan_a, nan_b), f"{what}: NaN positions differ"
    diff = np.nonzero((a != b) & ~nan_a)[0]
    assert diff.size == 0, (f"{what}: {diff.size} of {a.size} values differ; first at {diff[:5]}: "
                            f"{a[diff[:5]]} vs {b[diff[:5]]}")
