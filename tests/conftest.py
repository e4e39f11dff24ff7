"""Shared test setup.

* ``gpu`` marker: tests that launch CUDA kernels (run on a B200 with
  ``pytest -m gpu``); everything else runs on the CPU.
* The package lives in ``triton-kernel-test_b200/`` (importable as ``actcomp``)
  and the checker in ``oracle/`` (test infrastructure only).
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "triton-kernel-test_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden", "reference_golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def O():
    import oracle

    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


# ---------------------------------------------------------------- tensor <-> numpy helpers
def to_bf16(a: np.ndarray, device="cuda"):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).view(torch.bfloat16).to(device)


def bits(t) -> np.ndarray:
    import torch

    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)
