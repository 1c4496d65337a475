"""Shared fixtures. Tests marked ``gpu`` need a CUDA device (a B200); all
others run on the CPU. The oracle (oracle/) is the checker everywhere."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle, build
    build()
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference, reference_available
    if not reference_available():
        pytest.skip("compiled reference (oracle/_ref) not available")
    return Reference()


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for gpu-marked tests")
    from littlellm_b200 import build
    build.build()
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def ops(cuda):
    from littlellm_b200 import ops as _ops
    return _ops
