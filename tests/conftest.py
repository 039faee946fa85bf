"""Shared fixtures: the `gpu` marker, golden-vector loading and tolerances."""

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")
if REPO not in sys.path:
    sys.path.insert(0, REPO)

# Parity bars (rel-L2 = ||got-ref|| / ||ref||, max-rel = max|got-ref| / max|ref|):
# fp32 inputs against the fp32 reference algorithm; bf16 inputs against the
# reference algorithm run in fp32 on the same bf16-rounded inputs.
TOL_F32_REL_L2 = 1e-4
TOL_BF16_REL_L2 = 5e-3
TOL_BF16_MAX_REL = 2e-2


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and liballoy_ssd.so")


def load_golden(name):
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture
def golden():
    return load_golden
