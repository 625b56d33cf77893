"""Shared test fixtures.

Markers: `gpu` tests need a B200 and call the sm_100a library through its C
ABI; everything else runs on CPU (oracle vs golden fixtures, host logic, the
library's exported symbols, gloo multi-process logic).
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 and the built sm_100a library")


def load_golden(name: str) -> dict:
    with open(os.path.join(GOLDEN, f"{name}.json")) as f:
        return json.load(f)["data"]


def load_golden_arrays(name: str):
    return np.load(os.path.join(GOLDEN, f"{name}.npz"))


@pytest.fixture(scope="session")
def cuda_device():
    assert torch.cuda.is_available(), "GPU test needs CUDA (run with -m 'not gpu' on CPU)"
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def tiny_state_dicts():
    """The two-layer models the golden fixtures were made with (seed 3, biases and norm jitter)."""
    from kvengine_b200.config import TINY, TINY_HD128
    from kvengine_b200.weights import init_state_dict

    return {
        "tiny": (TINY, init_state_dict(TINY, seed=3, bias_std=0.02, norm_jitter=0.1)),
        "tiny_hd128": (TINY_HD128, init_state_dict(TINY_HD128, seed=3, bias_std=0.02, norm_jitter=0.1)),
    }
