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


@pytest.fixture(scope="session")
def shape3b_state_dicts():
    """The two-layer models with the benchmark's layer shapes (3B target seed 5,
    0.5B draft seed 6; biases and norm jitter), as tests/golden/make_golden.py made them."""
    from kvengine_b200.config import QWEN2_0_5B_L2, QWEN2_3B_L2
    from kvengine_b200.weights import init_state_dict

    return {
        "target": (QWEN2_3B_L2, init_state_dict(QWEN2_3B_L2, seed=5, bias_std=0.02, norm_jitter=0.1)),
        "draft": (QWEN2_0_5B_L2, init_state_dict(QWEN2_0_5B_L2, seed=6, bias_std=0.02, norm_jitter=0.1)),
    }


def top2_margins(top2: dict) -> list[float]:
    """Per-step margins (largest minus second largest logit) from a greedy run's
    top-2 record ({"values": [[v0, v1], ...]})."""
    return [float(v[0] - v[1]) for v in top2["values"]]


def first_divergence(got: list[int], want: list[int], margins: list[float] | None, tol: float):
    """Token-identity check with near-tie reporting.

    `margins[i]` is the reference's top-2 logit margin at the step that produced
    want[i]. Returns None when the sequences are equal; otherwise a dict naming
    the first differing position, with `near_tie` True when the margin there is
    below `tol` - the two candidates are closer than the logits tolerance, so
    either choice agrees numerically (bf16 logits over a 151,936-word vocabulary
    tie exactly every few dozen steps). Past a near-tie the two runs continue from
    different tokens and are not compared further. A caller reports near-ties
    and fails on everything else."""
    if got == want:
        return None
    i = next((j for j, (a, b) in enumerate(zip(got, want)) if a != b), min(len(got), len(want)))
    margin = float(margins[i]) if margins is not None and i < len(margins) else None
    return {"position": i, "got": got[i:i + 3], "want": want[i:i + 3], "margin": margin,
            "near_tie": margin is not None and margin < tol}
