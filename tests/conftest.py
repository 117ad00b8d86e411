"""Shared pytest setup: the `gpu` marker and seeded input generators that
follow the BASELINE configs' distributions."""
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
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def make_inputs(m: int, n: int, k: int, seed: int, dist: str = "uniform", c_in: str = "normal",
                c_dtype=np.float32):
    """Seeded f16 A[m,k], B[k,n] and C_in[m,n] (numpy default_rng(seed)).
    dist: "uniform" → U[-1,1]; "normal" → N(0,1)·0.1."""
    rng = np.random.default_rng(seed)
    if dist == "uniform":
        A = rng.uniform(-1, 1, (m, k)).astype(np.float16)
        B = rng.uniform(-1, 1, (k, n)).astype(np.float16)
    else:
        A = (rng.standard_normal((m, k)) * 0.1).astype(np.float16)
        B = (rng.standard_normal((k, n)) * 0.1).astype(np.float16)
    if c_in == "zeros":
        C = np.zeros((m, n), c_dtype)
    else:
        C = rng.standard_normal((m, n)).astype(c_dtype)
    return A, B, C


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
