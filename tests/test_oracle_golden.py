"""CPU: the oracle against the golden vectors generated from the reference's
own statement of tb.matmul (tools/build_triton_stage1_kernel.py, run with the
Triton CPU interpreter by tests/golden/make_golden.py).

Both compute C_in + Σ_k f32(A)·f32(B) in f32; they may sum in a different
order, so the bound is a few f32 ulps of the accumulated magnitude, far
below the GPU tolerance 1e-2·sqrt(K/32)."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

import oracle
from conftest import make_inputs

GOLDEN = sorted((Path(__file__).parent / "golden").glob("golden_*.npz"))


def test_golden_fixtures_present():
    assert len(GOLDEN) >= 8


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_oracle_matches_reference_triton_statement(path):
    g = np.load(path)
    meta = json.loads(str(g["meta"]))
    ref = oracle.matmul_ref(g["A"], g["B"], g["C_in"])
    # k-term magnitudes bound the f32 reassociation error
    mag = np.abs(g["A"].astype(np.float32)) @ np.abs(g["B"].astype(np.float32)) + np.abs(g["C_in"])
    bound = 8 * np.finfo(np.float32).eps * mag + 1e-7
    assert np.all(np.abs(ref - g["C_out"]) <= bound), meta


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_golden_inputs_follow_the_seeded_generator(path):
    """The fixtures' inputs are exactly tests/conftest.make_inputs(seed), so
    GPU tests can regenerate them from the seed."""
    g = np.load(path)
    meta = json.loads(str(g["meta"]))
    A, B, C = make_inputs(meta["m"], meta["n"], meta["k"], meta["seed"], meta["dist"])
    assert np.array_equal(A, g["A"]) and np.array_equal(B, g["B"]) and np.array_equal(C, g["C_in"])


def test_golden_pins_accumulate_semantics():
    """C_in is nonzero in the fixtures and the reference keeps it: C_out − A·B
    equals C_in (the op is C += A·B, not C = A·B)."""
    g = np.load(GOLDEN[0])
    prod = g["A"].astype(np.float64) @ g["B"].astype(np.float64)
    assert np.abs(g["C_in"]).max() > 0.5
    assert np.allclose(g["C_out"] - prod, g["C_in"], atol=1e-4)


def test_oracle_beta0_and_ragged_shapes():
    rng = np.random.default_rng(3)
    for m, n, k in [(1, 1, 1), (7, 5, 3), (33, 65, 17), (130, 70, 260)]:
        A = rng.uniform(-1, 1, (m, k)).astype(np.float16)
        B = rng.uniform(-1, 1, (k, n)).astype(np.float16)
        C = rng.standard_normal((m, n)).astype(np.float32)
        want = A.astype(np.float64) @ B.astype(np.float64)
        assert np.allclose(oracle.matmul_ref(A, B), want, atol=1e-4)
        assert np.allclose(oracle.matmul_ref(A, B, C), want + C, atol=1e-4)
        assert np.allclose(oracle.matmul_ref(A, B, C, beta=0), want, atol=1e-4)


def test_oracle_f16_special_values():
    """The oracle's f16 widening is exact (subnormals, signed zero, inf)."""
    vals = np.array([0.0, -0.0, 1.0, -2.5, 6.1e-5, 5.96e-8, 65504.0, np.inf], dtype=np.float16)
    A = vals.reshape(-1, 1)
    B = np.ones((1, 1), np.float16)
    out = oracle.matmul_ref(A, B)[:, 0]
    assert np.array_equal(out[:-1], vals[:-1].astype(np.float32))
    assert np.isinf(out[-1])


def test_tolerance_formula():
    assert oracle.tolerance(32) == pytest.approx(1e-2)
    assert oracle.tolerance(8192) == pytest.approx(1e-2 * 16)
