"""Dynamic-shape plans: one plan, knobs validated once, run over many m×n×k.

The reference only takes static memrefs (lib/Analysis/KernelConfig.cpp:98-103);
a static plan with an open dim keeps that rejection and message. CPU tests
check validation and the per-shape plan facts (which must equal a static
plan's for the same shape); GPU tests check parity with the oracle over a
sequence of shapes on one plan."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import mini_triton_nvgpu_v1_b200 as tb
from mini_triton_nvgpu_v1_b200 import _capi
from conftest import make_inputs

KNOBS = dict(block_m=128, block_n=128, block_k=64, exact_tile=False)


def _cfg(m=None, n=None, k=None, **kw):
    knobs = dict(KNOBS)
    knobs.update(kw)
    return tb.KernelConfig(m=m, n=n, k=k, **knobs)


def test_static_plan_rejects_open_dims_with_reference_message():
    with pytest.raises(tb.TBError, match="requires static rank-2 memrefs"):
        tb.MatmulPlan(_cfg(None, 64, 64))


def test_dynamic_plan_validates_knobs_at_creation():
    with pytest.raises(tb.TBError, match="block_m % 16 == 0"):
        tb.DynamicMatmulPlan(_cfg(block_m=40))
    with pytest.raises(tb.TBError, match="persistent and split-k"):
        tb.DynamicMatmulPlan(_cfg(persistent=True, split_k=2))
    with pytest.raises(tb.TBError, match="problem M/N/K must be positive"):
        tb.DynamicMatmulPlan(_cfg(0, None, None))
    p = tb.DynamicMatmulPlan(_cfg(n=256))
    info = p.info
    assert info["dynamic"] is True and info["problem"] == [None, 256, None]
    assert info["shapes_cached"] == 0


SHAPES = [(64, 64, 32), (96, 80, 32), (192, 128, 32), (4096, 4096, 4096), (300, 512, 1000),
          (8192, 8192, 8192), (512, 512, 65536)]


@pytest.mark.parametrize("extra", [dict(), dict(group_m=2), dict(persistent=True, num_ctas=148),
                                   dict(split_k=4, reduction_mode="split_k_serial"),
                                   dict(split_k=2, reduction_mode="split_k_parallel"),
                                   dict(block_m=256, block_n=256)])
def test_shape_plans_equal_static_plans(extra):
    dyn = tb.DynamicMatmulPlan(_cfg(**extra))
    for (m, n, k) in SHAPES:
        got = dyn.shape_info(m, n, k)
        want = tb.MatmulPlan(_cfg(m, n, k, **extra)).info
        assert got == want, (m, n, k)
        assert dyn.workspace_bytes(m, n, k) == want["workspace_bytes"]
    assert dyn.info["shapes_derived"] == len(SHAPES)
    assert dyn.info["shapes_cached"] == len(SHAPES)


def test_exact_tile_is_checked_per_shape():
    dyn = tb.DynamicMatmulPlan(_cfg(exact_tile=True))
    dyn.shape_info(256, 128, 64)
    with pytest.raises(tb.TBError, match="exact_tile=true requires"):
        dyn.shape_info(96, 80, 32)


def test_static_dims_of_a_dynamic_plan_are_enforced():
    dyn = tb.DynamicMatmulPlan(_cfg(n=256, k=512))
    dyn.shape_info(1000, 256, 512)
    with pytest.raises(tb.TBError, match="differs from the plan's static dims"):
        dyn.shape_info(1000, 128, 512)


def test_static_entry_points_reject_a_dynamic_plan():
    lib = _capi.load()
    dyn = tb.DynamicMatmulPlan(_cfg())
    st = lib.tb_matmul_run(dyn._h, None, 0, None, 0, None, 0, None, 0, None)
    assert st == _capi.TB_ERR_INVALID_ARGUMENT
    assert b"tb_matmul_run_dynamic" in lib.tb_last_error()
    assert lib.tb_matmul_workspace_bytes(dyn._h) == 0
    w = _capi.tb_program_work()
    assert lib.tb_matmul_program_work(dyn._h, 0, C.byref(w)) == _capi.TB_ERR_INVALID_ARGUMENT
    st = lib.tb_matmul_run_no_alloc(dyn._h, None, 0, None, 0, None, 0, None)
    assert st == _capi.TB_ERR_INVALID_ARGUMENT
    # and a static plan is not run through the dynamic entry point
    stat = tb.MatmulPlan(_cfg(64, 64, 64))
    st = lib.tb_matmul_run_dynamic(stat._h, 64, 64, 64, None, 0, None, 0, None, 0, None, None, 0, None)
    assert st == _capi.TB_ERR_INVALID_ARGUMENT


def test_cache_is_bounded():
    dyn = tb.DynamicMatmulPlan(_cfg())
    for i in range(300):
        dyn.workspace_bytes(64 + i, 64, 64)
    info = dyn.info
    assert info["shapes_derived"] == 300
    assert 0 < info["shapes_cached"] <= 256


@pytest.mark.gpu
@pytest.mark.parametrize("extra", [dict(), dict(split_k=3, reduction_mode="split_k_serial"),
                                   dict(split_k=2, reduction_mode="split_k_parallel"),
                                   dict(block_m=256, block_n=256, persistent=True, num_ctas=148)])
def test_one_plan_many_shapes_match_oracle(cuda, extra):
    import torch
    import oracle
    dyn = tb.DynamicMatmulPlan(_cfg(**extra), 0)
    shapes = [(64, 64, 32), (96, 80, 32), (640, 384, 256), (130, 136, 40), (1024, 768, 512),
              (64, 64, 32)]
    for i, (m, n, k) in enumerate(shapes):
        A, B, Cin = make_inputs(m, n, k, 60 + i, "uniform")
        tC = torch.from_numpy(Cin).to(cuda)
        dyn.run(torch.from_numpy(A).to(cuda), torch.from_numpy(B).to(cuda), tC)
        torch.cuda.synchronize()
        assert tb.device_status() == 0
        err = float(np.abs(tC.cpu().numpy() - oracle.matmul_ref(A, B, Cin)).max())
        assert err <= oracle.tolerance(k), ((m, n, k), err)
    assert dyn.info["shapes_derived"] == len(set(shapes))


@pytest.mark.gpu
def test_dynamic_plan_with_bias_and_f16_out(cuda):
    import torch
    import oracle
    dyn = tb.DynamicMatmulPlan(_cfg(c_dtype="f16", bias=True, activation="relu", beta=0), 0)
    for i, (m, n, k) in enumerate([(256, 256, 128), (200, 136, 96)]):
        A, B, _ = make_inputs(m, n, k, 70 + i, "uniform")
        bias = np.random.default_rng(71 + i).standard_normal(n).astype(np.float32)
        tC = torch.empty(m, n, dtype=torch.float16, device=cuda)
        dyn.run(torch.from_numpy(A).to(cuda), torch.from_numpy(B).to(cuda), tC,
                bias=torch.from_numpy(bias).to(cuda))
        want = oracle.apply_epilogue(oracle.matmul_ref(A, B, None, beta=0), bias, "relu")
        tol = oracle.tolerance(k) + float(np.abs(np.spacing(want.astype(np.float16))).max())
        assert float(np.abs(tC.float().cpu().numpy() - want).max()) <= tol
