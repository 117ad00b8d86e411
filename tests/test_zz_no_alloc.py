"""The allocation-free entry point, tb_matmul_run_no_alloc.

Some callers cannot allocate device memory while they run: an inference
engine's plugin executing inside a memory plan fixed ahead of time, a service
that reserved all of its device memory at start-up, or a path where an
allocator call and the synchronisation it may bring are not allowed. For
them the library keeps its split-K scratch in a fixed 16 MiB device array
instead of a caller-provided workspace.

These tests call that entry point through the C ABI (ctypes, raw device
pointers) and check it against the regular entry point, tb_matmul_run with a
caller-owned workspace, and against the CPU oracle, on two calls in a row. The file is named so pytest
collects it last; it must pass both alone in a fresh process (the first call
on the device sets the scratch address up) and after the other tests.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import oracle
from conftest import make_inputs

pytestmark = pytest.mark.gpu

TOL_SCALE = 1e-2  # max|Δ| ≤ 1e-2·sqrt(K/32), the tolerance of the parity tests


def _plan(m, n, k, **knobs):
    import mini_triton_nvgpu_v1_b200 as tb
    return tb.MatmulPlan(tb.KernelConfig(m=m, n=n, k=k, **knobs), device=0)


def _run_regular(plan, tA, tB, tC, stream):
    import torch
    from mini_triton_nvgpu_v1_b200 import _capi
    lib = _capi.load()
    ws = torch.empty(plan.workspace_bytes, dtype=torch.uint8, device=tC.device)
    rc = lib.tb_matmul_run(plan._h, C.c_void_p(tA.data_ptr()), tA.stride(0),
                           C.c_void_p(tB.data_ptr()), tB.stride(0), C.c_void_p(tC.data_ptr()),
                           tC.stride(0), C.c_void_p(ws.data_ptr()), ws.numel(), C.c_void_p(stream))
    assert rc == 0, lib.tb_last_error().decode()


def _run_no_alloc(plan, tA, tB, tC, stream):
    from mini_triton_nvgpu_v1_b200 import _capi
    lib = _capi.load()
    return lib.tb_matmul_run_no_alloc(plan._h, C.c_void_p(tA.data_ptr()), tA.stride(0),
                                      C.c_void_p(tB.data_ptr()), tB.stride(0),
                                      C.c_void_p(tC.data_ptr()), tC.stride(0), C.c_void_p(stream))


@pytest.mark.parametrize("shape,knobs", [
    # 16 × 512 × 512 × 4 B = exactly the 16 MiB the scratch holds
    ((512, 512, 8192), dict(block_m=128, block_n=256, block_k=64, split_k=16,
                            reduction_mode="split_k_serial")),
    ((200, 136, 1000), dict(block_m=256, block_n=128, block_k=32, split_k=3, exact_tile=False,
                            reduction_mode="split_k_serial")),
])
def test_no_alloc_matches_regular_entry_point_twice(cuda, shape, knobs):
    import torch
    from mini_triton_nvgpu_v1_b200 import _capi
    lib = _capi.load()
    m, n, k = shape
    plan = _plan(m, n, k, **knobs)
    assert 0 < plan.workspace_bytes <= 16 << 20
    stream = torch.cuda.current_stream(cuda).cuda_stream
    tol = TOL_SCALE * float(np.sqrt(k / 32.0))
    for call, seed in enumerate((31, 32)):  # two calls in a row, different data
        A, B, Cin = make_inputs(m, n, k, seed, "uniform")
        tA, tB = torch.from_numpy(A).to(cuda), torch.from_numpy(B).to(cuda)
        want = torch.from_numpy(Cin).to(cuda)
        got = want.clone()
        _run_regular(plan, tA, tB, want, stream)
        rc = _run_no_alloc(plan, tA, tB, got, stream)
        assert rc == 0, lib.tb_last_error().decode()
        torch.cuda.synchronize()
        err = float((got - want).abs().max())
        assert err <= tol, f"call {call}: max|Δ| vs tb_matmul_run = {err} > {tol}"
        # and against the CPU oracle, so a fault the two entry points share
        # cannot pass unseen
        ref = oracle.matmul_ref(A, B, Cin)
        err_ref = float(np.abs(got.cpu().numpy() - ref).max())
        assert err_ref <= tol, f"call {call}: max|Δ| vs the oracle = {err_ref} > {tol}"


def test_no_alloc_rejects_plans_beyond_the_scratch(cuda):
    import torch
    from mini_triton_nvgpu_v1_b200 import _capi
    lib = _capi.load()
    plan = _plan(1024, 1024, 4096, block_m=128, block_n=256, block_k=64, split_k=8,
                 reduction_mode="split_k_serial")  # 32 MiB of partials
    assert plan.workspace_bytes > 16 << 20
    A, B, Cin = make_inputs(1024, 1024, 4096, 33, "uniform")
    tA, tB = torch.from_numpy(A).to(cuda), torch.from_numpy(B).to(cuda)
    tC = torch.from_numpy(Cin).to(cuda)
    rc = _run_no_alloc(plan, tA, tB, tC, torch.cuda.current_stream(cuda).cuda_stream)
    assert rc == _capi.TB_ERR_WORKSPACE
    assert "16777216" in lib.tb_last_error().decode()
    torch.cuda.synchronize()
    assert torch.equal(tC.cpu(), torch.from_numpy(Cin)), "a rejected call must not launch"
