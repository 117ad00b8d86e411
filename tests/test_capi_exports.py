"""CPU: the C-ABI library loads without a GPU and exports every function
include/tb_gemm.h declares; argument errors are reported before any CUDA
call (no compute calls here)."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

from mini_triton_nvgpu_v1_b200 import _capi

HEADER = Path(__file__).resolve().parents[1] / "include" / "tb_gemm.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_]+\s*\*?\s*(tb_[a-z_]+)\s*\(", text, re.M)))


def test_header_declares_the_c_abi():
    names = declared_functions()
    for must in ("tb_matmul_desc_init", "tb_matmul_plan_create", "tb_matmul_run",
                 "tb_matmul_workspace_bytes", "tb_matmul_plan_destroy", "tb_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(str(_capi.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_bindings_cover_every_declared_symbol():
    assert set(declared_functions()) == set(_capi.PROTOTYPES)


def test_desc_init_defaults_match_reference_attribute_defaults():
    lib = _capi.load()
    d = _capi.tb_matmul_desc()
    assert lib.tb_matmul_desc_init(C.byref(d)) == 0
    assert (d.group_m, d.exact_tile, d.split_k, d.num_ctas, d.persistent) == (8, 1, 1, 1, 0)
    assert (d.a_dtype, d.b_dtype, d.c_dtype, d.beta) == (_capi.TB_F16, _capi.TB_F16, _capi.TB_F32, 1)


def test_null_arguments_are_rejected_without_touching_the_gpu():
    lib = _capi.load()
    assert lib.tb_matmul_desc_init(None) == _capi.TB_ERR_INVALID_ARGUMENT
    assert lib.tb_matmul_plan_create(None, -1, None) == _capi.TB_ERR_INVALID_ARGUMENT
    assert lib.tb_matmul_run(None, None, 0, None, 0, None, 0, None, 0, None) == _capi.TB_ERR_INVALID_ARGUMENT
    assert b"plan" in lib.tb_last_error()
    d = _capi.tb_matmul_desc()
    lib.tb_matmul_desc_init(C.byref(d))
    d.m, d.n, d.k, d.block_m, d.block_n, d.block_k = 64, 64, 32, 64, 64, 32
    plan = C.c_void_p()
    assert lib.tb_matmul_plan_create(C.byref(d), -1, C.byref(plan)) == 0
    # NULL operands, bad strides and a missing workspace fail before any launch
    assert lib.tb_matmul_run(plan, None, 32, None, 64, None, 64, None, 0, None) == _capi.TB_ERR_INVALID_ARGUMENT
    fake = C.c_void_p(0x1000)
    assert lib.tb_matmul_run(plan, fake, 16, fake, 64, fake, 64, None, 0, None) == _capi.TB_ERR_INVALID_ARGUMENT
    assert lib.tb_matmul_run(plan, fake, 36, fake, 64, fake, 64, None, 0, None) == _capi.TB_ERR_UNSUPPORTED
    assert lib.tb_matmul_run(plan, C.c_void_p(0x1008), 32, fake, 64, fake, 64, None, 0, None) \
        == _capi.TB_ERR_UNSUPPORTED
    lib.tb_matmul_plan_destroy(plan)
    d.split_k = 2
    assert lib.tb_matmul_plan_create(C.byref(d), -1, C.byref(plan)) == 0
    assert lib.tb_matmul_run(plan, fake, 64, fake, 64, fake, 64, None, 0, None) == _capi.TB_ERR_WORKSPACE
    lib.tb_matmul_plan_destroy(plan)


def test_describe_reports_buffer_size():
    lib = _capi.load()
    d = _capi.tb_matmul_desc()
    lib.tb_matmul_desc_init(C.byref(d))
    d.m, d.n, d.k, d.block_m, d.block_n, d.block_k = 64, 64, 32, 64, 64, 32
    plan = C.c_void_p()
    assert lib.tb_matmul_plan_create(C.byref(d), -1, C.byref(plan)) == 0
    need = C.c_size_t()
    small = C.create_string_buffer(4)
    assert lib.tb_matmul_plan_describe(plan, small, 4, C.byref(need)) == _capi.TB_ERR_INVALID_ARGUMENT
    assert need.value > 100
    lib.tb_matmul_plan_destroy(plan)


def test_version_string():
    assert b"sm_100a" in _capi.load().tb_version()


def test_kshard_nccl_rejects_bad_arguments_before_any_cuda_call():
    import mini_triton_nvgpu_v1_b200 as tb
    lib = _capi.load()
    plan = tb.MatmulPlan(tb.KernelConfig(m=512, n=512, k=1024, block_m=128, block_n=128, block_k=64))
    st = lib.tb_matmul_run_kshard_nccl(plan._h, None, None, 0, None, 0, None, 512, None, 0, None)
    assert st == _capi.TB_ERR_INVALID_ARGUMENT
    # staging m × n f32 (+ receive rows when ldc != n) + the plan's own workspace
    assert lib.tb_matmul_kshard_nccl_workspace_bytes(plan._h, 2, 512) == 512 * 512 * 4
    assert lib.tb_matmul_kshard_nccl_workspace_bytes(plan._h, 2, 520) == 512 * 512 * 4 + 256 * 512 * 4
    h = C.c_void_p()
    assert lib.tb_nccl_comm_create(3, 2, b"\0" * 128, C.byref(h)) == _capi.TB_ERR_INVALID_ARGUMENT


def test_missing_library_fails_loudly(tmp_path):
    """No CPU fallback: without the built library the bindings raise."""
    with pytest.raises(ImportError, match="no CPU fallback"):
        _capi.load(tmp_path / "libtbgemm.so")
