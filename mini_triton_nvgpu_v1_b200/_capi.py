"""ctypes binding of the C ABI in ``include/tb_gemm.h`` (``libtbgemm.so``).

This is the binding a Python caller of the reference would add: one ctypes
prototype per exported symbol, no logic. The library is loaded from the
package directory; if it is missing the import fails loudly — there is no
CPU fallback.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libtbgemm.so"

TB_OK = 0
TB_ERR_INVALID_ARGUMENT = 1
TB_ERR_UNSUPPORTED = 2
TB_ERR_CUDA = 3
TB_ERR_DEVICE_TIMEOUT = 4
TB_ERR_WORKSPACE = 5
TB_ERR_NCCL = 6

TB_F16, TB_F32, TB_BF16 = 0, 1, 2
TB_REDUCTION_UNSET, TB_REDUCTION_SPLIT_K_SERIAL, TB_REDUCTION_SPLIT_K_PARALLEL = 0, 1, 2
TB_ACT_NONE, TB_ACT_RELU, TB_ACT_SILU, TB_ACT_GELU_TANH = 0, 1, 2, 3
ACTIVATIONS = {None: TB_ACT_NONE, "relu": TB_ACT_RELU, "silu": TB_ACT_SILU, "gelu_tanh": TB_ACT_GELU_TANH}

STATUS_NAMES = {
    TB_OK: "TB_OK",
    TB_ERR_INVALID_ARGUMENT: "TB_ERR_INVALID_ARGUMENT",
    TB_ERR_UNSUPPORTED: "TB_ERR_UNSUPPORTED",
    TB_ERR_CUDA: "TB_ERR_CUDA",
    TB_ERR_DEVICE_TIMEOUT: "TB_ERR_DEVICE_TIMEOUT",
    TB_ERR_WORKSPACE: "TB_ERR_WORKSPACE",
    TB_ERR_NCCL: "TB_ERR_NCCL",
}


class tb_matmul_desc(C.Structure):
    _fields_ = [
        ("m", C.c_int64), ("n", C.c_int64), ("k", C.c_int64),
        ("block_m", C.c_int64), ("block_n", C.c_int64), ("block_k", C.c_int64),
        ("group_m", C.c_int64),
        ("exact_tile", C.c_int32),
        ("num_warps", C.c_int64),
        ("num_stages", C.c_int64),
        ("split_k", C.c_int64),
        ("reduction_mode", C.c_int32),
        ("persistent", C.c_int32),
        ("num_ctas", C.c_int64),
        ("programs_per_tile", C.c_int64),
        ("a_dtype", C.c_int32), ("b_dtype", C.c_int32),
        ("c_dtype", C.c_int32),
        ("beta", C.c_int32),
        ("bias", C.c_int32),
        ("activation", C.c_int32),
        ("clamp", C.c_int32),
        ("clamp_lo", C.c_float), ("clamp_hi", C.c_float),
        ("a_col_major", C.c_int32), ("b_col_major", C.c_int32),
        ("deterministic", C.c_int32),
    ]


TB_DIM_DYNAMIC = -(1 << 63)  # INT64_MIN, MLIR's ShapedType::kDynamic


class tb_program_work(C.Structure):
    _fields_ = [
        ("tile_m", C.c_int64), ("tile_n", C.c_int64), ("split_part", C.c_int64),
        ("k_tile_begin", C.c_int64), ("k_tile_count", C.c_int64),
    ]


class tb_peer_handle(C.Structure):
    _fields_ = [("rows_ipc", C.c_ubyte * 64), ("rows_offset", C.c_int64), ("flags_ipc", C.c_ubyte * 64)]


# Every symbol include/tb_gemm.h declares, with its ctypes prototype.
PROTOTYPES = {
    "tb_matmul_desc_init": (C.c_int, [C.POINTER(tb_matmul_desc)]),
    "tb_matmul_plan_create": (C.c_int, [C.POINTER(tb_matmul_desc), C.c_int, C.POINTER(C.c_void_p)]),
    "tb_matmul_plan_destroy": (C.c_int, [C.c_void_p]),
    "tb_matmul_workspace_bytes": (C.c_size_t, [C.c_void_p]),
    "tb_matmul_plan_describe": (C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "tb_matmul_program_work": (C.c_int, [C.c_void_p, C.c_int64, C.POINTER(tb_program_work)]),
    "tb_matmul_run": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p, C.c_int64,
                                C.c_void_p, C.c_int64, C.c_void_p, C.c_size_t, C.c_void_p]),
    "tb_matmul_run_no_alloc": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p, C.c_int64,
                                         C.c_void_p, C.c_int64, C.c_void_p]),
    "tb_matmul_run_epilogue": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p, C.c_int64,
                                         C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_size_t,
                                         C.c_void_p]),
    "tb_matmul_plan_create_dynamic": (C.c_int, [C.POINTER(tb_matmul_desc), C.c_int, C.POINTER(C.c_void_p)]),
    "tb_matmul_workspace_bytes_dynamic": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_int64,
                                                    C.POINTER(C.c_size_t)]),
    "tb_matmul_run_dynamic": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_void_p, C.c_int64,
                                        C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p,
                                        C.c_void_p, C.c_size_t, C.c_void_p]),
    "tb_matmul_plan_for_shape": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_int64,
                                           C.POINTER(C.c_void_p)]),
    "tb_matmul": (C.c_int, [C.POINTER(tb_matmul_desc), C.c_void_p, C.c_int64, C.c_void_p, C.c_int64,
                            C.c_void_p, C.c_int64, C.c_void_p, C.c_size_t, C.c_void_p]),
    "tb_matmul_nshard_columns": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_int64),
                                           C.POINTER(C.c_int64)]),
    "tb_matmul_nshard_workspace_bytes": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_size_t)]),
    "tb_matmul_run_nshard": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int64, C.c_void_p,
                                       C.c_int64, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p,
                                       C.c_size_t, C.c_void_p]),
    "tb_peer_comm_create": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_int64, C.c_int64, C.c_int64,
                                      C.POINTER(C.c_void_p), C.POINTER(tb_peer_handle)]),
    "tb_peer_comm_connect": (C.c_int, [C.c_void_p, C.POINTER(tb_peer_handle)]),
    "tb_peer_barrier": (C.c_int, [C.c_void_p, C.c_void_p]),
    "tb_matmul_run_kshard_peer": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p,
                                            C.c_int64, C.c_void_p]),
    "tb_peer_comm_status": (C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(C.c_uint32)]),
    "tb_peer_comm_destroy": (C.c_int, [C.c_void_p]),
    "tb_nccl_unique_id": (C.c_int, [C.c_char_p]),
    "tb_nccl_comm_create": (C.c_int, [C.c_int, C.c_int, C.c_char_p, C.POINTER(C.c_void_p)]),
    "tb_nccl_comm_destroy": (C.c_int, [C.c_void_p]),
    "tb_matmul_kshard_nccl_workspace_bytes": (C.c_size_t, [C.c_void_p, C.c_int, C.c_int64]),
    "tb_matmul_run_kshard_nccl": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p,
                                            C.c_int64, C.c_void_p, C.c_int64, C.c_void_p, C.c_size_t,
                                            C.c_void_p]),
    "tb_selftest_bounded_wait": (C.c_int, [C.c_void_p, C.c_uint64]),
    "tb_device_status": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint32)]),
    "tb_last_error": (C.c_char_p, []),
    "tb_version": (C.c_char_p, []),
}


def load(path: Path = LIB_PATH) -> C.CDLL:
    if not path.exists():
        raise ImportError(
            f"{path} is missing: build it with `python -m mini_triton_nvgpu_v1_b200.build` "
            "(nvcc, sm_100a). There is no CPU fallback.")
    lib = C.CDLL(str(path))
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib
