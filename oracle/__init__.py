"""CPU oracle for the `tb.matmul` path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm may import this package, and only as the checker or as the timed CPU
implementation; the product (mini_triton_nvgpu_v1_b200) never does.

* :func:`matmul_ref` — C_out = C_in + A·B, f16 inputs widened to f32, f32
  accumulation (the reference's op contract, see oracle/tb_oracle.c for the
  file:line citations), computed by the OpenMP C restatement.
* :mod:`oracle.mapping` — the reference's knob legality and program mapping
  restated in Python.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "libtboracle.so"
_lib = None


def build(force: bool = False) -> Path:
    src = HERE / "tb_oracle.c"
    if force or not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE), "-B", "libtboracle.so"], check=True)
    return LIB


def _load():
    global _lib
    if _lib is None:
        build()
        lib = C.CDLL(str(LIB))
        lib.tb_oracle_matmul.restype = None
        lib.tb_oracle_matmul.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p,
                                         C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int, C.c_int]
        lib.tb_oracle_max_threads.restype = C.c_int
        _lib = lib
    return _lib


def max_threads() -> int:
    return int(_load().tb_oracle_max_threads())


def matmul_ref(A: np.ndarray, B: np.ndarray, C_in: np.ndarray | None = None, beta: int = 1,
               threads: int = 0) -> np.ndarray:
    """f32 result of C_in + A·B (A [m,k] f16, B [k,n] f16, C_in [m,n] f32).
    Returns a new array; C_in is not modified."""
    A = np.ascontiguousarray(A, dtype=np.float16)
    B = np.ascontiguousarray(B, dtype=np.float16)
    m, k = A.shape
    k2, n = B.shape
    assert k == k2
    out = np.zeros((m, n), np.float32) if C_in is None else np.array(C_in, dtype=np.float32, copy=True)
    _load().tb_oracle_matmul(A.ctypes.data, k, B.ctypes.data, n, out.ctypes.data, n, m, n, k,
                             1 if (beta and C_in is not None) else 0, threads)
    return out


def tolerance(k: int) -> float:
    """max|C_gpu − C_ref| bound stated by the north star: 1e-2·sqrt(K/32)."""
    return 1e-2 * float(np.sqrt(k / 32.0))


def apply_epilogue(C: np.ndarray, bias=None, activation=None, clamp=None) -> np.ndarray:
    """The fused epilogue expressions in float64 (the order of the C ABI:
    bias per column, activation, clamp) applied to an f32 result."""
    v = C.astype(np.float64)
    if bias is not None:
        v = v + np.asarray(bias, np.float64)[None, :]
    if activation == "relu":
        v = np.maximum(v, 0.0)
    elif activation == "silu":
        v = v / (1.0 + np.exp(-v))
    elif activation == "gelu_tanh":
        v = 0.5 * v * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (v + 0.044715 * v ** 3)))
    if clamp is not None:
        v = np.clip(v, clamp[0], clamp[1])
    return v.astype(np.float32)
