"""Builds the in-tree shared library ``libtbgemm.so`` (the C ABI of
``include/tb_gemm.h``) with nvcc for sm_100a.

The library is written next to this file so it travels with the source tree;
``python -m mini_triton_nvgpu_v1_b200.build`` rebuilds it.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libtbgemm.so"

SOURCES = ["tb_plan.cpp", "tb_dynamic.cpp", "tb_launch.cu", "tb_peer.cu", "tb_nccl.cpp"]
HEADERS = ["tb_plan.h", "tb_mapping.h", "tb_sm100.cuh"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def _stale(out: Path, inputs: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(p.stat().st_mtime > t for p in inputs)


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False) -> Path:
    inputs = [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] + [ROOT / "include" / "tb_gemm.h",
                                                                           Path(__file__)]
    if not force and not _stale(LIB, inputs):
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [
        nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
        "-Xcompiler", "-Wall", "--expt-relaxed-constexpr",
        "-I", str(ROOT / "include"), "-I", str(CSRC),
        *(["-Xptxas", "-v"] if ptxas_v else []),
        *[str(CSRC / s) for s in SOURCES],
        "-o", str(tmp), "-ldl",
    ]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if verbose or ptxas_v:
        print(r.stdout, r.stderr, file=sys.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_v="--ptxas-v" in sys.argv)
    print(LIB)
