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

SOURCES = ["tb_plan.cpp", "tb_dynamic.cpp", "tb_shard.cpp", "tb_launch.cu", "tb_peer.cu", "tb_nccl.cpp"]
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


def _run(cmd: list[str], verbose: bool) -> str:
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False) -> Path:
    """Compiles each source to an object (in parallel, under ``_build/``) and
    links ``libtbgemm.so``; skipped when the library is newer than every input."""
    inputs = [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] + [ROOT / "include" / "tb_gemm.h",
                                                                           Path(__file__)]
    if not force and not _stale(LIB, inputs):
        return LIB
    objdir = ROOT / "_build"
    objdir.mkdir(exist_ok=True)
    common = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-Wall", "--expt-relaxed-constexpr",
              "-I", str(ROOT / "include"), "-I", str(CSRC)]
    objs = [objdir / (s + ".o") for s in SOURCES]
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        outs = list(ex.map(lambda so: _run(common + (["-Xptxas", "-v"] if ptxas_v and so[0].endswith(".cu")
                                                     else []) + ["-c", str(CSRC / so[0]), "-o", str(so[1])],
                                           verbose), zip(SOURCES, objs)))
    tmp = LIB.with_suffix(".so.tmp")
    _run([nvcc(), *ARCH, "-shared", *[str(o) for o in objs], "-o", str(tmp), "-ldl"], verbose)
    if verbose or ptxas_v:
        print("".join(outs), file=sys.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_v="--ptxas-v" in sys.argv)
    print(LIB)
