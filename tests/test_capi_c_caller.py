"""CPU: a plain C program compiles against include/tb_gemm.h, links
libtbgemm.so and drives the host side of the C ABI (plan, describe, the
program mapping, the reference-worded rejection) — the boundary a C/C++
caller of the reference's kernel switches to."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

from mini_triton_nvgpu_v1_b200 import _capi

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs a C compiler")
def test_plain_c_caller(tmp_path):
    exe = tmp_path / "capi_example"
    lib_dir = Path(_capi.LIB_PATH).parent
    subprocess.run(["gcc", "-std=c11", "-O1", "-I", str(ROOT / "include"), str(ROOT / "tests" / "capi_example.c"),
                    "-L", str(lib_dir), "-l:libtbgemm.so", f"-Wl,-rpath,{lib_dir}", "-o", str(exe)],
                   check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout + out.stderr
    text = out.stdout
    assert '"mapping_kind": "grouped_tile"' in text and '"total_programs": 6' in text
    # grouped order with group_m = 2 over 3 × 2 tiles (LowerPipelineToNVGPU.cpp:283-304)
    assert "pid 0 -> tile (0, 0)" in text and "pid 1 -> tile (1, 0)" in text and "pid 2 -> tile (0, 1)" in text
    assert "pid 4 -> tile (2, 0)" in text and "pid 5 -> tile (2, 1)" in text
    assert "rejected: stage1 requires block_m % 16 == 0" in text
    # N-shard columns: 32 tiles of 256 over 3 ranks -> 11, 11, 10 tiles
    assert "nshard rank 0: columns 0 + 2816, workspace 0" in text
    assert "nshard rank 1: columns 2816 + 2816" in text
    assert "nshard rank 2: columns 5632 + 2560" in text
