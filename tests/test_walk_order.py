"""CPU: the order in which resident CTAs take work items (the kernels' and the
plan's shared csrc/tb_mapping.h) is a permutation of the reference's
programs: every program once, fused pairs still adjacent tiles. Built with
the host compiler from the same header the sm_100a kernels include."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

import mini_triton_nvgpu_v1_b200 as tb

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs a host C++ compiler")
def test_walk_is_a_permutation_of_the_programs(tmp_path):
    exe = tmp_path / "walk_check"
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", str(ROOT / "mini_triton_nvgpu_v1_b200" / "csrc"),
                    str(ROOT / "tests" / "walk_check.cpp"), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0 and out.stdout.startswith("OK"), out.stdout


def test_plans_report_their_walk():
    kn = dict(block_m=256, block_n=256, block_k=64)
    assert tb.MatmulPlan(tb.KernelConfig(m=8192, n=8192, k=8192, **kn)).info["hardware_walk"] == \
        "serpentine_groups"
    assert tb.MatmulPlan(tb.KernelConfig(m=8192, n=8192, k=8192, persistent=True, num_ctas=148, **kn)) \
        .info["hardware_walk"] == "row_groups"
    assert tb.MatmulPlan(tb.KernelConfig(m=512, n=512, k=8192, split_k=4, **kn)).info["hardware_walk"] == \
        "program_order"
