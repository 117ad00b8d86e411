#!/usr/bin/env python3
"""Generates the golden fixtures under tests/golden/ from the reference.

Run in a container where the reference checkout is available (it is not on
the GPU box; the fixtures it writes are committed):

    python tests/golden/make_golden.py /path/to/mini_triton_nvgpu_v1

1. golden_<case>.npz — the reference's own statement of tb.matmul semantics,
   `matmul_kernel` in tools/build_triton_stage1_kernel.py:14-74 (C loaded as
   the accumulator init, `acc += tl.dot(a, b)` over BLOCK_K steps, masked
   ragged edges, GROUP_M program swizzle), executed with the Triton CPU
   interpreter (TRITON_INTERPRET=1) on seeded inputs with a NONZERO C_in, so
   the C += A·B contract is pinned, not just A·B. Split-K has no Triton
   statement in the reference; its golden value is the same op (split-K must
   reproduce it).
2. contract_facts.json — the structural facts the reference's FileCheck
   tests assert (test/Transforms/*.mlir): knobs parsed from each test's
   module, and the CHECK lines' key = value pairs.
"""
from __future__ import annotations

import importlib.util
import json
import os
import re
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402

HERE = Path(__file__).resolve().parent

# name, (m, n, k), Triton BLOCK_M/N/K, GROUP_M, exact_tile, dist, seed, c_in
CASES = [
    ("smoke_64x64x32", (64, 64, 32), (64, 64, 32), 1, True, "uniform", 0),
    ("ragged_96x80x32_t64", (96, 80, 32), (64, 64, 32), 1, False, "uniform", 1),
    ("ragged_96x80x32_t128", (96, 80, 32), (128, 128, 64), 1, False, "uniform", 1),
    ("grouped_192x128x32_g2", (192, 128, 32), (64, 64, 32), 2, True, "normal", 3),
    ("splitk_64x64x64", (64, 64, 64), (64, 64, 32), 1, True, "uniform", 5),
    ("persistent_192x128x32", (192, 128, 32), (64, 64, 32), 1, True, "uniform", 7),
    ("ragged_160x96x48", (160, 96, 48), (64, 64, 16), 1, False, "uniform", 8),
    ("grouped_256x192x96_g2", (256, 192, 96), (64, 64, 32), 2, True, "normal", 9),
]


def make_inputs(m, n, k, seed, dist):
    """Same generator as tests/conftest.make_inputs (numpy default_rng)."""
    rng = np.random.default_rng(seed)
    if dist == "uniform":
        A = rng.uniform(-1, 1, (m, k)).astype(np.float16)
        B = rng.uniform(-1, 1, (k, n)).astype(np.float16)
    else:
        A = (rng.standard_normal((m, k)) * 0.1).astype(np.float16)
        B = (rng.standard_normal((k, n)) * 0.1).astype(np.float16)
    C = rng.standard_normal((m, n)).astype(np.float32)
    return A, B, C


def run_reference_triton(ref_root: Path):
    import torch
    import triton
    spec = importlib.util.spec_from_file_location(
        "tb_ref_triton", ref_root / "tools" / "build_triton_stage1_kernel.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    for name, (m, n, k), (bm, bn, bk), gm, exact, dist, seed in CASES:
        A, B, C = make_inputs(m, n, k, seed, dist)
        tA, tB = torch.from_numpy(A), torch.from_numpy(B)
        tC = torch.from_numpy(C.copy())
        grid = (triton.cdiv(m, bm) * triton.cdiv(n, bn),)
        mod.matmul_kernel[grid](tA, tB, tC, tA.stride(0), tB.stride(0), tC.stride(0), m, n, k,
                                BLOCK_M=bm, BLOCK_N=bn, BLOCK_K=bk, GROUP_M=gm, EXACT_TILE=exact)
        np.savez_compressed(HERE / f"golden_{name}.npz", A=A, B=B, C_in=C, C_out=tC.numpy(),
                            meta=json.dumps(dict(m=m, n=n, k=k, block=[bm, bn, bk], group_m=gm,
                                                 exact_tile=exact, dist=dist, seed=seed)))
        print("wrote", name)


_KV = re.compile(r'([A-Za-z_]+)\s*=\s*("([^"]*)"|array<i64:\s*([0-9, ]+)>|[-0-9]+)')


def parse_lit(ref_root: Path):
    facts = {}
    for f in sorted((ref_root / "test" / "Transforms").glob("*.mlir")):
        text = f.read_text()
        mod_attrs = dict(re.findall(r'"(tb\.[a-z-]+)"\s*=\s*(true|false|"[^"]*"|[0-9]+)', text))
        op = re.search(r"tb\.matmul %A, %B, %C \{([^}]*)\}", text, re.S)
        shapes = re.findall(r"memref<(\d+)x(\d+)xf(16|32)>", text.split("func.func")[1]) if "func.func" in text else []
        checks = []
        for line in text.splitlines():
            if "// CHECK" not in line:
                continue
            body = line.split(":", 1)[1].strip()
            kvs = {}
            for key, raw, s, arr in _KV.findall(body):
                if s:
                    kvs[key] = s
                elif arr:
                    kvs[key] = [int(x) for x in arr.replace(" ", "").split(",")]
                else:
                    kvs[key] = int(raw) if raw.lstrip("-").isdigit() else raw
            checks.append({"line": body, "kv": kvs})
        entry = {"module_attrs": {k: v.strip('"') for k, v in mod_attrs.items()}, "checks": checks}
        if op:
            entry["op_attrs"] = dict(re.findall(r"([a-z_]+) = ([0-9a-z]+)", op.group(1)))
        if len(shapes) >= 3:
            (am, ak, _), (bk_, bn, _), (cm, cn, _) = shapes[:3]
            entry["problem"] = [int(am), int(bn), int(ak)]
        facts[f.name] = entry
    (HERE / "contract_facts.json").write_text(json.dumps(facts, indent=1, sort_keys=True))
    print("wrote contract_facts.json with", len(facts), "files")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout>")
    root = Path(sys.argv[1])
    run_reference_triton(root)
    parse_lit(root)
