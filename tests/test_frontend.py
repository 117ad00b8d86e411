"""The `.mlir` front-end: the reference's tb.matmul module spelling → knobs →
plan, with the reference's diagnostics, and the plan facts its FileCheck
tests look for visible in the dry-run text."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

import mini_triton_nvgpu_v1_b200 as tb
from mini_triton_nvgpu_v1_b200 import frontend as fe

FACTS = json.loads((Path(__file__).parent / "golden" / "contract_facts.json").read_text())


def module_text(m, n, k, mod_attrs: dict, op_attrs: dict, c_elem="f32", a_elem="f16") -> str:
    def val(v):
        if v in ("true", "false") or isinstance(v, bool):
            return str(v).lower()
        if isinstance(v, str) and not v.lstrip("-").isdigit():
            return f'"{v}"'
        return f"{v} : i64"
    mattrs = ", ".join(f'"{key}" = {val(v)}' for key, v in mod_attrs.items())
    oattrs = ", ".join(f"{key} = {val(v)}" for key, v in op_attrs.items())
    head = f"module attributes {{{mattrs}}} {{" if mattrs else "module {"
    ta, tb_, tc = f"memref<{m}x{k}x{a_elem}>", f"memref<{k}x{n}xf16>", f"memref<{m}x{n}x{c_elem}>"
    return (f"{head}\n  // a comment with {{braces}}\n"
            f"  func.func @kernel(%A: {ta}, %B: {tb_},\n                    %C: {tc}) {{\n"
            f"    tb.matmul %A, %B, %C {{{oattrs}}}\n      : {ta}, {tb_}, {tc}\n"
            f"    func.return\n  }}\n}}\n")


NOT_APPLICABLE = {"perPhase", "maxPhase", "swizzlingByteWidth", "required_sync_kind",
                  "workspace_barrier_count", "workspace_sync_kind", "selected_buffering_kind",
                  "selected_c_landing_kind", "selected_shared_workspace_policy", "landing_owner",
                  "reorder_owner"}
NA_KINDS = {"register_pack_global_vector", "cta_shared_row_reorder"}


@pytest.mark.parametrize("name", [n for n, f in sorted(FACTS.items()) if "problem" in f])
def test_dry_run_prints_the_reference_plan_facts(name):
    f = FACTS[name]
    m, n, k = f["problem"]
    text = module_text(m, n, k, f["module_attrs"], f["op_attrs"])
    (spec,) = fe.parse_module(text)
    out = fe.plan_facts(tb.MatmulPlan(spec.config))
    for chk in f["checks"]:
        for key, v in chk["kv"].items():
            if key in NOT_APPLICABLE or (key == "kind" and v in NA_KINDS):
                continue
            want = (f"{key} = array<i64: {v[0]}, {v[1]}>" if isinstance(v, list)
                    else f'{key} = "{v}"' if isinstance(v, str) else f"{key} = {v}")
            assert want in out, (name, want, out)
    assert "tb.pipeline_mainline" in out


def test_defaults_and_knobs_parse():
    text = module_text(192, 128, 32, {"tb.num-warps": 4, "tb.requested-stages": 2,
                                      "tb.persistent": "true", "tb.num-ctas": 2},
                       {"block_m": 64, "block_n": 64, "block_k": 32})
    (spec,) = fe.parse_module(text)
    c = spec.config
    assert (c.m, c.n, c.k, c.block_m, c.block_n, c.block_k) == (192, 128, 32, 64, 64, 32)
    assert c.group_m == 8 and c.exact_tile and c.persistent and c.num_ctas == 2
    assert c.num_warps == 4 and c.num_stages == 2 and c.split_k == 1


@pytest.mark.parametrize("mutate,message", [
    (lambda t: t.replace('"tb.num-warps" = 4 : i64, ', ""), "missing module context attr `tb.num-warps`"),
    (lambda t: t.replace('"tb.requested-stages" = 2 : i64', '"tb.requested-stages" = "two"'),
     "missing module context attr `tb.requested-stages`"),
    (lambda t: t.replace("xf32>", "xf16>"), "'tb.matmul' op expected fp16 x fp16 -> fp32 operand element types"),
    (lambda t: t.replace("memref<96x32xf16>", "memref<96x48xf16>"),
     "'tb.matmul' op expected A:[M,K], B:[K,N], C:[M,N] operand shapes"),
    (lambda t: t.replace("96x32xf16", "?x32xf16").replace("96x80xf32", "?x80xf32"),
     "stage1 supported envelope currently requires static rank-2 memrefs"),
    (lambda t: t.replace("memref<96x32xf16>", "memref<96x32x1xf16>"), "tb.matmul currently requires rank-2 memrefs"),
    (lambda t: t.replace("block_m = 64 : i64", "block_m = 0 : i64"), "'tb.matmul' op block sizes must be positive"),
    (lambda t: t.replace('"tb.num-warps" = 4 : i64', '"tb.num-warps" = 4 : i64, "tb.persistent" = 3 : i64'),
     "module attr `tb.persistent` must be a bool attribute"),
    (lambda t: t.replace('"tb.num-warps" = 4 : i64', '"tb.num-warps" = 4 : i64, "tb.split-k" = "2"'),
     "module attr `tb.split-k` must be an i64 attribute"),
])
def test_reference_diagnostics(mutate, message):
    base = module_text(96, 80, 32, {"tb.num-warps": 4, "tb.requested-stages": 2},
                       {"block_m": 64, "block_n": 64, "block_k": 32, "exact_tile": "false"})
    with pytest.raises(tb.TBError) as e:
        fe.parse_module(mutate(base))
    assert message in e.value.message


def test_knob_errors_surface_at_plan_time():
    text = module_text(96, 80, 32, {"tb.num-warps": 4, "tb.requested-stages": 2},
                       {"block_m": 64, "block_n": 64, "block_k": 32})  # exact_tile defaults true
    (spec,) = fe.parse_module(text)
    with pytest.raises(tb.TBError, match="exact_tile=true requires"):
        tb.MatmulPlan(spec.config)


def test_f16_c_is_an_opt_in_extension():
    text = module_text(64, 64, 32, {"tb.num-warps": 4, "tb.requested-stages": 2},
                       {"block_m": 64, "block_n": 64, "block_k": 32}, c_elem="f16")
    with pytest.raises(tb.TBError):
        fe.parse_module(text)
    (spec,) = fe.parse_module(text, allow_f16_c=True)
    assert spec.config.c_dtype == "f16"


def test_cli_dry_run(tmp_path, capsys):
    p = tmp_path / "k.mlir"
    p.write_text(module_text(64, 64, 64, {"tb.num-warps": 1, "tb.requested-stages": 2, "tb.split-k": 2,
                                         "tb.reduction-mode": "split_k_parallel"},
                             {"block_m": 64, "block_n": 64, "block_k": 32, "exact_tile": "true"}))
    assert fe.main([str(p)]) == 0
    out = capsys.readouterr().out
    assert 'mapping_kind = "split_k"' in out and 'kind = "split_k_atomic"' in out
    bad = tmp_path / "bad.mlir"
    bad.write_text("module {}")
    assert fe.main([str(bad)]) == 1


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["grouped_mapping_contract.mlir", "splitk_mapping_contract.mlir",
                                  "persistent_mapping_contract.mlir", "non_exact_shared_pack_contract.mlir",
                                  "two_warp_shape_closure_contract.mlir"])
def test_run_from_module_text_matches_oracle(cuda, name):
    import oracle
    f = FACTS[name]
    m, n, k = f["problem"]
    (spec,) = fe.parse_module(module_text(m, n, k, f["module_attrs"], f["op_attrs"]))
    A, B, C = fe.run_spec(spec, seed=3)
    ref = oracle.matmul_ref(A.cpu().numpy(), B.cpu().numpy())
    assert float(np.abs(C.cpu().numpy() - ref).max()) <= oracle.tolerance(k)
    line = fe.checksum_line(C)
    assert line.startswith("c00=") and "checksum=" in line


DYN_TEXT = """module attributes {"tb.num-warps" = 4 : i64, "tb.requested-stages" = 2 : i64} {
  func.func @k(%A: memref<?x256xf16>, %B: memref<256x?xf16>, %C: memref<?x?xf32>) {
    tb.matmul %A, %B, %C {block_m = 128 : i64, block_n = 128 : i64, block_k = 64 : i64, exact_tile = false}
      : memref<?x256xf16>, memref<256x?xf16>, memref<?x?xf32>
    return
  }
}
"""


def test_dynamic_dims_are_opt_in(tmp_path, capsys):
    with pytest.raises(tb.TBError, match="requires static rank-2 memrefs"):
        fe.parse_module(DYN_TEXT)
    (spec,) = fe.parse_module(DYN_TEXT, allow_dynamic=True)
    assert (spec.config.m, spec.config.n, spec.config.k) == (None, None, 256)
    p = tmp_path / "dyn.mlir"
    p.write_text(DYN_TEXT)
    assert fe.main([str(p)]) == 1
    assert fe.main([str(p), "--dynamic", "--shape", "1000x512x256"]) == 0
    out = capsys.readouterr().out
    assert 'problem = "?x?x256"' in out and "total_programs = 32" in out
    # the open dims must agree with the static K
    assert fe.main([str(p), "--dynamic", "--shape", "1000x512x128"]) == 1


@pytest.mark.gpu
def test_dynamic_module_runs_at_two_shapes(cuda):
    import oracle
    (spec,) = fe.parse_module(DYN_TEXT, allow_dynamic=True)
    for shape in [(1000, 512, 256), (96, 80, 256)]:
        A, B, C = fe.run_spec(spec, seed=4, shape=shape)
        ref = oracle.matmul_ref(A.cpu().numpy(), B.cpu().numpy())
        assert float(np.abs(C.cpu().numpy() - ref).max()) <= oracle.tolerance(256)
