"""Text front-end for the reference's `tb.matmul` module spelling.

Accepts the MLIR the reference's examples and tests are written in::

    module attributes {"tb.num-warps" = 4 : i64, "tb.requested-stages" = 2 : i64,
                       "tb.split-k" = 2 : i64, "tb.reduction-mode" = "split_k_parallel"} {
      func.func @kernel(%A: memref<64x64xf16>, %B: memref<64x64xf16>, %C: memref<64x64xf32>) {
        tb.matmul %A, %B, %C {block_m = 64 : i64, block_n = 64 : i64, block_k = 32 : i64,
                              exact_tile = true}
          : memref<64x64xf16>, memref<64x64xf16>, memref<64x64xf32>
        func.return
      }
    }

and turns every `tb.matmul` into a :class:`KernelConfig`. Errors carry the
reference's diagnostics: the op verifier (lib/IR/TBOps.cpp:33-60, :176-184),
the module-attribute readers (lib/Analysis/KernelConfig.cpp:24-48,
ProgramMappingPlan.cpp:80-121). :func:`plan_facts` prints a plan in the
attribute spelling tb-opt attaches to `tb.pipeline_mainline`, so the facts the
reference's FileCheck tests look for can be read off a dry run.

CLI::

    python -m mini_triton_nvgpu_v1_b200.frontend FILE.mlir [--run] [--seed S]

prints the plan facts of each op; `--run` executes it on cuda:0 with seeded
inputs and prints the checksum line the reference's bench driver prints
(c00 / cmid / clast / checksum).
"""
from __future__ import annotations

import argparse
import re
import sys
from dataclasses import dataclass
from typing import Optional

from . import DynamicMatmulPlan, KernelConfig, MatmulPlan, TBError
from . import _capi

_ERR = _capi.TB_ERR_INVALID_ARGUMENT


@dataclass
class MatmulSpec:
    func: str
    config: KernelConfig
    a_type: str
    b_type: str
    c_type: str


def _strip_comments(text: str) -> str:
    return re.sub(r"//[^\n]*", "", text)


def _balanced(text: str, start: int) -> tuple[str, int]:
    """Content of the {...} starting at text[start] == '{' and the index after it."""
    depth = 0
    for i in range(start, len(text)):
        if text[i] == "{":
            depth += 1
        elif text[i] == "}":
            depth -= 1
            if depth == 0:
                return text[start + 1:i], i + 1
    raise TBError(_ERR, "unbalanced braces in module")


def _split_top(s: str) -> list[str]:
    out, depth, cur = [], 0, []
    for ch in s:
        if ch in "<{[(":
            depth += 1
        elif ch in ">}])":
            depth -= 1
        if ch == "," and depth == 0:
            out.append("".join(cur))
            cur = []
        else:
            cur.append(ch)
    if "".join(cur).strip():
        out.append("".join(cur))
    return [x.strip() for x in out if x.strip()]


def _parse_value(raw: str):
    """MLIR attribute value: `4 : i64`, `true`, `"text"`."""
    v = raw.strip()
    if v.startswith('"'):
        return ("string", v.strip('"'))
    if v in ("true", "false"):
        return ("bool", v == "true")
    m = re.fullmatch(r"(-?\d+)\s*(?::\s*(i\d+|index))?", v)
    if m:
        return ("int", int(m.group(1)))
    return ("other", v)


def _parse_attr_dict(body: str, quoted_keys: bool) -> dict:
    out = {}
    for item in _split_top(body):
        if "=" not in item:
            continue
        k, v = item.split("=", 1)
        k = k.strip()
        if quoted_keys:
            k = k.strip('"')
        out[k] = _parse_value(v)
    return out


_MEMREF = re.compile(r"memref<([^>]*)>")


def _memref(t: str):
    """('f16', [d0, d1]) of memref<d0xd1xf16>; '?' dims become None."""
    m = _MEMREF.fullmatch(t.strip())
    if not m:
        return None
    parts = m.group(1).split("x")
    elem = parts[-1].strip()
    dims = [None if p.strip() == "?" else int(p) for p in parts[:-1]]
    return elem, dims


def _op_error(msg: str) -> TBError:
    return TBError(_ERR, f"'tb.matmul' op {msg}")


def parse_module(text: str, allow_f16_c: bool = False, allow_dynamic: bool = False) -> list[MatmulSpec]:
    """Every tb.matmul of `text` as a MatmulSpec (knobs validated by the
    reference's rules when a plan is made). `allow_dynamic` accepts `?` dims
    (the reference rejects them): they stay None in the config and need a
    DynamicMatmulPlan."""
    text = _strip_comments(text)
    mod_attrs: dict = {}
    m = re.search(r"module\s+attributes\s*\{", text)
    if m:
        body, _ = _balanced(text, m.end() - 1)
        mod_attrs = _parse_attr_dict(body, quoted_keys=True)

    def req_i64(name):
        v = mod_attrs.get(name)
        if v is None or v[0] != "int":
            raise TBError(_ERR, f"missing module context attr `{name}`")
        return v[1]

    def opt(name, kind, default):
        v = mod_attrs.get(name)
        if v is None:
            return default
        if v[0] != kind:
            word = {"int": "an i64", "bool": "a bool", "string": "a string"}[kind]
            raise TBError(_ERR, f"module attr `{name}` must be {word} attribute")
        return v[1]

    specs = []
    for fm in re.finditer(r"func\.func\s+@([\w$.]+)\s*\(", text):
        # argument list up to the matching ')'
        depth, i = 1, fm.end()
        while depth and i < len(text):
            depth += {"(": 1, ")": -1}.get(text[i], 0)
            i += 1
        args = {}
        for a in _split_top(text[fm.end():i - 1]):
            am = re.fullmatch(r"%(\w+)\s*:\s*(.+)", a)
            if am:
                args[am.group(1)] = am.group(2).strip()
        body_start = text.index("{", i)
        body, _ = _balanced(text, body_start)
        for om in re.finditer(r"tb\.matmul\s+%(\w+)\s*,\s*%(\w+)\s*,\s*%(\w+)\s*\{", body):
            attrs_txt, _ = _balanced(body, om.end() - 1)
            attrs = _parse_attr_dict(attrs_txt, quoted_keys=False)
            types = [args.get(om.group(j)) for j in (1, 2, 3)]
            if any(t is None for t in types):
                raise _op_error("operands must be function arguments of memref type")
            parsed = [_memref(t) for t in types]
            for p, name in zip(parsed, "abc"):
                if p is None:
                    raise TBError(_ERR, "tb.matmul operands must be memrefs")
                if len(p[1]) != 2:
                    raise TBError(_ERR, "tb.matmul currently requires rank-2 memrefs")
            (ae, ad), (be, bd), (ce, cd) = parsed
            c_ok = ce == "f32" or (allow_f16_c and ce == "f16")
            if ae != "f16" or be != "f16" or not c_ok:
                raise _op_error("expected fp16 x fp16 -> fp32 operand element types")

            def mismatch(x, y):
                return x is not None and y is not None and x != y
            if mismatch(ad[1], bd[0]) or mismatch(ad[0], cd[0]) or mismatch(bd[1], cd[1]):
                raise _op_error("expected A:[M,K], B:[K,N], C:[M,N] operand shapes")
            if None in ad + bd + cd and not allow_dynamic:
                raise TBError(_ERR, "stage1 supported envelope currently requires static "
                                    "rank-2 memrefs to derive problem shape coverage")

            def op_i64(name, default=None):
                v = attrs.get(name)
                if v is None:
                    if default is None:
                        raise _op_error(f"requires attribute '{name}'")
                    return default
                return v[1]
            bm, bn, bk = op_i64("block_m"), op_i64("block_n"), op_i64("block_k")
            if bm <= 0 or bn <= 0 or bk <= 0:
                raise _op_error("block sizes must be positive")
            gm = op_i64("group_m", 8)
            if gm <= 0:
                raise _op_error("group_m must be positive")
            exact = attrs.get("exact_tile", ("bool", True))[1]
            red = opt("tb.reduction-mode", "string", "")
            def pick(x, y):
                return x if x is not None else y
            cfg = KernelConfig(
                m=pick(ad[0], cd[0]), n=pick(bd[1], cd[1]), k=pick(ad[1], bd[0]), block_m=bm, block_n=bn, block_k=bk, group_m=gm,
                exact_tile=bool(exact), num_warps=req_i64("tb.num-warps"),
                num_stages=req_i64("tb.requested-stages"), split_k=opt("tb.split-k", "int", 1),
                reduction_mode=red or None, persistent=opt("tb.persistent", "bool", False),
                num_ctas=opt("tb.num-ctas", "int", 1),
                programs_per_tile=opt("tb.programs-per-tile", "int", 0),
                c_dtype="f16" if ce == "f16" else "f32")
            specs.append(MatmulSpec(fm.group(1), cfg, types[0], types[1], types[2]))
    if not specs:
        raise TBError(_ERR, "no tb.matmul op found")
    return specs


class _ShapeView:
    """plan_facts input made from a describe dict."""

    def __init__(self, info: dict):
        self.info = info


def plan_facts(plan: MatmulPlan) -> str:
    """The plan in the attribute spelling of tb-opt's pipeline_mainline
    attributes (tb.program_mapping_plan / tb.reduction_plan /
    tb.persistent_work_plan / resource closure / warp grid)."""
    i = plan.info
    red_kind = i["reduction_kind"] if i["reduction_kind"] != "none" else "none"
    lines = [
        "tb.pipeline_mainline",
        (f'tb.program_mapping_plan = {{mapping_kind = "{i["mapping_kind"]}", '
         f'launch_order = "{i["launch_order"]}", swizzle_kind = "{i["swizzle_kind"]}", '
         f'group_m = {i["group_m"]}, group_tile_span_m = {i["group_tile_span_m"]}, '
         f'group_tile_span_n = {i["group_tile_span_n"]}, '
         f'programs_per_launch_group = {i["programs_per_launch_group"]}, '
         f'launch_group_count = {i["launch_group_count"]}, total_programs = {i["total_programs"]}, '
         f'split_k = {i["split_k"]}, programs_per_tile = {i["programs_per_tile"]}, '
         f'num_ctas = {i["num_ctas"]}}}'),
        f'tb.reduction_plan = {{kind = "{red_kind}", split_k = {i["split_k"]}}}',
        (f'tb.persistent_work_plan = {{kind = "{i["persistent_kind"]}", '
         f'resident_programs = {i["resident_programs"]}}}'),
        f'selected_mainline_kind = "{i["selected_mainline_kind"]}"',
        f'num_warps = {i["num_warps"]}, warp_grid = array<i64: {i["warp_grid"][0]}, {i["warp_grid"][1]}>',
        (f'sm100 = {{kernel = "{i["kernel"]}", cta_tile = {i["cta_tile"]}, stages = {i["stages"]}, '
         f'grid = {i["grid"]}, epilogue = "{i["epilogue"]}", workspace_bytes = {i["workspace_bytes"]}}}'),
    ]
    return "\n".join(lines)


def checksum_line(C) -> str:
    """c00 / cmid / clast / checksum of an m×n result, the values the
    reference's bench driver prints per case (bench_stage1_fair.py:567-586)."""
    flat = C.reshape(-1)
    mid = flat.numel() // 2 if hasattr(flat, "numel") else flat.size // 2
    return (f"c00={float(flat[0]):.6g} cmid={float(flat[mid]):.6g} clast={float(flat[-1]):.6g} "
            f"checksum={float(flat.double().sum() if hasattr(flat, 'double') else flat.sum()):.6g}")


def dynamic_facts(plan: DynamicMatmulPlan) -> str:
    """The shape-independent facts of a dynamic plan, `?` for open dims."""
    i = plan.info
    dims = "x".join("?" if d is None else str(d) for d in i["problem"])
    return (f'tb.dynamic_plan = {{problem = "{dims}", tile = {i["tile"]}, num_warps = {i["num_warps"]}, '
            f'warp_grid = array<i64: {i["warp_grid"][0]}, {i["warp_grid"][1]}>, '
            f'split_k = {i["split_k"]}, reduction_kind = "{i["reduction_kind"]}", '
            f'persistent = {str(i["persistent"]).lower()}}}')


def run_spec(spec: MatmulSpec, seed: int = 0, device: int = 0, shape=None):
    """Runs one tb.matmul on seeded U[-1,1] inputs (C_in = 0) and returns C.
    `shape` (m, n, k) fills a dynamic spec's open dims (through one
    DynamicMatmulPlan)."""
    import torch
    from . import matmul
    cfg = spec.config
    dev = torch.device("cuda", device)
    m, n, k = shape if shape is not None else (cfg.m, cfg.n, cfg.k)
    g = torch.Generator(device=dev).manual_seed(seed)
    A = (torch.rand(m, k, device=dev, generator=g) * 2 - 1).half()
    B = (torch.rand(k, n, device=dev, generator=g) * 2 - 1).half()
    C = torch.zeros(m, n, device=dev,
                    dtype=torch.float16 if cfg.c_dtype == "f16" else torch.float32)
    if None in (cfg.m, cfg.n, cfg.k):
        DynamicMatmulPlan(cfg, device).run(A, B, C)
        torch.cuda.synchronize(dev)
        return A, B, C
    matmul(A, B, C, block_m=cfg.block_m, block_n=cfg.block_n, block_k=cfg.block_k,
           group_m=cfg.group_m, exact_tile=cfg.exact_tile, num_warps=cfg.num_warps,
           num_stages=cfg.num_stages, split_k=cfg.split_k, reduction_mode=cfg.reduction_mode,
           persistent=cfg.persistent, num_ctas=cfg.num_ctas)
    torch.cuda.synchronize(dev)
    return A, B, C


def main(argv: Optional[list] = None) -> int:
    ap = argparse.ArgumentParser(prog="python -m mini_triton_nvgpu_v1_b200.frontend")
    ap.add_argument("file")
    ap.add_argument("--run", action="store_true", help="execute on cuda:0 and print a checksum line")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--allow-f16-c", action="store_true")
    ap.add_argument("--dynamic", action="store_true",
                    help="accept `?` dims (one plan for every shape)")
    ap.add_argument("--shape", default=None, help="MxNxK for --run of a dynamic op")
    args = ap.parse_args(argv)
    try:
        specs = parse_module(open(args.file).read(), allow_f16_c=args.allow_f16_c,
                             allow_dynamic=args.dynamic)
        shape = tuple(int(x) for x in args.shape.split("x")) if args.shape else None
        for spec in specs:
            print(f"// @{spec.func}: tb.matmul {spec.a_type}, {spec.b_type}, {spec.c_type}")
            cfg = spec.config
            if None in (cfg.m, cfg.n, cfg.k):
                dplan = DynamicMatmulPlan(cfg, None)
                print(dynamic_facts(dplan))
                if shape is not None:
                    print(plan_facts(_ShapeView(dplan.shape_info(*shape))))
                if args.run:
                    if shape is None:
                        raise TBError(_ERR, "--run of an op with `?` dims needs --shape MxNxK")
                    _, _, C = run_spec(spec, args.seed, shape=shape)
                    print(checksum_line(C))
                continue
            plan = MatmulPlan(cfg, None)
            print(plan_facts(plan))
            if args.run:
                _, _, C = run_spec(spec, args.seed)
                print(checksum_line(C))
    except TBError as e:
        print(f"error: {e.message}", file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
