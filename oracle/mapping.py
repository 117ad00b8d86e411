"""Python restatement of the reference's knob legality and program mapping —
TEST INFRASTRUCTURE ONLY (the checker for the C ABI's plan).

Each function cites the reference code it follows (paths inside
zrqnwu/mini_triton_nvgpu_v1).
"""
from __future__ import annotations

from dataclasses import dataclass


MAX_WARPS_PER_CTA = 8  # maxWarpsPerCTA, lib/Analysis/TargetInfo.cpp:126


def cdiv(a: int, b: int) -> int:
    return (a + b - 1) // b


def verify_kernel_config(m, n, k, bm, bn, bk, num_warps, stages, group_m, exact_tile,
                         a="f16", b="f16", c="f32") -> str | None:
    """verifySupportedKernelConfig, lib/Analysis/KernelConfig.cpp:202-246.
    Returns the reference's error message, or None when legal (f16 C is
    accepted as this build's extension)."""
    if a != "f16" or b != "f16" or c not in ("f32", "f16"):
        return "stage1 currently supports fp16 x fp16 -> fp32 matmul kernels"
    if m <= 0 or n <= 0 or k <= 0:
        return "problem M/N/K must be positive"
    if bm <= 0 or bn <= 0 or bk <= 0:
        return "block M/N/K must be positive"
    if bm % 16 or bn % 8 or bk % 16:
        return ("stage1 requires block_m % 16 == 0, block_n % 8 == 0 and "
                "block_k % 16 == 0 for mma.sync m16n8k16 legality")
    if stages < 2 or stages > 4:
        return "stage1 currently supports num_stages in [2, 4]"
    if num_warps <= 0:
        return "num_warps must be positive"
    if group_m <= 0:
        return "group_m must be positive"
    if exact_tile and (m % bm or n % bn or k % bk):
        return "exact_tile=true requires problem M/N/K to be divisible by block M/N/K"
    return None


def warp_grid(num_warps: int, bm: int, bn: int) -> tuple[int, int] | None:
    """deriveWarpGrid, lib/Analysis/EncodingPlan.cpp:283-321 (m16n8k16)."""
    best = None
    best_m = best_n = -1
    for wm in range(1, num_warps + 1):
        if num_warps % wm:
            continue
        wn = num_warps // wm
        if bm % wm or bn % wn:
            continue
        tm, tn = bm // wm, bn // wn
        if tm % 16 or tn % 8:
            continue
        score = abs(tm - tn)
        if best is None or score < best or (score == best and (
                (bm >= bn and wm > best_m) or (bm < bn and wn > best_n))):
            best, best_m, best_n = score, wm, wn
    return None if best is None else (best_m, best_n)


@dataclass
class Mapping:
    kind: str
    tiles_m: int
    tiles_n: int
    tiles_k: int
    group_span_m: int
    group_span_n: int
    programs_per_group: int
    launch_group_count: int
    total_programs: int
    split_k: int
    num_ctas: int
    reduction: str
    mainline: str


def program_mapping(m, n, k, bm, bn, bk, group_m=8, split_k=1, persistent=False, num_ctas=1,
                    reduction_mode=None, num_sms=148, num_warps=4) -> Mapping:
    """deriveProgramMappingPlan, lib/Analysis/ProgramMappingPlan.cpp:329-458,
    deriveReductionPlan (ReductionPlan.cpp:137-192) and the mainline kind of
    ResourceClosurePlan.cpp:154-161."""
    tm, tn, tk = cdiv(m, bm), cdiv(n, bn), cdiv(k, bk)
    s = max(split_k, 1)
    if persistent and s != 1:
        raise ValueError("stage1 does not allow persistent and split-k in the same "
                         "program mapping contract yet")
    if num_ctas <= 0:
        raise ValueError("module attr `tb.num-ctas` must be positive")
    red = "none"
    if persistent:
        kind, span_m, span_n = "persistent_tile", 1, tn
        ppg, groups, total = tn, tm, tm * tn
        num_ctas = min(num_ctas, total)
        mainline = "persistent_tile_loop"
    elif s > 1:
        kind, span_m, span_n = "split_k", 1, tn * s
        ppg, groups, total = tn * s, tm, tm * tn * s
        red = "split_k_atomic" if reduction_mode == "split_k_parallel" else "split_k_serial"
        mainline = "split_k"
    elif max(1, group_m) > 1 and tm > 1 and tn > 1:
        kind, span_m, span_n = "grouped_tile", group_m, tn
        ppg, groups, total = group_m * tn, cdiv(tm, group_m), tm * tn
        mainline = "grouped_tile"
    else:
        kind, span_m, span_n = "tile", 1, tn
        ppg, groups, total = tn, tm, tm * tn
        mainline = "single_tile"
    if num_sms > 0 and num_warps > MAX_WARPS_PER_CTA:  # ProgramMappingPlan.cpp:446-449
        raise ValueError("num_warps exceeds target max warps per CTA")
    if persistent and num_ctas > num_sms:
        num_ctas = num_sms
    return Mapping(kind, tm, tn, tk, span_m, span_n, ppg, groups, total, s, num_ctas, red, mainline)


def program_work(mp: Mapping, pid: int) -> tuple[int, int, int, int, int]:
    """buildProgramWorkAssignment (LowerPipelineToNVGPU.cpp:279-323) and the
    split-K K range (buildSplitKGroupActivePredicate, :325-357):
    (tile_m, tile_n, part, k_tile_begin, k_tile_count)."""
    if mp.kind == "split_k":
        g, ing = divmod(pid, mp.programs_per_group)
        tile_n, part = divmod(ing, mp.split_k)
        base, extra = divmod(mp.tiles_k, mp.split_k)
        start = part * base + min(part, extra)
        count = base + (1 if part < extra else 0)
        return g, tile_n, part, start, count
    g = pid // mp.programs_per_group
    first_m = g * mp.group_span_m
    size_m = min(mp.group_span_m, mp.tiles_m - first_m)
    ing = pid % mp.programs_per_group
    return first_m + ing % size_m, ing // size_m, 0, 0, mp.tiles_k


def triton_program_tile(pid: int, m: int, n: int, bm: int, bn: int, group_m: int) -> tuple[int, int]:
    """The same mapping as the reference's Triton kernel states it
    (tools/build_triton_stage1_kernel.py:31-44) — a second, independent
    statement used to cross-check program_work."""
    num_pid_m, num_pid_n = cdiv(m, bm), cdiv(n, bn)
    if group_m > 1:
        per_group = group_m * num_pid_n
        gid = pid // per_group
        first = gid * group_m
        gsz = min(num_pid_m - first, group_m)
        pig = pid % per_group
        return first + pig % gsz, pig // gsz
    return pid // num_pid_n, pid % num_pid_n


def persistent_programs(total: int, resident: int, cta: int) -> list[int]:
    """Tile-stride loop of a persistent CTA (PersistentWorkPlan.cpp:112-125,
    LowerPipelineToNVGPU.cpp:2588-2598)."""
    return list(range(cta, total, resident))
