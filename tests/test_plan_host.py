"""CPU: the C ABI's plan (knob legality, program mapping, structural plan
facts) against the Python restatement of the reference (oracle.mapping) and
against the facts the reference's FileCheck tests assert
(tests/golden/contract_facts.json). No GPU: plans are created for a B200
without touching CUDA (device=None)."""
from __future__ import annotations

import itertools
import json
from pathlib import Path

import pytest

import mini_triton_nvgpu_v1_b200 as tb
from oracle import mapping as om

FACTS = json.loads((Path(__file__).parent / "golden" / "contract_facts.json").read_text())


def plan(m, n, k, bm, bn, bk, **kw):
    return tb.MatmulPlan(tb.KernelConfig(m=m, n=n, k=k, block_m=bm, block_n=bn, block_k=bk, **kw))


# ---------------------------------------------------------------- legality

LEGALITY_GRID = list(itertools.product(
    [(64, 64, 32), (96, 80, 32), (0, 64, 32), (64, 64, -1), (200, 120, 40)],
    [(64, 64, 32), (16, 8, 16), (24, 64, 32), (64, 12, 32), (64, 64, 24), (0, 64, 32), (128, 128, 64)],
    [2, 1, 5, 4],           # num_stages
    [4, 0, 1],              # num_warps
    [8, 0, 2],              # group_m
    [True, False],          # exact_tile
))


@pytest.mark.parametrize("case", LEGALITY_GRID[::7])
def test_legality_messages_match_reference(case):
    (m, n, k), (bm, bn, bk), st, nw, gm, ex = case
    want = om.verify_kernel_config(m, n, k, bm, bn, bk, nw, st, gm, ex)
    if want is None and om.warp_grid(nw, bm, bn) is None:
        want = ("failed to derive a legal warp grid from module num-warps, block shape and "
                "mma instruction shape")
    try:
        plan(m, n, k, bm, bn, bk, num_stages=st, num_warps=nw, group_m=gm, exact_tile=ex)
        got = None
    except tb.TBError as e:
        got = e.message
        assert e.code == 1, e
    assert got == want


def test_dtype_rule_and_f16_extension():
    with pytest.raises(tb.TBError, match="fp16 x fp16 -> fp32"):
        plan(64, 64, 32, 64, 64, 32, c_dtype="bf16")
    p = plan(64, 64, 32, 64, 64, 32, c_dtype="f16")
    assert p.info["dtypes"] == "f16xf16->f16"


def test_mapping_errors():
    with pytest.raises(tb.TBError, match="persistent and split-k"):
        plan(64, 64, 64, 64, 64, 32, persistent=True, split_k=2)
    with pytest.raises(tb.TBError, match="tb.num-ctas` must be positive"):
        plan(64, 64, 64, 64, 64, 32, num_ctas=0)
    with pytest.raises(tb.TBError, match="split_k_serial` or"):
        plan(64, 64, 64, 64, 64, 32, split_k=2, reduction_mode="bogus")


def test_split_k_below_one_is_clamped_like_the_reference():
    """ProgramMappingPlan.cpp:361 clamps split-k to >= 1 before its check."""
    p = plan(64, 64, 64, 64, 64, 32, split_k=0)
    assert p.info["mapping_kind"] == "tile" and p.info["split_k"] == 1


def test_num_warps_limit_matches_reference():
    """ProgramMappingPlan.cpp:446-449: more than maxWarpsPerCTA = 8 warps
    (TargetInfo.cpp:126) is rejected once the target's SM count is known."""
    p = plan(256, 256, 64, 128, 128, 32, num_warps=8)
    assert p.info["num_warps"] == 8
    for nw in (9, 16, 32):
        with pytest.raises(tb.TBError) as e:
            plan(256, 256, 64, 128, 128, 32, num_warps=nw)
        assert e.value.code == 1 and e.value.message == "num_warps exceeds target max warps per CTA"
        with pytest.raises(ValueError, match="num_warps exceeds target max warps per CTA"):
            om.program_mapping(256, 256, 64, 128, 128, 32, num_warps=nw)


@pytest.mark.parametrize("bm,bn,tile,sub", [
    (512, 256, "tb_gemm_sm100_pair_256x256", [2, 1]),
    (256, 1024, "tb_gemm_sm100_pair_256x256", [1, 4]),
    (512, 128, "tb_gemm_sm100_pair_256x128", [2, 1]),
    (128, 640, "tb_gemm_sm100_128x256", [1, 3]),
    (384, 384, "tb_gemm_sm100_pair_256x512", [2, 1]),
    (272, 64, "tb_gemm_sm100_pair_256x128", [2, 1]),
])
def test_large_program_tiles_run_as_subtiles(bm, bn, tile, sub):
    """KernelConfig.cpp:217-221 only asks block_m % 16 and block_n % 8: a
    program tile larger than every hardware tile runs as sub-tiles, with the
    reference's program mapping unchanged."""
    m, n = 2 * bm + 16, 3 * bn
    p = plan(m, n, 256, bm, bn, 64, exact_tile=False)
    info = p.info
    assert info["kernel"] == tile and info["program_subtiles"] == sub
    want = om.program_mapping(m, n, 256, bm, bn, 64)
    assert info["total_programs"] == want.total_programs
    assert info["work_items"] == want.total_programs * sub[0] * sub[1]
    assert info["fused_program_pairs"] == "none"


def test_tail_split_plan_facts():
    """8192 x 2048 x 8192 (one rank of a 4-way N-shard): 256 pair items on
    74 CTA pairs; two whole waves, then the last 108 items' 108 · 128 ring
    fills cut into 74 equal ranges (stream-K tail), at most three segments
    per slot. The 8-way slice (no whole wave first) stays whole. f16 C, beta = 0,
    split-K and deterministic plans keep whole items; 8192^3 (13.8 waves)
    gains too little."""
    p = plan(8192, 2048, 8192, 256, 256, 64)
    assert p.info["tail_split"] == {"whole_items": 148, "stream_k_items": 108, "slots": 74,
                                    "segments_per_slot": 3, "fills_per_item": 128}
    assert p.info["walk_positions"] == 148 + 3 * 74 and p.info["grid"] == 148
    # no whole wave before the tail: measured slower, kept whole
    assert plan(8192, 1024, 8192, 256, 256, 64).info["tail_split"] is None
    for kw in (dict(c_dtype="f16"), dict(beta=0), dict(deterministic=True), dict(split_k=2)):
        r = plan(8192, 1024, 8192, 256, 256, 64, **kw)
        assert r.info["tail_split"] is None, kw
    assert plan(8192, 8192, 8192, 256, 256, 64).info["tail_split"] is None


def _stream_k_cover(items, fills, slots, segs):
    """Restates the kernel's position → (item, fill range) rule and checks
    that the segments cover every fill of the tail exactly once."""
    U = items * fills
    seen = [[0] * fills for _ in range(items)]
    for seg in range(segs):
        for q in range(slots):
            u0, u1 = q * U // slots, (q + 1) * U // slots
            i = u0 // fills + seg
            if i >= items:
                continue
            b = i * fills
            f0, f1 = max(u0, b) - b, min(u1, b + fills) - b
            for f in range(f0, max(f0, f1)):
                seen[i][f] += 1
    return all(c == 1 for row in seen for c in row)


@pytest.mark.parametrize("n", [1024, 2048, 2560, 3072])
def test_stream_k_tail_covers_every_fill_once(n):
    p = plan(8192, n, 8192, 256, 256, 64)
    ts = p.info["tail_split"]
    if ts is None:
        pytest.skip("no tail for this shape")
    assert _stream_k_cover(ts["stream_k_items"], ts["fills_per_item"], ts["slots"], ts["segments_per_slot"])


# ---------------------------------------------------------------- mapping

MAP_CASES = [
    dict(m=192, n=128, k=32, bm=64, bn=64, bk=32, group_m=2),
    dict(m=192, n=128, k=32, bm=64, bn=64, bk=32, group_m=8),
    dict(m=8192, n=8192, k=8192, bm=256, bn=256, bk=64, group_m=8),
    dict(m=1000, n=700, k=520, bm=128, bn=256, bk=64, group_m=3),
    dict(m=96, n=80, k=32, bm=64, bn=64, bk=32, group_m=8),
    dict(m=64, n=64, k=64, bm=64, bn=64, bk=32, split_k=2, reduction_mode="split_k_parallel"),
    dict(m=512, n=512, k=65536, bm=128, bn=256, bk=64, split_k=16),
    dict(m=64, n=64, k=64, bm=64, bn=64, bk=32, split_k=4),
    dict(m=300, n=200, k=1000, bm=64, bn=64, bk=48 // 16 * 16, split_k=7),
    dict(m=192, n=128, k=32, bm=64, bn=64, bk=32, persistent=True, num_ctas=2),
    dict(m=8192, n=8192, k=64, bm=128, bn=128, bk=64, persistent=True, num_ctas=1000),
]


def _mk(c):
    kw = {k: v for k, v in c.items() if k not in ("m", "n", "k", "bm", "bn", "bk")}
    kw["exact_tile"] = c["m"] % c["bm"] == 0 and c["n"] % c["bn"] == 0 and c["k"] % c["bk"] == 0
    return plan(c["m"], c["n"], c["k"], c["bm"], c["bn"], c["bk"], **kw), om.program_mapping(
        c["m"], c["n"], c["k"], c["bm"], c["bn"], c["bk"], group_m=c.get("group_m", 8),
        split_k=c.get("split_k", 1), persistent=c.get("persistent", False),
        num_ctas=c.get("num_ctas", 1), reduction_mode=c.get("reduction_mode"))


@pytest.mark.parametrize("c", MAP_CASES, ids=[str(i) for i in range(len(MAP_CASES))])
def test_mapping_plan_matches_oracle(c):
    p, want = _mk(c)
    info = p.info
    assert info["mapping_kind"] == want.kind
    assert info["problem_tiles"] == [want.tiles_m, want.tiles_n, want.tiles_k]
    assert info["total_programs"] == want.total_programs
    assert info["launch_group_count"] == want.launch_group_count
    assert info["programs_per_launch_group"] == want.programs_per_group
    assert info["group_tile_span_m"] == want.group_span_m
    assert info["group_tile_span_n"] == want.group_span_n
    assert info["split_k"] == want.split_k
    assert info["reduction_kind"] == want.reduction
    assert info["selected_mainline_kind"] == want.mainline
    if c.get("persistent"):
        assert info["num_ctas"] == want.num_ctas
        assert info["resident_programs"] == min(want.num_ctas, 148)


@pytest.mark.parametrize("c", MAP_CASES, ids=[str(i) for i in range(len(MAP_CASES))])
def test_program_work_matches_oracle_and_covers_every_tile(c):
    p, want = _mk(c)
    total = p.total_programs
    step = max(1, total // 4096)  # every pid for small cases, a stride for 8192³
    seen = {}
    for pid in range(0, total, step):
        got = p.program_work(pid)
        assert got == om.program_work(want, pid), pid
        if want.kind != "split_k":
            tm, tn = om.triton_program_tile(pid, c["m"], c["n"], c["bm"], c["bn"],
                                            want.group_span_m if want.kind == "grouped_tile" else 1)
            assert (got[0], got[1]) == (tm, tn), pid
        seen.setdefault((got[0], got[1]), []).append((got[2], got[3], got[4]))
    if step == 1:
        # every (tile) exactly once, or split_k times with disjoint K ranges
        # covering all K tiles
        assert len(seen) == want.tiles_m * want.tiles_n
        for parts in seen.values():
            assert len(parts) == want.split_k
            ranges = sorted((b, b + cnt) for _, b, cnt in parts)
            cur = 0
            for b, e in ranges:
                assert b == cur
                cur = e
            assert cur == want.tiles_k


def test_persistent_stride_loop_visits_each_program_once():
    p = plan(192, 128, 32, 64, 64, 32, persistent=True, num_ctas=2)
    resident = p.info["resident_programs"]
    assert resident == 2
    visits = sorted(pid for cta in range(resident)
                    for pid in om.persistent_programs(p.total_programs, resident, cta))
    assert visits == list(range(p.total_programs))


def test_num_ctas_clamped_to_sms_and_programs():
    assert plan(8192, 8192, 64, 128, 128, 64, persistent=True, num_ctas=1000).info["num_ctas"] == 148
    assert plan(192, 128, 32, 64, 64, 32, persistent=True, num_ctas=100).info["num_ctas"] == 6


def test_program_pairing():
    """Two consecutive programs with adjacent tiles share a hardware tile when
    every pair in the launch order is aligned; the program set is unchanged."""
    p = plan(2048, 2048, 4096, 128, 128, 64)                     # grouped, group 8
    assert p.info["fused_program_pairs"] == "vertical" and p.info["kernel"] == "tb_gemm_sm100_pair_256x128"
    assert p.info["work_items"] * 2 == p.total_programs
    for w in range(0, p.info["work_items"], 37):
        a, b = p.program_work(2 * w), p.program_work(2 * w + 1)
        assert a[0] % 2 == 0 and b[0] == a[0] + 1 and b[1] == a[1]          # vertical neighbours
    # enough programs for every CTA pair: 2 × 2 blocks share a 256 × 256 pair tile
    f = plan(4096, 4096, 4096, 128, 128, 64)
    assert f.info["fused_program_pairs"] == "2x2" and f.info["kernel"] == "tb_gemm_sm100_pair_256x256"
    assert f.info["work_items"] * 4 == f.total_programs
    # 256 × 128 programs side by side in grouped order: one 256 × 256 pair tile
    h = plan(4096, 4096, 4096, 256, 128, 64)
    assert h.info["fused_program_pairs"] == "horizontal" and h.info["kernel"] == "tb_gemm_sm100_pair_256x256"
    assert h.info["work_items"] * 2 == h.total_programs
    q = plan(192, 128, 32, 64, 64, 32, persistent=True, num_ctas=2)          # row-major persistent
    assert q.info["fused_program_pairs"] == "horizontal"
    for w in range(q.info["work_items"]):
        a, b = q.program_work(2 * w), q.program_work(2 * w + 1)
        assert a[1] % 2 == 0 and b[1] == a[1] + 1 and b[0] == a[0]
    assert plan(192, 128, 32, 64, 64, 32, group_m=2).info["fused_program_pairs"] == "none"   # 3 tile rows
    assert plan(512, 512, 8192, 128, 256, 64, split_k=4).info["fused_program_pairs"] == "none"
    assert plan(8192, 8192, 8192, 256, 256, 64).info["fused_program_pairs"] == "none"


def test_workspace_bytes():
    assert plan(512, 512, 65536, 128, 256, 64, split_k=16).workspace_bytes == 16 * 512 * 512 * 4
    assert plan(512, 512, 65536, 128, 256, 64, split_k=16,
                reduction_mode="split_k_parallel").workspace_bytes == 0
    assert plan(8192, 8192, 8192, 256, 256, 64).workspace_bytes == 0


def test_hardware_tile_selection():
    assert plan(64, 64, 256, 64, 64, 32).info["kernel"] == "tb_gemm_sm100_128x64"
    assert plan(96, 80, 320, 128, 128, 64, exact_tile=False).info["kernel"] == "tb_gemm_sm100_128x128"
    assert plan(8192, 8192, 8192, 128, 256, 64, group_m=3).info["kernel"] == "tb_gemm_sm100_128x256"
    info = plan(8192, 8192, 8192, 256, 256, 64).info
    assert info["kernel"] == "tb_gemm_sm100_pair_256x256" and info["ctas_per_tile"] == 2
    assert info["grid"] == 148 and info["tmem_cols"] == 512 and info["smem_bytes"] <= 232448
    # block_n in (256, 512]: one 256 × 512 pair accumulator (two N = 256 MMAs)
    for bm, bn in ((256, 512), (128, 384)):
        info = plan(8192, 8192, 8192, bm, bn, 64, exact_tile=False).info
        assert info["kernel"] == "tb_gemm_sm100_pair_256x512" and info["tmem_cols"] == 512
        assert info["cta_tile"] == [256, 512, 64] and info["smem_bytes"] <= 232448


# ------------------------------------------- the reference's FileCheck facts

# Facts about the sm_80 mma.sync lowering (shared-memory swizzle of 16-byte
# chunks, register-pack C landing, CTA row reorder) have no counterpart in the
# sm_100a kernels (TMA 128-byte swizzle, TMEM accumulators) and are not
# asserted.
NOT_APPLICABLE = {"perPhase", "maxPhase", "swizzlingByteWidth", "kind:register_pack_global_vector",
                  "required_sync_kind", "kind:cta_shared_row_reorder", "workspace_barrier_count",
                  "workspace_sync_kind", "selected_buffering_kind", "selected_c_landing_kind",
                  "selected_shared_workspace_policy", "landing_owner", "reorder_owner"}

KEYMAP = {"kind:split_k_atomic": ("reduction_kind", "split_k_atomic"),
          "kind:tile_stride_loop": ("persistent_kind", "tile_stride_loop")}


@pytest.mark.parametrize("name", [n for n, f in sorted(FACTS.items()) if "problem" in f])
def test_reference_filecheck_facts(name):
    f = FACTS[name]
    ma, op = f["module_attrs"], f["op_attrs"]
    m, n, k = f["problem"]
    p = plan(m, n, k, int(op["block_m"]), int(op["block_n"]), int(op["block_k"]),
             exact_tile=op.get("exact_tile", "true") == "true", group_m=int(op.get("group_m", 8)),
             num_warps=int(ma["tb.num-warps"]), num_stages=int(ma["tb.requested-stages"]),
             split_k=int(ma.get("tb.split-k", 1)), reduction_mode=ma.get("tb.reduction-mode"),
             persistent=ma.get("tb.persistent") == "true", num_ctas=int(ma.get("tb.num-ctas", 1)))
    info = p.info
    checked = 0
    for chk in f["checks"]:
        for key, val in chk["kv"].items():
            tag = f"{key}:{val}" if key == "kind" else key
            if key in NOT_APPLICABLE or tag in NOT_APPLICABLE:
                continue
            if tag in KEYMAP:
                ikey, ival = KEYMAP[tag]
                assert info[ikey] == ival, (name, tag)
            else:
                assert info[key] == val, (name, key, info.get(key), val)
            checked += 1
    # every key = value fact was either asserted above or is listed as
    # sm_80-lowering-only in NOT_APPLICABLE (the loop fails on anything else)
    assert checked >= 0


def test_filecheck_facts_cover_the_mapping_contract():
    """Across the reference's lit tests, the mapping-level facts asserted
    here include every mapping kind this build plans."""
    kinds = {kv.get("mapping_kind") for f in FACTS.values() for c in f["checks"] for kv in [c["kv"]]}
    assert {"grouped_tile", "split_k", "persistent_tile"} <= kinds


# ------------------------------------------------- randomized mapping check
from hypothesis import assume, given, settings, strategies as st  # noqa: E402


@settings(max_examples=150, deadline=None)
@given(m=st.integers(1, 900), n=st.integers(1, 900), k=st.integers(16, 3000),
       bm=st.sampled_from([16, 64, 128, 256]), bn=st.sampled_from([8, 64, 128, 256]),
       bk=st.sampled_from([16, 32, 64]), group_m=st.integers(1, 9), split_k=st.integers(1, 9),
       persistent=st.booleans(), num_ctas=st.integers(1, 300))
def test_random_mappings_match_oracle(m, n, k, bm, bn, bk, group_m, split_k, persistent, num_ctas):
    """Any legal knob set: plan facts and every program's work equal the
    restatement of ProgramMappingPlan.cpp / LowerPipelineToNVGPU.cpp:279-357."""
    if persistent:
        split_k = 1
    assume(om.warp_grid(4, bm, bn) is not None)   # else the reference rejects the knobs
    p = plan(m, n, k, bm, bn, bk, group_m=group_m, split_k=split_k, persistent=persistent,
             num_ctas=num_ctas, exact_tile=False)
    want = om.program_mapping(m, n, k, bm, bn, bk, group_m=group_m, split_k=split_k,
                              persistent=persistent, num_ctas=num_ctas)
    info = p.info
    assert info["mapping_kind"] == want.kind
    assert info["total_programs"] == want.total_programs
    for pid in range(0, want.total_programs, max(1, want.total_programs // 512)):
        assert p.program_work(pid) == om.program_work(want, pid), pid


@pytest.mark.parametrize("n,bn,world", [(8192, 256, 8), (8192, 256, 3), (1000, 64, 4), (100, 64, 4),
                                        (4096, 128, 5)])
def test_nshard_columns_match_partition(n, bn, world):
    """tb_matmul_nshard_columns gives each rank whole block_n tiles, balanced,
    covering [0, n) once — the partition parallel.column_shard states."""
    from mini_triton_nvgpu_v1_b200 import parallel as par
    cfg = tb.KernelConfig(m=512, n=n, k=128, block_m=128, block_n=bn, block_k=64, exact_tile=False)
    end = 0
    for r in range(world):
        sh = par.NShard(cfg, r, world)
        assert (sh.col0, sh.ncols) == par.column_shard(n, world, r, bn)
        assert sh.col0 == end
        end += sh.ncols
    assert end == n


@pytest.mark.parametrize("shape,knobs,kernel", [
    ((64, 64, 32), dict(block_m=64, block_n=64, block_k=32), "tb_gemm_sm100_small_128x64"),
    ((96, 80, 32), dict(block_m=128, block_n=128, block_k=64, exact_tile=False), "tb_gemm_sm100_small_128x128"),
    ((192, 128, 32), dict(block_m=64, block_n=64, block_k=32, group_m=8), "tb_gemm_sm100_small_128x64"),
    ((64, 64, 64), dict(block_m=64, block_n=64, block_k=32, split_k=2), "tb_gemm_sm100_small_128x64"),
    ((192, 128, 32), dict(block_m=64, block_n=64, block_k=32, persistent=True, num_ctas=2),
     "tb_gemm_sm100_small_128x128"),
    ((512, 512, 512), dict(block_m=128, block_n=128, block_k=64), "tb_gemm_sm100_pair_256x128"),
    ((64, 64, 256), dict(block_m=64, block_n=64, block_k=32), "tb_gemm_sm100_128x64"),
    ((64, 512, 32), dict(block_m=64, block_n=512, block_k=32), "tb_gemm_sm100_pair_256x512"),
])
def test_small_problems_take_the_latency_kernel(shape, knobs, kernel):
    """Every work item within 128 K elements on a one-CTA tile at most 128
    wide: the latency kernel; anything else: the pipelined kernels."""
    m, n, k = shape
    assert tb.MatmulPlan(tb.KernelConfig(m=m, n=n, k=k, **knobs)).info["kernel"] == kernel
