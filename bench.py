#!/usr/bin/env python3
"""bench.py — TFLOP/s of the B200-native `tb.matmul` at 8192³ f16→f32.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one tb.matmul (C ← C_in + A·B, f16 A/B, f32 C) of the fixed
8192 × 8192 × 8192 problem with GROUP_M=8 program swizzle (the BASELINE
"Grouped-M swizzle" config). With N GPUs the same problem is sharded along
N: rank r owns 8192/N columns of B and C (whole 256-column program tiles), A
is replicated, no collective (strong scaling; `--scaling weak` gives every
rank a full 8192-column slice instead). Inputs are seeded synthetic
N(0,1)·0.1 f16; A+B+C exceed the 126 MB L2 at every N (A alone is 128 MiB),
so no flush is needed between steps.

JSON keys: value = whole-job TFLOP/s with inputs resident in HBM (CUDA
events, max over ranks); e2e = the same through the public API
(parallel.NShard → tb_matmul_run_nshard) with the step's inputs copied from
pinned host memory and C copied back inside the timed region; roofline = the
GEMM kernel's achieved TFLOP/s against the measured cuBLAS bf16 peak (burst
figure for a timed region under 0.5 s, sustained figure for longer ones);
cpu_baseline = the CPU oracle on the host cores.

--impl reference times the reference's CPU path for tb.matmul on the host
cores: the reference itself cannot be built here (it is an MLIR dialect and
needs an LLVM/MLIR toolchain this image lacks), so its semantics are run
through the C restatement in oracle/ (kind "port") with every host thread.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "GEMM TFLOP/s & % of B200 dense f16 peak at 8192^3 f16->f32"
M = N_PER_GPU = K = 8192
BLOCK = dict(block_m=256, block_n=256, block_k=64, group_m=8, num_warps=4, num_stages=4)
FALLBACK_PEAK_TFLOPS = 1590.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-kshard", action="store_true",
                    help="gemm8192 at N>1: skip the extra K-sharded split-K measurement")
    ap.add_argument("--workload", default="gemm8192", choices=["gemm8192", "splitk", "sweep", "cublas"],
                    help="gemm8192: the headline 8192^3 N-sharded GEMM; splitk: the skinny "
                         "512x512x65536 split-K config (K-sharded + reduce-scatter at N>1)")
    ap.add_argument("--only", default=None, help="sweep: only the configs whose name contains this")
    ap.add_argument("--launches", type=int, default=0,
                    help="sweep: run each selected config this many times and time nothing "
                         "(a fixed launch sequence for a profiler)")
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="gemm8192 at N>1: strong = the fixed 8192^3 problem split along N "
                         "(BASELINE's config); weak = 8192 columns per GPU")
    ap.add_argument("--kshard", default="peer", choices=["peer", "capi", "nccl"],
                    help="splitk at N>1: reduce-scatter fused into the GEMM over NVLink (peer), "
                         "the C ABI's NCCL reduce-scatter run (capi), or torch.distributed's "
                         "reduce-scatter after the GEMM (nccl)")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("bf16_tflops", FALLBACK_PEAK_TFLOPS), d.get("bf16_tflops_sustained"), "measured"
    return FALLBACK_PEAK_TFLOPS, 1400.0, "fallback"


def traffic_for(kernel: str, n: int):
    """DRAM bytes per launch of `kernel` on the M x n x K slice, from the
    committed ncu summary (profiles/traffic.json); None when not captured."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    e = d.get(f"{kernel} {M}x{n}x{K}")
    return None if e is None else e.get("dram_bytes_per_launch")


class ClockSampler:
    """SM clock, power and clock-event reasons of one GPU, polled through
    NVML every ~2 ms while running (so a timed region of a few ms still gets
    samples); nvidia-smi at 200 ms when NVML is unavailable."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ((0x8, "hw_slowdown"), (0x40, "hw_thermal_slowdown"), (0x20, "sw_thermal_slowdown"),
               (0x4, "sw_power_cap"), (0x80, "hw_power_brake_slowdown"))

    def __init__(self, phys_index: int, period_s: float = 0.002):
        self.idx = phys_index
        self.period = period_s
        self.rows = []
        self.proc = None
        self.t = None
        self.stop_flag = threading.Event()
        self.nvml = None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(self.idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            return
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _poll(self):
        nv = self.nvml
        while not self.stop_flag.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                pw = nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.rows.append((time.perf_counter(), sm, pw, rs))
            except Exception:
                pass
            time.sleep(self.period)

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self, window=None):
        """Summary of the samples inside `window` (perf_counter start, end)
        when given, else of all samples."""
        if self.nvml is not None:
            self.stop_flag.set()
            if self.t:
                self.t.join(timeout=2)
            rows = [r for r in self.rows if window is None or window[0] <= r[0] <= window[1]]
            if not rows:
                rows = self.rows[-3:]
            if not rows:
                return None
            reasons = sorted({name for r in rows for bit, name in self.REASONS if r[3] & bit})
            return {"sm_mhz": statistics.median(r[1] for r in rows), "sm_max_mhz": self.max_mhz,
                    "reasons": reasons, "samples": len(rows),
                    "sm_mhz_min": min(r[1] for r in rows), "power_w_max": round(max(r[2] for r in rows), 1),
                    "source": f"NVML every {self.period * 1e3:.0f} ms inside the timed region"}
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)
        if not self.rows:
            return None
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows), "source": "nvidia-smi every 200 ms"}


def phys_gpu_index(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        if local < len(ids) and ids[local].isdigit():
            return int(ids[local])
    return local


_CPU_INPUTS = {}


def cpu_sample(rows: int, threads: int = 0, seed: int = 4):
    """Times the CPU oracle on `rows` rows of the 8192³ problem (same K, N;
    inputs generated once, outside the timing). Returns (seconds, flops)."""
    import numpy as np
    import oracle
    if "B" not in _CPU_INPUTS:
        rng = np.random.default_rng(seed)
        _CPU_INPUTS["B"] = (rng.standard_normal((K, N_PER_GPU), dtype=np.float32) * 0.1).astype(np.float16)
        _CPU_INPUTS["A"] = (rng.standard_normal((M, K), dtype=np.float32) * 0.1).astype(np.float16)
    A = _CPU_INPUTS["A"][:rows]
    B = _CPU_INPUTS["B"]
    C = np.zeros((rows, N_PER_GPU), np.float32)
    t0 = time.perf_counter()
    oracle.matmul_ref(A, B, C, threads=threads)
    return time.perf_counter() - t0, 2.0 * rows * N_PER_GPU * K


def cpu_baseline_block(budget_s: float = 10.0):
    import oracle
    threads = oracle.max_threads()
    dt, fl = cpu_sample(64, threads)
    rate = fl / dt
    rows = int(max(64, min(M, (budget_s * rate) / (2.0 * N_PER_GPU * K))) // 64 * 64)
    dt, fl = cpu_sample(rows, threads)
    return {"value": round(fl / dt / 1e12, 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{rows} of {M} rows of the {M}x{N_PER_GPU}x{K} problem (C_in + A·B, f16->f32), "
                      f"{dt:.1f} s, oracle/tb_oracle.c with {threads} POSIX threads"}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    import oracle
    threads = oracle.max_threads()
    steps, warm = max(1, args.steps), max(0, args.warmup)
    dt, fl = cpu_sample(64, threads)
    per_step_budget = min(10.0, 150.0 / (steps + warm))
    rows = int(max(16, min(M, per_step_budget * (fl / dt) / (2.0 * N_PER_GPU * K))) // 16 * 16)
    for _ in range(warm):
        cpu_sample(rows, threads)
    total_t, total_f = 0.0, 0.0
    for _ in range(steps):
        t, f = cpu_sample(rows, threads)
        total_t += t
        total_f += f
    value = total_f / total_t / 1e12
    sample = (f"{rows} of {M} rows of the {M}x{N_PER_GPU}x{K} tb.matmul per step (reference semantics "
              f"through oracle/tb_oracle.c; the MLIR reference needs an LLVM/MLIR toolchain absent here)")
    n_glob = N_PER_GPU * max(1, args.gpus) if args.scaling == "weak" else N_PER_GPU
    out = {
        "impl": "reference", "metric": METRIC, "value": round(value, 5), "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": steps, "warmup": warm,
        "ms_per_step": round(1e3 * total_t / steps, 3), "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": f"tb.matmul {M}x{n_glob}x{K} f16->f32 C+=A·B, GROUP_M=8",
                   "m": M, "n": n_glob, "k": K, **{k: v for k, v in BLOCK.items()},
                   "rows_per_step": rows,
                   "parallelism": f"host threads ({threads}); each step a {rows}-row sample of the "
                                  f"{M}-row problem (a rate over the same per-row work)"},
        "cpu_baseline": {"value": round(value, 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(out), flush=True)
    return 0


BURST_REGION_S = 0.5  # timed regions shorter than this are compared with the burst peak


def roofline_denominator(region_s: float, peak_burst: float, peak_sustained):
    """(peak, is_burst): the measured cuBLAS burst figure for a timed region
    shorter than BURST_REGION_S (a kernel timed nearly alone, before the
    power cap settles the clock), the sustained figure for longer ones."""
    if region_s < BURST_REGION_S or peak_sustained is None:
        return peak_burst, True
    return peak_sustained, False


def run_ours(args):
    import torch
    import torch.distributed as dist
    import mini_triton_nvgpu_v1_b200 as tb
    from mini_triton_nvgpu_v1_b200 import parallel as par

    rank, world, local = dist_env()
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)

    # The whole problem is M x n_glob x K; rank r owns columns [col0, col0 +
    # ncols) of B and C (tb_matmul_nshard_columns: whole 256-column tiles).
    n_glob = N_PER_GPU * world if args.scaling == "weak" else N_PER_GPU
    cfg = tb.KernelConfig(m=M, n=n_glob, k=K, **BLOCK)
    shard = par.NShard(cfg, rank, world, local)
    col0, ncols = shard.col0, shard.ncols
    g = torch.Generator(device=dev).manual_seed(4)
    A = (torch.randn(M, K, device=dev, generator=g) * 0.1).half()
    # B's column slice, generated in 1024-column blocks of the seeded global B
    B = torch.empty(K, ncols, device=dev, dtype=torch.float16)
    for c in range(0, ncols, 1024):
        g.manual_seed(1000 + (col0 + c) // 1024)
        w = min(1024, ncols - c)
        B[:, c:c + w] = (torch.randn(K, 1024, device=dev, generator=g) * 0.1).half()[:, :w]
    Cm = torch.zeros(M, ncols, device=dev, dtype=torch.float32)
    ws = torch.empty(max(1, shard.workspace_bytes), dtype=torch.uint8, device=dev)
    local_plan = tb.MatmulPlan(tb.KernelConfig(m=M, n=ncols, k=K, **BLOCK), local)
    info = local_plan.info
    launches_per_step = 1 + (1 if info["epilogue"] == "workspace_partial" else 0)

    def step():
        shard.run_ptr(A.data_ptr(), K, B.data_ptr(), ncols, Cm.data_ptr(), ncols, ws.data_ptr(),
                      shard.workspace_bytes, stream.cuda_stream)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(3, args.warmup)):
        step()
    barrier()
    tb.device_status(stream)

    sampler = ClockSampler(phys_gpu_index(local))
    sampler.start()
    time.sleep(0.05)
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_start = time.perf_counter()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    barrier()
    t_end = time.perf_counter()
    clocks = sampler.stop((t_start, t_end))
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    ms_step = ms_max / args.steps
    flops_step = 2.0 * M * n_glob * K          # whole job
    flops_rank = 2.0 * M * ncols * K
    value = flops_step / (ms_step * 1e-3) / 1e12
    tb.device_status(stream)

    # ---- e2e: public API, inputs from pinned host memory, result read back ----
    # Every step copies its A, B and C_in host→device and its C device→host.
    # Steps are pipelined over two device buffer sets: the upload of step i+1
    # (copy stream) and the download of step i (another copy stream, the other
    # PCIe direction) overlap the GEMM of the compute stream.
    hA = A.cpu().pin_memory()
    hB = B.cpu().pin_memory()
    hC = torch.zeros(M, ncols, dtype=torch.float32).pin_memory()
    hOut = [torch.empty(M, ncols, dtype=torch.float32).pin_memory() for _ in range(2)]
    bufs = [(torch.empty_like(A), torch.empty_like(B), torch.empty_like(Cm)) for _ in range(2)]
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event()
    freed = [None, None]

    def e2e_step(i):
        bi = i % 2
        dA, dB, dC = bufs[bi]
        with torch.cuda.stream(up):
            if freed[bi] is not None:
                up.wait_event(freed[bi])          # buffer set bi downloaded (and so computed)
            dA.copy_(hA, non_blocking=True)
            dB.copy_(hB, non_blocking=True)
            dC.copy_(hC, non_blocking=True)
            uploaded = ev()
            uploaded.record(up)
        stream.wait_event(uploaded)
        shard.run(dA, dB, dC, workspace=ws, stream=stream)
        computed = ev()
        computed.record(stream)
        with torch.cuda.stream(down):
            down.wait_event(computed)
            hOut[bi].copy_(dC, non_blocking=True)
            freed[bi] = ev()
            freed[bi].record(down)

    for i in range(2):
        e2e_step(i)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(up)
    for i in range(args.e2e_steps):
        e2e_step(i)
    down.wait_stream(stream)
    down.wait_stream(up)
    e1.record(down)
    barrier()
    te = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = float(te.item()) / args.e2e_steps
    e2e_value = flops_step / (e2e_ms * 1e-3) / 1e12
    # whole-job bytes per step: every rank uploads A, its B and C_in slices
    # and downloads its C slice
    h2d = torch.tensor([A.numel() * 2 + B.numel() * 2 + Cm.numel() * 4], device=dev, dtype=torch.float64)
    d2h = torch.tensor([Cm.numel() * 4], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(h2d)
        dist.all_reduce(d2h)

    # At N > 1 the skinny split-K config runs K-sharded as well, so a scaling
    # run records the fused reduce-scatter (and NCCL's, for comparison).
    kshard = None
    if world > 1 and not args.no_kshard:
        kshard = {}
        for mode in ("peer", "nccl"):
            try:
                r = splitk_measure(mode, 50, 5)
                kshard[mode] = {"workload": r["workload"], "ms_per_step": round(r["ms_per_step"], 5),
                                "tflops": round(r["tflops"], 2), "hbm_frac_per_gpu": round(r["gbs_per_gpu"] / r["hbm"], 4)}
            except Exception as exc:  # report, do not lose the headline line
                kshard[mode] = {"error": f"{type(exc).__name__}: {exc}"[:200]}
    if rank == 0:
        peak, peak_sus, peak_src = peaks()
        achieved = flops_rank / (ms_step * 1e-3) / 1e12  # rank 0's kernel: one launch per step
        region_s = ms_max * 1e-3
        denom, burst = roofline_denominator(region_s, peak, peak_sus)
        kern = info["kernel"]
        cpu = None if args.no_cpu_baseline or world > 1 else cpu_baseline_block()
        alg_bytes = 2 * (M * K + K * ncols) + 8 * M * ncols
        traffic = traffic_for(kern, ncols)
        strong = args.scaling == "strong"
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f16",
            "data": "synthetic",
            "config": {"workload": f"tb.matmul {M}x{n_glob}x{K} f16->f32 C+=A·B, N-sharded "
                                   f"{'into ' + str(world) + ' column slices' if strong else str(N_PER_GPU) + ' columns per GPU'}, GROUP_M=8",
                       "m": M, "n": n_glob, "k": K, "n_per_gpu": ncols, **{k: v for k, v in BLOCK.items()},
                       "kernel": kern, "grid": info["grid"], "stages": info["stages"],
                       "tail_split": info["tail_split"],
                       "l2": "inputs larger than L2 (A alone 128 MiB), no flush",
                       "parallelism": f"N-shard x{world} through tb_matmul_run_nshard, no collective"},
            "pct_of_peak": round(100.0 * achieved / peak, 2),
            "pct_of_peak_note": "rank 0's kernel TFLOP/s over the measured cuBLAS bf16 burst peak per GPU",
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": denom,
                         "unit": "TFLOP/s", "frac": round(achieved / denom, 4),
                         "peak_source": f"{peak_src} cuBLAS bf16 {'burst' if burst else 'sustained'} "
                                        f"(MEASURED_PEAKS.json): the timed region lasted {region_s:.3f} s "
                                        f"({'<' if burst else '>='} {BURST_REGION_S} s)",
                         "timed_region_s": round(region_s, 4),
                         "frac_of_burst": round(achieved / peak, 4),
                         "frac_of_sustained": None if peak_sus is None else round(achieved / peak_sus, 4),
                         "traffic": traffic, "algorithmic_bytes": alg_bytes,
                         "traffic_over_algorithmic": None if traffic is None else round(traffic / alg_bytes, 3)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 3), "unit": "TFLOP/s", "ms_per_step": round(e2e_ms, 3),
                    "h2d_bytes_per_step": int(h2d.item()), "d2h_bytes_per_step": int(d2h.item()),
                    "api": "mini_triton_nvgpu_v1_b200.parallel.NShard.run (tb_matmul_run_nshard)",
                    "note": "whole-job bytes; steps pipelined over two buffer sets: upload, GEMM and "
                            "download overlap"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
        }
        if kshard is not None:
            out["kshard_splitk_512x512x65536"] = kshard
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


SK_M = SK_N = 512
SK_K = 65536
SK_SPLIT = 16
SK_BLOCK = dict(block_m=256, block_n=256, block_k=64, num_warps=4, num_stages=4)


def splitk_measure(mode: str, steps: int, warmup: int):
    """Times 512 x 512 x 65536 split-K on this process's GPU (the process
    group, if any, is already up). mode: "local" (1 GPU, split_k_serial), or
    at N > 1 with K sharded across ranks: "peer" (reduce-scatter fused into
    the GEMM over NVLink, tb_matmul_run_kshard_peer), "capi"
    (tb_matmul_run_kshard_nccl) or "nccl" (torch.distributed reduce-scatter
    after the GEMM). Returns the line's measured fields (max over ranks)."""
    import torch
    import torch.distributed as dist
    import mini_triton_nvgpu_v1_b200 as tb
    from mini_triton_nvgpu_v1_b200 import parallel as par

    rank, world, local = dist_env()
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    k0, kr = par.k_shard(SK_K, world, rank, SK_BLOCK["block_k"])
    g = torch.Generator(device=dev).manual_seed(6)
    A = (torch.rand(SK_M, SK_K, device=dev, generator=g) * 2 - 1).half()[:, k0:k0 + kr].contiguous()
    B = (torch.rand(SK_K, SK_N, device=dev, generator=g) * 2 - 1).half()[k0:k0 + kr].contiguous()
    peer, capi = mode == "peer", mode == "capi"
    split_local = SK_SPLIT if peer else max(1, SK_SPLIT // world)
    cfg = tb.KernelConfig(m=SK_M, n=SK_N, k=kr, split_k=split_local,
                          reduction_mode="split_k_parallel" if peer else "split_k_serial", **SK_BLOCK)
    plan = tb.MatmulPlan(cfg, local)
    ws = torch.empty(max(1, plan.workspace_bytes), dtype=torch.uint8, device=dev)
    r0, mr = par.row_shard(SK_M, world, rank)
    C_rows = torch.zeros(mr, SK_N, device=dev)
    partial = torch.zeros(SK_M, SK_N, device=dev)
    recv = torch.empty_like(C_rows)
    comm = par.PeerKShard(C_rows) if peer else None
    ncomm = par.NcclKShard(C_rows) if capi else None

    def step():
        if mode == "local":
            plan.run_ptr(A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0), C_rows.data_ptr(),
                         SK_N, ws.data_ptr(), ws.numel(), stream.cuda_stream)
        elif peer:
            comm.run(plan, A, B)
        elif capi:
            ncomm.run(plan, A, B)
        else:
            partial.zero_()
            plan.run_ptr(A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0), partial.data_ptr(),
                         SK_N, ws.data_ptr(), ws.numel(), stream.cuda_stream)
            dist.reduce_scatter_tensor(recv, partial, op=dist.ReduceOp.SUM)
            C_rows.add_(recv)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(3, warmup)):
        step()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        step()
    ev1.record(stream)
    barrier()
    t = torch.tensor([ev0.elapsed_time(ev1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = float(t.item()) / steps
    if comm is not None:
        comm.check()
        comm.close()
    if ncomm is not None:
        ncomm.close()
    flops = 2.0 * SK_M * SK_N * SK_K
    bytes_alg = 2.0 * (SK_M * SK_K + SK_K * SK_N) + 8.0 * SK_M * SK_N
    hbm = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()).get("hbm_gbs", 6650.0) \
        if (ROOT / "MEASURED_PEAKS.json").exists() else 6650.0
    gbs = bytes_alg / world / (ms_step * 1e-3) / 1e9
    what = {"local": "1 GPU", "peer": f"K-shard x{world}, reduce-scatter fused into the GEMM over NVLink",
            "capi": f"K-shard x{world}, tb_matmul_run_kshard_nccl",
            "nccl": f"K-shard x{world} + NCCL reduce-scatter"}[mode]
    return {"ms_per_step": ms_step, "tflops": flops / (ms_step * 1e-3) / 1e12, "gbs_per_gpu": gbs, "hbm": hbm,
            "workload": f"tb.matmul {SK_M}x{SK_N}x{SK_K} split_k={SK_SPLIT} ({what})",
            "split_k_per_rank": split_local, "kernel": plan.info["kernel"],
            "launches_per_step": 2 if mode == "local" else 3 if peer else 2}


def run_splitk(args):
    """512 x 512 x 65536 with split_k = 16 (split_k_serial: f32 workspace +
    ordered reduction). At N > 1 the K dimension is sharded across ranks and
    the f32 partials are combined by a reduce-scatter (rank r keeps rows
    [r·512/N, (r+1)·512/N)). Reported against the HBM roofline."""
    import torch
    import torch.distributed as dist
    rank, world, local = dist_env()
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    r = splitk_measure("local" if world == 1 else args.kshard, args.steps, args.warmup)
    if rank == 0:
        print(json.dumps({
            "metric": "GEMM TFLOP/s, 512x512x65536 split-K (HBM-roofline config)",
            "value": round(r["tflops"], 2), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": round(r["ms_per_step"], 5),
            "higher_is_better": True, "scaling": "strong", "dtype": "f16", "data": "synthetic",
            "config": {"workload": r["workload"], "split_k_per_rank": r["split_k_per_rank"],
                       "kernel": r["kernel"]},
            "roofline": {"bound": "hbm", "achieved": round(r["gbs_per_gpu"], 1), "peak": r["hbm"], "unit": "GB/s",
                         "frac": round(r["gbs_per_gpu"] / r["hbm"], 4),
                         "note": "algorithmic bytes per GPU (its A/B K-slice + C_in + C) / step time"},
            "gpu_launches": args.steps * r["launches_per_step"],
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# Every BASELINE config on one GPU: (name, m, n, k, knobs, c dtype, bound).
SWEEP = [
    ("smoke 64x64x32 (tile 64x64x32, 4 warps)", 64, 64, 32,
     dict(block_m=64, block_n=64, block_k=32, num_warps=4), "f32", "latency"),
    ("ragged 96x80x32 (tile 128x128x64, f16 out)", 96, 80, 32,
     dict(block_m=128, block_n=128, block_k=64, exact_tile=False), "f16", "latency"),
    ("ragged scale-up 4096^3 (tile 128x128x64, f16 out)", 4096, 4096, 4096,
     dict(block_m=128, block_n=128, block_k=64), "f16", "tensor"),
    ("grouped 192x128x32 (tile 64x64x32, GROUP_M=8)", 192, 128, 32,
     dict(block_m=64, block_n=64, block_k=32, group_m=8), "f32", "latency"),
    ("grouped 8192^3 (GROUP_M=8, pair 256x256)", 8192, 8192, 8192,
     dict(block_m=256, block_n=256, block_k=64, group_m=8), "f32", "tensor"),
    ("split-K 64x64x64 (split 2)", 64, 64, 64,
     dict(block_m=64, block_n=64, block_k=32, split_k=2, reduction_mode="split_k_serial"), "f32", "latency"),
    ("split-K 512x512x65536 (split 16, serial)", 512, 512, 65536,
     dict(block_m=256, block_n=256, block_k=64, split_k=16, reduction_mode="split_k_serial"), "f32", "hbm"),
    ("split-K 512x512x65536 (split 16, parallel)", 512, 512, 65536,
     dict(block_m=256, block_n=256, block_k=64, split_k=16, reduction_mode="split_k_parallel"), "f32", "hbm"),
    ("persistent 192x128x32 (num_ctas=2)", 192, 128, 32,
     dict(block_m=64, block_n=64, block_k=32, persistent=True, num_ctas=2), "f16", "latency"),
    ("persistent 2048^3 (pair, grid=SMs, f16 out)", 2048, 2048, 2048,
     dict(block_m=256, block_n=256, block_k=64, persistent=True, num_ctas=148), "f16", "tensor"),
    ("persistent 8192^3 (pair, grid=SMs, f16 out)", 8192, 8192, 8192,
     dict(block_m=256, block_n=256, block_k=64, persistent=True, num_ctas=148), "f16", "tensor"),
    ("persistent 16384^3 (pair, grid=SMs, f16 out)", 16384, 16384, 16384,
     dict(block_m=256, block_n=256, block_k=64, persistent=True, num_ctas=148), "f16", "tensor"),
    # one rank's slice of the 8192^3 problem N-sharded over 2 / 4 / 8 GPUs,
    # with the tail split (default) and with whole items (deterministic)
    ("N-shard slice 1/2: 8192x4096x8192", 8192, 4096, 8192,
     dict(block_m=256, block_n=256, block_k=64, group_m=8), "f32", "tensor"),
    ("N-shard slice 1/4: 8192x2048x8192", 8192, 2048, 8192,
     dict(block_m=256, block_n=256, block_k=64, group_m=8), "f32", "tensor"),
    ("N-shard slice 1/4, whole items", 8192, 2048, 8192,
     dict(block_m=256, block_n=256, block_k=64, group_m=8, deterministic=True), "f32", "tensor"),
    ("N-shard slice 1/8: 8192x1024x8192", 8192, 1024, 8192,
     dict(block_m=256, block_n=256, block_k=64, group_m=8), "f32", "tensor"),
    ("N-shard slice 1/8, whole items", 8192, 1024, 8192,
     dict(block_m=256, block_n=256, block_k=64, group_m=8, deterministic=True), "f32", "tensor"),
]


def run_sweep(args):
    """One JSON line per BASELINE config: device time per call (CUDA events,
    ~0.3 s of back-to-back calls after warm-up, best of 3), the distribution
    of 21 calls timed one at a time (median / min / max / spread), the
    CUDA-graph time per call, TFLOP/s and the fraction of the roofline that
    bounds the config."""
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    dev = torch.device("cuda", 0)
    peak_b, peak_s, _ = peaks()
    hbm = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()).get("hbm_gbs", 6650.0) \
        if (ROOT / "MEASURED_PEAKS.json").exists() else 6650.0
    only = getattr(args, "only", None)
    for name, m, n, k, kn, cdt, bound in SWEEP:
        if only and only not in name:
            continue
        g = torch.Generator(device=dev).manual_seed(2)
        A = (torch.rand(m, k, device=dev, generator=g) * 2 - 1).half()
        B = (torch.rand(k, n, device=dev, generator=g) * 2 - 1).half()
        C = torch.zeros(m, n, device=dev, dtype=torch.float16 if cdt == "f16" else torch.float32)
        ws = None
        f = lambda: tb.matmul(A, B, C, workspace=ws, **kn)
        if getattr(args, "launches", 0):
            for _ in range(args.launches):
                f()
            torch.cuda.synchronize()
            tb.device_status()
            print(json.dumps({"workload": "sweep", "config": name, "launches": args.launches}), flush=True)
            del A, B, C
            torch.cuda.empty_cache()
            continue
        for _ in range(5):
            f()
        torch.cuda.synchronize()
        t0 = time.time()
        n_ = 0
        while time.time() - t0 < 0.05:
            f()
            n_ += 1
        torch.cuda.synchronize()
        reps = max(10, int(0.3 / ((time.time() - t0) / n_)))
        best = 1e30
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                f()
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1) / reps)
        # per-call distribution (each call timed alone, stream idle before it):
        # median / min / max / spread, as the reference's bench reports them
        single = []
        for _ in range(21):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            f()
            e1.record()
            torch.cuda.synchronize()
            single.append(e0.elapsed_time(e1) * 1e3)
        single.sort()
        med = single[len(single) // 2]
        per_call = {"median": round(med, 2), "min": round(single[0], 2), "max": round(single[-1], 2),
                    "spread_pct": round(100.0 * (single[-1] - single[0]) / med, 1)}
        tb.device_status()
        # device-only time per call: replay a CUDA graph of back-to-back calls
        graph_us = None
        try:
            if ws is None and kn.get("split_k", 1) > 1 and kn.get("reduction_mode") == "split_k_serial":
                ws = torch.empty(tb.MatmulPlan(tb.KernelConfig(m=m, n=n, k=k, c_dtype=cdt, **{
                    kk: v for kk, v in kn.items()}), 0).workspace_bytes, dtype=torch.uint8, device=dev)
            gr = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                f()
            torch.cuda.current_stream(dev).wait_stream(side)
            n_g = 20
            with torch.cuda.graph(gr):
                for _ in range(n_g):
                    f()
            gr.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            reps_g = max(3, int(reps / n_g))
            e0.record()
            for _ in range(reps_g):
                gr.replay()
            e1.record()
            torch.cuda.synchronize()
            graph_us = round(e0.elapsed_time(e1) / (reps_g * n_g) * 1e3, 2)
            del gr
        except Exception as exc:  # capture unsupported: report the eager number only
            graph_us = f"capture failed: {type(exc).__name__}"
        tb.device_status()
        flops = 2.0 * m * n * k
        cb = 2 if cdt == "f16" else 4
        alg_bytes = 2.0 * (m * k + k * n) + 2 * cb * m * n
        line = {"workload": "sweep", "config": name, "us": round(best * 1e3, 2), "graph_us": graph_us,
                "tflops": round(flops / (best * 1e-3) / 1e12, 2),
                "gbs": round(alg_bytes / (best * 1e-3) / 1e9, 1), "bound": bound,
                "single_call_us": per_call}
        if bound == "tensor":
            line["frac_of_sustained_peak"] = round(line["tflops"] / peak_s, 3)
        elif bound == "hbm":
            line["frac_of_hbm"] = round(line["gbs"] / hbm, 3)
        print(json.dumps(line), flush=True)
        del A, B, C
        torch.cuda.empty_cache()
    return 0


def run_cublas(args):
    """Context only, not the product: cuBLAS (through torch) on the same
    8192³ inputs — f16·f16 → f32 with beta = 0 (torch.mm, out_dtype f32) and
    with C += A·B (aten.addmm.dtype, f32 C) — against this library's run, all
    in one process, over 20 and 300 back-to-back calls."""
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(4)
    A = (torch.randn(M, K, device=dev, generator=g) * 0.1).half()
    B = (torch.randn(K, N_PER_GPU, device=dev, generator=g) * 0.1).half()
    C = torch.zeros(M, N_PER_GPU, device=dev)
    fns = {
        "tb.matmul C += A·B (this library)": lambda: tb.matmul(A, B, C, **BLOCK),
        "cuBLAS torch.mm f16->f32 (beta = 0)": lambda: torch.mm(A, B, out_dtype=torch.float32),
        "cuBLAS aten.addmm.dtype f16->f32, C += A·B": lambda: torch.ops.aten.addmm.dtype(C, A, B, torch.float32),
    }
    for name, f in fns.items():
        for _ in range(10):
            f()
        torch.cuda.synchronize()
        res = {}
        for n in (20, 300):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(n):
                f()
            e1.record()
            torch.cuda.synchronize()
            res[f"tflops_{n}_calls"] = round(2.0 * M * N_PER_GPU * K / (e0.elapsed_time(e1) / n * 1e-3) / 1e12, 1)
        print(json.dumps({"workload": "cublas_context", "impl": name, **res}), flush=True)
        time.sleep(2)
    # f16-output configs of the sweep (C += A·B with f16 C), back-to-back calls
    for (mm, nn, kk, kn) in ((2048, 2048, 2048, dict(block_m=256, block_n=256, block_k=64, persistent=True,
                                                    num_ctas=148)),
                             (4096, 4096, 4096, dict(block_m=128, block_n=128, block_k=64))):
        g.manual_seed(2)
        A = (torch.rand(mm, kk, device=dev, generator=g) * 2 - 1).half()
        B = (torch.rand(kk, nn, device=dev, generator=g) * 2 - 1).half()
        C = torch.zeros(mm, nn, device=dev, dtype=torch.float16)
        for name, f in ((f"tb.matmul {mm}^3 f16 C (this library)", lambda: tb.matmul(A, B, C, **kn)),
                        (f"cuBLAS torch.addmm {mm}^3 f16 C", lambda: torch.addmm(C, A, B))):
            for _ in range(10):
                f()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(100):
                f()
            e1.record()
            torch.cuda.synchronize()
            print(json.dumps({"workload": "cublas_context_f16", "impl": name,
                              "us_per_call": round(e0.elapsed_time(e1) / 100 * 1e3, 2)}), flush=True)
    # the skinny split-K config: time per call with L2 flushed before each
    g.manual_seed(6)
    A = (torch.rand(SK_M, SK_K, device=dev, generator=g) * 2 - 1).half()
    B = (torch.rand(SK_K, SK_N, device=dev, generator=g) * 2 - 1).half()
    C = torch.zeros(SK_M, SK_N, device=dev)
    ws = torch.empty(16 << 20, dtype=torch.uint8, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    fns = {
        "tb.matmul split_k=16 parallel (this library)": lambda: tb.matmul(
            A, B, C, split_k=SK_SPLIT, reduction_mode="split_k_parallel", **SK_BLOCK),
        "tb.matmul split_k=16 serial (this library)": lambda: tb.matmul(
            A, B, C, workspace=ws, split_k=SK_SPLIT, reduction_mode="split_k_serial", **SK_BLOCK),
        "cuBLAS aten.addmm.dtype f16->f32, C += A·B": lambda: torch.ops.aten.addmm.dtype(C, A, B, torch.float32),
        "cuBLAS torch.mm f16->f32 (beta = 0)": lambda: torch.mm(A, B, out_dtype=torch.float32),
    }
    for name, f in fns.items():
        for _ in range(5):
            f()
        ts = []
        for _ in range(30):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            f()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3)
        ts.sort()
        print(json.dumps({"workload": "cublas_context_splitk", "impl": name, "us_median": round(ts[15], 1),
                          "us_min": round(ts[0], 1)}), flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "splitk":
        return run_splitk(args)
    if args.workload == "sweep":
        return run_sweep(args)
    if args.workload == "cublas":
        return run_cublas(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
