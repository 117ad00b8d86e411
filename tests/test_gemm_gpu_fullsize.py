"""GPU parity at the BASELINE configs' full sizes and against the golden
vectors of the reference's own statement of tb.matmul.

Full sizes (8192³, 4096³ f16 out, 16384³, 512×512×65536 split-K, persistent
2048/8192/16384³ f16 out) are compared element by element with the CPU
oracle running on every host thread (seconds per config; ~30 s for 16384³),
tolerance 1e-2·sqrt(K/32). Size-independent properties are checked on top:
  * exact scaling: C(A, 2·B) − C_in == 2·(C(A, B) − C_in) bit for bit on
    beta = 0 results (powers of two scale every product and partial sum
    exactly in f16/f32 barring overflow);
  * checksum: Σ_rows C = (1ᵀ·A)·B + Σ_rows C_in, computed in float64.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest


pytestmark = pytest.mark.gpu

GOLDEN = sorted((Path(__file__).parent / "golden").glob("golden_*.npz"))


def _knobs_for(name, meta):
    bm, bn, bk = meta["block"]
    kn = dict(block_m=bm, block_n=bn, block_k=bk, group_m=meta["group_m"],
              exact_tile=meta["exact_tile"])
    if name.startswith("golden_splitk"):
        kn.update(split_k=2, reduction_mode="split_k_parallel")
    if name.startswith("golden_persistent"):
        kn.update(persistent=True, num_ctas=2)
    return kn


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
@pytest.mark.parametrize("variant", ["as_reference", "serial_splitk", "pair_tile"])
def test_kernel_matches_reference_golden(cuda, path, variant):
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    import oracle
    g = np.load(path)
    meta = json.loads(str(g["meta"]))
    kn = _knobs_for(path.stem, meta)
    if variant == "serial_splitk":
        kn = dict(kn, split_k=max(2, kn.get("split_k", 1)), reduction_mode="split_k_serial",
                  persistent=False, num_ctas=1)
    elif variant == "pair_tile":
        kn = dict(kn, block_m=256, block_n=256, exact_tile=False, split_k=1, reduction_mode=None)
    tC = torch.from_numpy(g["C_in"].copy()).to(cuda)
    tb.matmul(torch.from_numpy(g["A"]).to(cuda), torch.from_numpy(g["B"]).to(cuda), tC, **kn)
    out = tC.cpu().numpy()
    err = float(np.abs(out - g["C_out"]).max())
    assert err <= oracle.tolerance(meta["k"]), (kn, err)


def _inputs(cuda, m, n, k, seed, dist):
    """Seeded f16 A, B and f32 C_in, generated on the GPU (U[-1,1] or
    N(0,1)·0.1, as the BASELINE configs state) and copied to the host."""
    import torch
    g = torch.Generator(device=cuda).manual_seed(seed)
    if dist == "uniform":
        tA = (torch.rand(m, k, device=cuda, generator=g) * 2 - 1).half()
        tB = (torch.rand(k, n, device=cuda, generator=g) * 2 - 1).half()
    else:
        tA = (torch.randn(m, k, device=cuda, generator=g) * 0.1).half()
        tB = (torch.randn(k, n, device=cuda, generator=g) * 0.1).half()
    tCin = torch.randn(m, n, device=cuda, generator=g)
    return tA, tB, tCin


def _all_elements_check(tA, tB, tCin, tOut, k):
    """Every element of the GPU result against the CPU oracle (all host
    threads), max|Δ| ≤ 1e-2·sqrt(K/32)."""
    import oracle
    ref = oracle.matmul_ref(tA.cpu().numpy(), tB.cpu().numpy(), tCin.cpu().numpy())
    err = float(np.abs(tOut.cpu().numpy() - ref).max())
    assert err <= oracle.tolerance(k), err
    return ref


def _f16_is_rounded_f32(tC16, tC32):
    """f16 output = the f32 result of the same knobs and summation order
    rounded to f16, within 1 ulp."""
    import torch
    want = tC32.half().float()
    diff = (tC16.float() - want).abs()
    ulp = torch.from_numpy(np.spacing(want.cpu().numpy().astype(np.float16)).astype(np.float32)).to(
        tC16.device).abs()
    assert bool((diff <= ulp + 1e-6).all())


FULL = [
    dict(shape=(8192, 8192, 8192), knobs=dict(block_m=256, block_n=256, block_k=64, group_m=8),
         dist="normal", seed=4, out="f32"),
    dict(shape=(4096, 4096, 4096), knobs=dict(block_m=128, block_n=128, block_k=64, group_m=8),
         dist="uniform", seed=2, out="f16"),
    dict(shape=(512, 512, 65536), knobs=dict(block_m=128, block_n=256, block_k=64, split_k=16,
                                             reduction_mode="split_k_serial"),
         dist="uniform", seed=6, out="f32"),
    dict(shape=(512, 512, 65536), knobs=dict(block_m=256, block_n=256, block_k=64, split_k=16,
                                             reduction_mode="split_k_serial"),
         dist="uniform", seed=6, out="f32"),
    dict(shape=(512, 512, 65536), knobs=dict(block_m=256, block_n=256, block_k=64, split_k=16,
                                             reduction_mode="split_k_parallel"),
         dist="uniform", seed=6, out="f32"),
    dict(shape=(2048, 2048, 2048), knobs=dict(block_m=256, block_n=256, block_k=64, persistent=True,
                                              num_ctas=148), dist="uniform", seed=7, out="f16"),
    dict(shape=(8192, 8192, 8192), knobs=dict(block_m=256, block_n=256, block_k=64, persistent=True,
                                              num_ctas=148), dist="uniform", seed=9, out="f16"),
    # one rank's slice of the 8-way N-sharded 8192^3 problem: 128 pair work
    # items on 74 CTA pairs (whole items: no whole wave before a tail)
    dict(shape=(8192, 1024, 8192), knobs=dict(block_m=256, block_n=256, block_k=64, group_m=8),
         dist="normal", seed=10, out="f32"),
    # a 4-way slice: two whole waves, then 108 items spread stream-K
    dict(shape=(8192, 2048, 8192), knobs=dict(block_m=256, block_n=256, block_k=64, group_m=8),
         dist="normal", seed=11, out="f32"),
]


@pytest.mark.parametrize("cfg", FULL, ids=["grouped_8192", "ragged_scaleup_4096_f16", "splitk_serial_skinny",
                                          "splitk_serial_skinny_pair", "splitk_parallel_skinny_pair",
                                          "persistent_2048_f16", "persistent_8192_f16", "nshard8_slice",
                                          "nshard4_slice_tail"])
def test_fullsize_every_element(cuda, cfg):
    """Every element of each full-size BASELINE config against the CPU
    oracle; f16-output configs are checked on their f32 result (same knobs)
    and the f16 result must equal it rounded to f16; the column checksum
    Σ_rows C = (1ᵀ·A)·B + Σ_rows C_in (float64) is checked on top."""
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    import oracle
    m, n, k = cfg["shape"]
    tA, tB, tCin = _inputs(cuda, m, n, k, cfg["seed"], cfg["dist"])
    if cfg["out"] == "f16":
        tCin = tCin.half().float()
    tC = tCin.clone()
    tb.matmul(tA, tB, tC, **cfg["knobs"])
    torch.cuda.synchronize()
    assert tb.device_status() == 0
    _all_elements_check(tA, tB, tCin, tC, k)
    colsum_ref = (tA.double().sum(0) @ tB.double()) + tCin.double().sum(0)
    assert float((tC.double().sum(0) - colsum_ref).abs().max()) <= oracle.tolerance(k) * m ** 0.5 * 4
    if cfg["out"] == "f16":
        # f16 plans keep every work item whole (no reduce-added K pieces):
        # compare with the f32 result of the same summation order
        tC32 = tCin.clone()
        tb.matmul(tA, tB, tC32, deterministic=True, **cfg["knobs"])
        tC16 = tCin.half()
        tb.matmul(tA, tB, tC16, **cfg["knobs"])
        _f16_is_rounded_f32(tC16, tC32)


def test_fullsize_16384_persistent_every_element(cuda):
    """16384³ persistent pair-tile GEMM (the largest config of the persistent
    sweep): every element of the f32 result against the oracle, and the f16
    output (the BASELINE's persistent config) equal to it rounded."""
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    m = n = k = 16384
    knobs = dict(block_m=256, block_n=256, block_k=64, persistent=True, num_ctas=148)
    tA, tB, tCin = _inputs(cuda, m, n, k, 8, "uniform")
    tCin = tCin.half().float()
    tC = tCin.clone()
    tb.matmul(tA, tB, tC, **knobs)
    torch.cuda.synchronize()
    assert tb.device_status() == 0
    _all_elements_check(tA, tB, tCin, tC, k)
    tC16 = tCin.half()
    del tCin
    tb.matmul(tA, tB, tC16, **knobs)
    _f16_is_rounded_f32(tC16, tC)  # 16384^3 on 148 pairs: 4096 items, no tail split


@pytest.mark.parametrize("knobs", [dict(block_m=256, block_n=256, block_k=64, group_m=8),
                                   dict(block_m=128, block_n=256, block_k=64, split_k=8,
                                        reduction_mode="split_k_serial")])
def test_power_of_two_scaling_is_exact(cuda, knobs):
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    m = n = 2048
    k = 4096
    g = torch.Generator(device=cuda).manual_seed(11)
    tA = (torch.rand(m, k, device=cuda, generator=g) * 2 - 1).half()
    tB = (torch.rand(k, n, device=cuda, generator=g) * 2 - 1).half()
    c1 = torch.zeros(m, n, device=cuda)
    c2 = torch.zeros(m, n, device=cuda)
    tb.matmul(tA, tB, c1, beta=0, **knobs)
    tb.matmul(tA, tB * 2, c2, beta=0, **knobs)
    assert torch.equal(c2, c1 * 2)


def test_deterministic_serial_split_k(cuda):
    """split_k_serial reduces partials in a fixed order: repeated runs are
    bitwise identical."""
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    g = torch.Generator(device=cuda).manual_seed(12)
    tA = (torch.rand(512, 16384, device=cuda, generator=g) * 2 - 1).half()
    tB = (torch.rand(16384, 512, device=cuda, generator=g) * 2 - 1).half()
    outs = []
    for _ in range(3):
        c = torch.zeros(512, 512, device=cuda)
        tb.matmul(tA, tB, c, block_m=128, block_n=128, block_k=64, split_k=16,
                  reduction_mode="split_k_serial")
        outs.append(c)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])


@pytest.mark.parametrize("col_major_a", [False, True])
def test_operands_past_4_gib(cuda, col_major_a):
    """An A of 2^31 f16 elements (4 GiB): rows far past the 32-bit byte range
    (TMA coordinates and epilogue row offsets in 64-bit arithmetic), in both
    A layouts, checked on sampled rows including the last ones."""
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    import oracle
    m, n, k = 131072, 256, 16384
    g = torch.Generator(device=cuda).manual_seed(21)
    if col_major_a:
        tA = ((torch.rand(k, m, device=cuda, generator=g) * 2 - 1).half()).t()   # m × k, unit row stride
    else:
        tA = (torch.rand(m, k, device=cuda, generator=g) * 2 - 1).half()
    tB = (torch.rand(k, n, device=cuda, generator=g) * 2 - 1).half()
    tC = torch.randn(m, n, device=cuda, generator=g)
    C0 = tC.clone()
    tb.matmul(tA, tB, tC, block_m=256, block_n=256, block_k=64)
    torch.cuda.synchronize()
    assert tb.device_status() == 0
    rows = np.array([0, 1, 8191, 65535, 65536, 100000, 131071 - 255, 131070, 131071])
    ridx = torch.from_numpy(rows).to(cuda)
    A_rows = tA[ridx].contiguous().cpu().numpy()
    ref = oracle.matmul_ref(A_rows, tB.cpu().numpy(), C0[ridx].cpu().numpy())
    err = float(np.abs(tC[ridx].cpu().numpy() - ref).max())
    assert err <= oracle.tolerance(k), err
