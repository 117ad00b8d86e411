"""GPU parity for the work decompositions that do not change a program's
result: program tiles larger than every hardware tile (run as sub-tiles),
the stream-K tail (the last work items' K fills spread evenly over the
slots, partial items reduce-added into C), and the N-shard entry point run rank by rank on one GPU. Every
element is compared with the CPU oracle, tolerance 1e-2·sqrt(K/32)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _inputs(cuda, m, n, k, seed):
    import torch
    g = torch.Generator(device=cuda).manual_seed(seed)
    tA = (torch.rand(m, k, device=cuda, generator=g) * 2 - 1).half()
    tB = (torch.rand(k, n, device=cuda, generator=g) * 2 - 1).half()
    tC = torch.randn(m, n, device=cuda, generator=g)
    return tA, tB, tC


def _oracle(tA, tB, tCin, beta=1):
    import oracle
    return oracle.matmul_ref(tA.cpu().numpy(), tB.cpu().numpy(), tCin.cpu().numpy(), beta=beta)


@pytest.mark.parametrize("shape,knobs,sub", [
    ((1024, 512, 256), dict(block_m=512, block_n=256, block_k=64), [2, 1]),
    ((512, 2048, 320), dict(block_m=256, block_n=1024, block_k=64), [1, 4]),
    ((1040, 384, 192), dict(block_m=512, block_n=128, block_k=32, exact_tile=False), [2, 1]),
    ((700, 1300, 200), dict(block_m=128, block_n=640, block_k=32, exact_tile=False), [1, 3]),
    ((800, 800, 256), dict(block_m=384, block_n=384, block_k=64, exact_tile=False), [2, 1]),
    ((600, 200, 128), dict(block_m=272, block_n=64, block_k=64, exact_tile=False), [2, 1]),
    ((1024, 1024, 512), dict(block_m=512, block_n=512, block_k=64, persistent=True, num_ctas=3), [2, 1]),
    ((1024, 512, 2048), dict(block_m=512, block_n=256, block_k=64, split_k=3,
                             reduction_mode="split_k_serial"), [2, 1]),
    ((1024, 512, 2048), dict(block_m=512, block_n=256, block_k=64, split_k=2,
                             reduction_mode="split_k_parallel"), [2, 1]),
], ids=["512x256", "256x1024", "512x128_ragged", "128x640_ragged", "384x384_ragged", "272x64_ragged",
        "512x512_persistent", "512x256_splitk_serial", "512x256_splitk_parallel"])
@pytest.mark.parametrize("out", ["f32", "f16"])
def test_large_program_tiles(cuda, shape, knobs, sub, out):
    """KernelConfig.cpp:217-221 allows any block_m % 16 / block_n % 8: a
    program larger than the hardware tile computes its tile as sub-tiles."""
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    import oracle
    if out == "f16" and knobs.get("reduction_mode") == "split_k_parallel":
        pytest.skip("split_k_parallel needs f32 C")
    m, n, k = shape
    cfg = tb.KernelConfig(m=m, n=n, k=k, c_dtype=out, **knobs)
    assert tb.MatmulPlan(cfg, 0).info["program_subtiles"] == sub
    tA, tB, tCin = _inputs(cuda, m, n, k, 41)
    if out == "f16":
        tCin = tCin.half().float()
    tC = tCin.clone() if out == "f32" else tCin.half()
    tb.matmul(tA, tB, tC, **knobs)
    torch.cuda.synchronize()
    assert tb.device_status() == 0
    ref = _oracle(tA, tB, tCin)
    got = tC.float().cpu().numpy()
    tol = oracle.tolerance(k) + (float(np.abs(ref).max()) * 2 ** -10 if out == "f16" else 0.0)
    assert float(np.abs(got - ref).max()) <= tol


@pytest.mark.parametrize("shape,tile", [((4096, 2560, 8192), (256, 256)), ((2304, 4352, 8192), (256, 256)),
                                        ((4096, 2560, 8192), (128, 128)), ((2560, 4096, 8192), (256, 128))],
                         ids=["pair", "pair_ragged_m", "fused_128", "fused_256x128"])
@pytest.mark.parametrize("persistent", [False, True])
def test_tail_split_matches_oracle_and_whole_items(cuda, shape, tile, persistent):
    """Plans whose last wave is partly idle spread the tail items' K fills
    evenly over the slots (stream-K; partial items reduce-added into C); the
    result matches the oracle and the deterministic (whole item) run within
    tolerance, and the deterministic run repeats bitwise."""
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    import oracle
    m, n, k = shape
    knobs = dict(block_m=tile[0], block_n=tile[1], block_k=64, exact_tile=False)
    if persistent:
        knobs.update(persistent=True, num_ctas=148)
    info = tb.MatmulPlan(tb.KernelConfig(m=m, n=n, k=k, **knobs), 0).info
    assert info["tail_split"] is not None, info
    tA, tB, tCin = _inputs(cuda, m, n, k, 43)
    tC = tCin.clone()
    tb.matmul(tA, tB, tC, **knobs)
    torch.cuda.synchronize()
    assert tb.device_status() == 0
    ref = _oracle(tA, tB, tCin)
    tol = oracle.tolerance(k)
    assert float(np.abs(tC.cpu().numpy() - ref).max()) <= tol
    det = [tCin.clone(), tCin.clone()]
    for d in det:
        tb.matmul(tA, tB, d, deterministic=True, **knobs)
    assert torch.equal(det[0], det[1])
    assert float((det[0] - tC).abs().max()) <= tol
    # beta = 0 keeps whole items (pieces add into C's prior value)
    z = torch.full_like(tCin, float("nan"))
    tb.matmul(tA, tB, z, beta=0, **knobs)
    assert float(np.abs(z.cpu().numpy() - (ref - tCin.cpu().numpy())).max()) <= tol * 2


def test_tail_split_falls_back_when_c_is_not_tma_addressable(cuda):
    """A C view whose row stride is not a multiple of 16 bytes has no TMA
    map: the same plan runs every item whole (direct stores)."""
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    import oracle
    m, n, k = 4096, 2560, 8192
    tA, tB, _ = _inputs(cuda, m, n, k, 44)
    big = torch.randn(m, n + 1, device=cuda)
    tC = big[:, :n]
    C0 = tC.clone()
    tb.matmul(tA, tB, tC, block_m=256, block_n=256, block_k=64)
    torch.cuda.synchronize()
    ref = _oracle(tA, tB, C0)
    assert float(np.abs(tC.cpu().numpy() - ref).max()) <= oracle.tolerance(k)


@pytest.mark.parametrize("world", [1, 3, 8])
@pytest.mark.parametrize("slices", ["own", "views"])
def test_nshard_entry_rank_by_rank(cuda, world, slices):
    """tb_matmul_run_nshard through the C ABI: every rank's slice run in turn
    on one GPU, either from rank-owned slice buffers or from column views of
    the full matrices; the assembled C equals the oracle's."""
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    import oracle
    from mini_triton_nvgpu_v1_b200 import parallel as par
    m, n, k = 1024, 2304, 1024
    tA, tB, tCin = _inputs(cuda, m, n, k, 45)
    cfg = tb.KernelConfig(m=m, n=n, k=k, block_m=256, block_n=256, block_k=64)
    full = tCin.clone()
    for r in range(world):
        sh = par.NShard(cfg, r, world, 0)
        c0, nc = sh.col0, sh.ncols
        if nc == 0:
            continue
        if slices == "own":
            b = tB[:, c0:c0 + nc].clone()
            c = tCin[:, c0:c0 + nc].clone()
            sh.run(tA, b, c)
            full[:, c0:c0 + nc] = c
        else:
            sh.run(tA, tB[:, c0:c0 + nc], full[:, c0:c0 + nc])
    torch.cuda.synchronize()
    ref = _oracle(tA, tB, tCin)
    assert float(np.abs(full.cpu().numpy() - ref).max()) <= oracle.tolerance(k)
