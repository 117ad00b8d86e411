"""Parity of the sm_100a tb.matmul kernels (through the C ABI) against the
CPU oracle on seeded inputs. Tolerance: max|C_gpu − C_ref| ≤ 1e-2·sqrt(K/32)
on the f32 result (the north star's bound); f16 output is checked on the
f32 result of the same launch configuration before the downcast, and the f16
output must equal that f32 result rounded to f16 within one f16 ulp."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import make_inputs

pytestmark = pytest.mark.gpu


def _run(cfg_kwargs, A, B, C, cuda, c_dtype="f32"):
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    tA = torch.from_numpy(A).to(cuda)
    tB = torch.from_numpy(B).to(cuda)
    tC = torch.from_numpy(C).to(cuda)
    tb.matmul(tA, tB, tC, **cfg_kwargs)
    torch.cuda.synchronize()
    assert tb.device_status() == 0
    return tC.cpu().numpy()


def _check(out, A, B, C, beta=1):
    import oracle
    ref = oracle.matmul_ref(A, B, C if beta else None, beta=beta)
    err = float(np.abs(out.astype(np.float32) - ref).max())
    tol = oracle.tolerance(A.shape[1])
    assert err <= tol, f"max|Δ|={err} > tol={tol}"
    return ref


CASES = [
    # name, (m, n, k), knobs, dist, seed
    ("smoke_64x64x32", (64, 64, 32), dict(block_m=64, block_n=64, block_k=32, num_warps=4), "uniform", 0),
    ("smoke_1warp", (64, 64, 32), dict(block_m=64, block_n=64, block_k=32, num_warps=1), "uniform", 0),
    ("ragged_96x80x32_t64", (96, 80, 32), dict(block_m=64, block_n=64, block_k=32, num_warps=1,
                                               exact_tile=False), "uniform", 1),
    ("ragged_96x80x32_t128", (96, 80, 32), dict(block_m=128, block_n=128, block_k=64,
                                                exact_tile=False), "uniform", 1),
    ("grouped_192x128x32_g2", (192, 128, 32), dict(block_m=64, block_n=64, block_k=32, group_m=2),
     "normal", 3),
    ("grouped_192x128x32_g8", (192, 128, 32), dict(block_m=64, block_n=64, block_k=32, group_m=8),
     "normal", 3),
    ("splitk_64x64x64_serial", (64, 64, 64), dict(block_m=64, block_n=64, block_k=32, num_warps=1,
                                                  split_k=2, reduction_mode="split_k_serial"),
     "uniform", 5),
    ("splitk_64x64x64_parallel", (64, 64, 64), dict(block_m=64, block_n=64, block_k=32, num_warps=1,
                                                    split_k=2, reduction_mode="split_k_parallel"),
     "uniform", 5),
    ("splitk_empty_parts", (64, 64, 64), dict(block_m=64, block_n=64, block_k=32, split_k=4,
                                              reduction_mode="split_k_serial"), "uniform", 5),
    ("persistent_192x128x32_2ctas", (192, 128, 32), dict(block_m=64, block_n=64, block_k=32,
                                                         persistent=True, num_ctas=2), "uniform", 7),
    ("k_tail_130x136x40", (130, 136, 40), dict(block_m=128, block_n=128, block_k=16,
                                               exact_tile=False), "uniform", 8),
    ("tile128x64_multi_k", (256, 192, 320), dict(block_m=128, block_n=64, block_k=64), "uniform", 9),
    ("tile128x128_grouped", (512, 384, 256), dict(block_m=128, block_n=128, block_k=64, group_m=2),
     "uniform", 10),
    ("tile128x256_grouped", (1024, 1024, 1024), dict(block_m=128, block_n=256, block_k=64, group_m=8),
     "normal", 4),
    ("tile128x256_ragged", (1000, 1000, 520), dict(block_m=128, block_n=256, block_k=64,
                                                   exact_tile=False), "uniform", 11),
    ("persistent_many_tiles", (1024, 1536, 512), dict(block_m=128, block_n=256, block_k=64,
                                                      persistent=True, num_ctas=148), "uniform", 12),
    ("splitk_skinny_512x512x8192_s16", (512, 512, 8192), dict(block_m=128, block_n=256, block_k=64,
                                                              split_k=16,
                                                              reduction_mode="split_k_serial"),
     "uniform", 6),
    ("pair256x256_grouped", (1024, 1024, 1024), dict(block_m=256, block_n=256, block_k=64, group_m=8),
     "normal", 4),
    ("pair256x256_ragged", (1000, 1000, 520), dict(block_m=256, block_n=256, block_k=64,
                                                   exact_tile=False), "uniform", 11),
    ("skinny_parallel_512x512x16384", (512, 512, 16384), dict(block_m=256, block_n=256, block_k=64,
                                                              split_k=16, reduction_mode="split_k_parallel"),
     "uniform", 15),
    ("ragged_parallel_700x300x9000", (700, 300, 9000), dict(block_m=128, block_n=128, block_k=32, split_k=3,
                                                            reduction_mode="split_k_parallel",
                                                            exact_tile=False), "uniform", 16),
    ("fused_2x2_ragged", (2200, 2300, 300), dict(block_m=128, block_n=128, block_k=64, group_m=8,
                                                 exact_tile=False), "uniform", 17),
    ("fused_2x2_exact", (2304, 2304, 256), dict(block_m=128, block_n=128, block_k=64, group_m=4),
     "normal", 18),
    ("fused_horizontal_ragged", (2200, 2300, 300), dict(block_m=256, block_n=128, block_k=64, group_m=8,
                                                        exact_tile=False), "uniform", 19),
    ("fused_horizontal_exact", (2304, 2304, 256), dict(block_m=256, block_n=128, block_k=64, group_m=3),
     "normal", 20),
    ("pair256x512_grouped", (1024, 2048, 1024), dict(block_m=256, block_n=512, block_k=64, group_m=8),
     "normal", 4),
    ("pair256x512_ragged", (1000, 1300, 520), dict(block_m=256, block_n=512, block_k=64,
                                                   exact_tile=False), "uniform", 11),
    ("pair256x384_split_serial", (512, 768, 2048), dict(block_m=128, block_n=384, block_k=64,
                                                        split_k=4, reduction_mode="split_k_serial"),
     "uniform", 13),
    ("pair256x512_persistent", (768, 1536, 256), dict(block_m=256, block_n=512, block_k=64,
                                                      persistent=True, num_ctas=5), "uniform", 14),
    ("pair256x128_ragged_k_tail", (300, 200, 72), dict(block_m=256, block_n=128, block_k=16,
                                                       exact_tile=False), "uniform", 13),
    ("pair_block192x200", (800, 640, 256), dict(block_m=192, block_n=200, block_k=64,
                                                exact_tile=False, group_m=3), "uniform", 14),
    ("pair_persistent", (1536, 1024, 512), dict(block_m=256, block_n=256, block_k=64,
                                                persistent=True, num_ctas=64), "uniform", 15),
    ("pair_splitk_serial", (512, 512, 4096), dict(block_m=256, block_n=256, block_k=64, split_k=8,
                                                  reduction_mode="split_k_serial"), "uniform", 6),
    ("pair_splitk_parallel", (512, 512, 2048), dict(block_m=256, block_n=256, block_k=64, split_k=4,
                                                    reduction_mode="split_k_parallel"), "uniform", 6),
    ("splitk_serial_ragged_tma", (1000, 600, 2048), dict(block_m=128, block_n=256, block_k=64, split_k=5,
                                                         exact_tile=False,
                                                         reduction_mode="split_k_serial"), "uniform", 16),
    ("splitk_parallel_ragged_tma", (1000, 600, 2048), dict(block_m=256, block_n=256, block_k=64,
                                                           split_k=5, exact_tile=False,
                                                           reduction_mode="split_k_parallel"), "uniform", 16),
    ("fused_vertical_ragged", (1000, 600, 256), dict(block_m=128, block_n=128, block_k=64, group_m=4,
                                                     exact_tile=False), "uniform", 17),
    ("fused_horizontal_ragged", (300, 1000, 200), dict(block_m=128, block_n=128, block_k=64, group_m=1,
                                                       exact_tile=False), "uniform", 18),
    ("fused_horizontal_persistent", (512, 1024, 256), dict(block_m=128, block_n=64, block_k=64,
                                                           persistent=True, num_ctas=7), "uniform", 19),
    ("splitk_parallel_512x512x4096_s8", (512, 512, 4096), dict(block_m=128, block_n=128, block_k=64,
                                                               split_k=8,
                                                               reduction_mode="split_k_parallel"),
     "uniform", 6),
]


@pytest.mark.parametrize("name,shape,knobs,dist,seed", CASES, ids=[c[0] for c in CASES])
def test_parity_f32(cuda, name, shape, knobs, dist, seed):
    m, n, k = shape
    A, B, C = make_inputs(m, n, k, seed, dist)
    out = _run(knobs, A, B, C, cuda)
    _check(out, A, B, C)


@pytest.mark.parametrize("name,shape,knobs,dist,seed",
                         [c for c in CASES if c[2].get("reduction_mode") != "split_k_parallel"],
                         ids=[c[0] for c in CASES if c[2].get("reduction_mode") != "split_k_parallel"])
def test_parity_beta0(cuda, name, shape, knobs, dist, seed):
    m, n, k = shape
    A, B, C = make_inputs(m, n, k, seed, dist)
    out = _run(dict(knobs, beta=0), A, B, C, cuda)
    _check(out, A, B, C, beta=0)


F16_CASES = [c for c in CASES if c[2].get("reduction_mode") != "split_k_parallel"]


@pytest.mark.parametrize("name,shape,knobs,dist,seed", F16_CASES, ids=[c[0] for c in F16_CASES])
def test_parity_f16_output(cuda, name, shape, knobs, dist, seed):
    """f16 C: C_in is f16; the f32 result (same knobs, f32 C holding the same
    C_in values) is checked against the oracle first, then the f16 output must
    be that result rounded to f16 (≤ 1 ulp apart: both round the same f32 sum,
    possibly accumulated in a different order)."""
    m, n, k = shape
    A, B, C = make_inputs(m, n, k, seed, dist)
    C16 = C.astype(np.float16)
    C32 = C16.astype(np.float32)
    out32 = _run(knobs, A, B, C32, cuda)
    _check(out32, A, B, C32)
    out16 = _run(knobs, A, B, C16.copy(), cuda, c_dtype="f16")
    assert out16.dtype == np.float16
    want = out32.astype(np.float16)
    ulp = np.abs(np.spacing(want.astype(np.float16))).astype(np.float32)
    diff = np.abs(out16.astype(np.float32) - want.astype(np.float32))
    assert np.all(diff <= ulp + 1e-6), f"max f16 diff {diff.max()}"


def test_repeat_accumulates(cuda):
    """Two launches on the same C accumulate twice (C += A·B each time), as
    the reference's in-place memref update does."""
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    import oracle
    A, B, C = make_inputs(256, 256, 128, 21, "uniform")
    tA, tB, tC = (torch.from_numpy(x).to(cuda) for x in (A, B, C))
    for _ in range(2):
        tb.matmul(tA, tB, tC, block_m=128, block_n=128, block_k=64)
    once = oracle.matmul_ref(A, B, C)
    twice = oracle.matmul_ref(A, B, once)
    assert float(np.abs(tC.cpu().numpy() - twice).max()) <= 2 * oracle.tolerance(128)


def test_strided_operands(cuda):
    """Row strides larger than the row (views into wider buffers)."""
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    import oracle
    A, B, C = make_inputs(200, 160, 96, 22, "uniform")
    bigA = torch.zeros(200, 128, dtype=torch.float16, device=cuda)
    bigB = torch.zeros(96, 200, dtype=torch.float16, device=cuda)
    bigC = torch.zeros(200, 172, dtype=torch.float32, device=cuda)
    bigA[:, :96] = torch.from_numpy(A).to(cuda)
    bigB[:, :160] = torch.from_numpy(B).to(cuda)
    bigC[:, :160] = torch.from_numpy(C).to(cuda)
    tb.matmul(bigA[:, :96], bigB[:, :160], bigC[:, :160], block_m=128, block_n=128, block_k=32,
              exact_tile=False)
    out = bigC.cpu().numpy()
    ref = oracle.matmul_ref(A, B, C)
    assert float(np.abs(out[:, :160] - ref).max()) <= oracle.tolerance(96)
    assert np.all(out[:, 160:] == 0), "wrote outside the C view"
