"""GPU parity of the latency kernel (tb_gemm_small_kernel): every work item
within 128 K elements on a one-CTA tile at most 128 wide. Cases cover the
host-derived work table (at most 64 walk positions) and the device-derived
path (more positions), every mapping kind, ragged edges, f16 output, the
epilogue kinds (store, split_k_serial workspace, split_k_parallel atomics)
and fused expressions. Every element is compared with the CPU oracle."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CASES = [
    ((64, 64, 32), dict(block_m=64, block_n=64, block_k=32)),
    ((96, 80, 32), dict(block_m=128, block_n=128, block_k=64, exact_tile=False)),
    ((192, 128, 32), dict(block_m=64, block_n=64, block_k=32, group_m=2)),
    ((192, 128, 32), dict(block_m=64, block_n=64, block_k=32, persistent=True, num_ctas=2)),
    ((64, 64, 64), dict(block_m=64, block_n=64, block_k=32, split_k=2, reduction_mode="split_k_serial")),
    ((64, 64, 64), dict(block_m=64, block_n=64, block_k=32, split_k=2, reduction_mode="split_k_parallel")),
    ((200, 300, 120), dict(block_m=128, block_n=128, block_k=48, group_m=1, exact_tile=False)),
    ((130, 70, 17), dict(block_m=64, block_n=64, block_k=16, exact_tile=False)),
    ((300, 260, 500), dict(block_m=128, block_n=128, block_k=32, split_k=4, exact_tile=False,
                           reduction_mode="split_k_serial")),
    # more walk positions than the host table holds: derived on the device
    ((2048, 1024, 64), dict(block_m=128, block_n=64, block_k=64, group_m=1)),
    ((1024, 2048, 96), dict(block_m=128, block_n=64, block_k=32, persistent=True, num_ctas=148,
                            exact_tile=False)),
]


def _inputs(cuda, m, n, k, seed):
    import torch
    g = torch.Generator(device=cuda).manual_seed(seed)
    tA = (torch.rand(m, k, device=cuda, generator=g) * 2 - 1).half()
    tB = (torch.rand(k, n, device=cuda, generator=g) * 2 - 1).half()
    tC = torch.randn(m, n, device=cuda, generator=g)
    return tA, tB, tC


@pytest.mark.parametrize("shape,knobs", CASES, ids=[str(i) for i in range(len(CASES))])
@pytest.mark.parametrize("out", ["f32", "f16"])
def test_small_kernel_matches_oracle(cuda, shape, knobs, out):
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    import oracle
    if out == "f16" and knobs.get("reduction_mode") == "split_k_parallel":
        pytest.skip("split_k_parallel needs f32 C")
    m, n, k = shape
    info = tb.MatmulPlan(tb.KernelConfig(m=m, n=n, k=k, c_dtype=out, **knobs), 0).info
    assert info["kernel"].startswith("tb_gemm_sm100_small_"), info["kernel"]
    tA, tB, tCin = _inputs(cuda, m, n, k, 61)
    if out == "f16":
        tCin = tCin.half().float()
    for call in range(2):  # twice: the second call reuses the first call's buffers
        tC = tCin.clone() if out == "f32" else tCin.half()
        tb.matmul(tA, tB, tC, **knobs)
        torch.cuda.synchronize()
        assert tb.device_status() == 0
        ref = oracle.matmul_ref(tA.cpu().numpy(), tB.cpu().numpy(), tCin.cpu().numpy())
        tol = oracle.tolerance(k) + (float(np.abs(ref).max()) * 2 ** -10 if out == "f16" else 0.0)
        assert float(np.abs(tC.float().cpu().numpy() - ref).max()) <= tol, call


def test_small_kernel_beta0_and_exprs(cuda):
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    import oracle
    m, n, k = 160, 96, 64
    tA, tB, _ = _inputs(cuda, m, n, k, 62)
    bias = torch.randn(n, device=cuda)
    tC = torch.full((m, n), float("nan"), device=cuda)
    tb.matmul(tA, tB, tC, beta=0, bias=bias, activation="gelu_tanh", clamp=(-1.0, 2.0),
              block_m=128, block_n=128, block_k=64, exact_tile=False)
    ref = oracle.apply_epilogue(oracle.matmul_ref(tA.cpu().numpy(), tB.cpu().numpy()),
                                bias.cpu().numpy(), "gelu_tanh", (-1.0, 2.0))
    assert float(np.abs(tC.cpu().numpy() - ref).max()) <= oracle.tolerance(k) * 1.15 + 1e-5
