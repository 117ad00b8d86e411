"""Fused epilogue expressions (bias, activation, clamp, convert): plan rules
on CPU, parity against the oracle with the expressions applied in float64 on
the GPU. Tolerance: 1e-2·sqrt(K/32) on the f32 result before the expressions
(every expression is 1-Lipschitz up to small factors: relu/clamp/bias exactly,
silu ≤ 1.1, gelu_tanh ≤ 1.13), plus 1e-5 for their own f32 evaluation."""
from __future__ import annotations

import numpy as np
import pytest

import mini_triton_nvgpu_v1_b200 as tb
from conftest import make_inputs


def test_plan_describes_exprs_in_reference_spelling():
    p = tb.MatmulPlan(tb.KernelConfig(m=256, n=256, k=64, block_m=128, block_n=128, block_k=64,
                                      bias=True, activation="relu", clamp=(-1.0, 1.0), c_dtype="f16"))
    assert p.info["epilogue_exprs"] == ["add(c_in)", "load_bias", "add", "activation(relu)", "clamp",
                                        "convert(f16)"]


def test_plan_rules():
    with pytest.raises(tb.TBError, match="use split_k_serial"):
        tb.MatmulPlan(tb.KernelConfig(m=256, n=256, k=1024, block_m=128, block_n=128, block_k=64,
                                      split_k=4, reduction_mode="split_k_parallel", activation="relu"))
    with pytest.raises(tb.TBError, match="clamp_lo <= clamp_hi"):
        tb.MatmulPlan(tb.KernelConfig(m=64, n=64, k=64, block_m=64, block_n=64, block_k=64, clamp=(1, 0)))
    with pytest.raises(tb.TBError, match="unknown epilogue activation"):
        tb.MatmulPlan(tb.KernelConfig(m=64, n=64, k=64, block_m=64, block_n=64, block_k=64,
                                      activation="tanh"))
    tb.MatmulPlan(tb.KernelConfig(m=256, n=256, k=1024, block_m=128, block_n=128, block_k=64,
                                  split_k=4, reduction_mode="split_k_serial", activation="silu"))


CASES = [
    ((512, 512, 256), dict(block_m=256, block_n=256, block_k=64), dict(bias=True, activation="relu")),
    ((500, 296, 200), dict(block_m=128, block_n=128, block_k=64, exact_tile=False),
     dict(bias=True, activation="gelu_tanh", clamp=(-0.5, 2.0))),
    ((256, 384, 512), dict(block_m=128, block_n=256, block_k=64), dict(activation="silu")),
    ((512, 512, 2048), dict(block_m=256, block_n=256, block_k=64, split_k=4,
                            reduction_mode="split_k_serial"), dict(bias=True, clamp=(-3.0, 3.0))),
    ((96, 80, 32), dict(block_m=64, block_n=64, block_k=32, exact_tile=False),
     dict(bias=True, activation="relu")),
]


@pytest.mark.gpu
@pytest.mark.parametrize("shape,knobs,ex", CASES, ids=[str(i) for i in range(len(CASES))])
@pytest.mark.parametrize("out", ["f32", "f16"])
def test_fused_exprs_match_oracle(cuda, shape, knobs, ex, out):
    import torch
    import oracle
    m, n, k = shape
    A, B, Cin = make_inputs(m, n, k, 51, "uniform")
    if out == "f16":
        Cin = Cin.astype(np.float16).astype(np.float32)
    rng = np.random.default_rng(52)
    bias = rng.standard_normal(n).astype(np.float32) if ex.get("bias") else None
    tC = torch.from_numpy(Cin.astype(np.float16) if out == "f16" else Cin).to(cuda)
    tb.matmul(torch.from_numpy(A).to(cuda), torch.from_numpy(B).to(cuda), tC,
              bias=None if bias is None else torch.from_numpy(bias).to(cuda),
              activation=ex.get("activation"), clamp=ex.get("clamp"), **knobs)
    want = oracle.apply_epilogue(oracle.matmul_ref(A, B, Cin), bias, ex.get("activation"), ex.get("clamp"))
    got = tC.float().cpu().numpy()
    tol = oracle.tolerance(k) * 1.15 + 1e-5
    if out == "f16":
        tol += float(np.abs(np.spacing(want.astype(np.float16))).max())
    assert float(np.abs(got - want).max()) <= tol


@pytest.mark.gpu
def test_bias_must_match_the_plan(cuda):
    import torch
    A = torch.zeros(64, 64, dtype=torch.float16, device=cuda)
    C = torch.zeros(64, 64, device=cuda)
    p = tb.MatmulPlan(tb.KernelConfig(m=64, n=64, k=64, block_m=64, block_n=64, block_k=64, bias=True), 0)
    with pytest.raises(tb.TBError, match="tb_matmul_run_epilogue"):
        p.run_ptr(A.data_ptr(), 64, A.data_ptr(), 64, C.data_ptr(), 64)
