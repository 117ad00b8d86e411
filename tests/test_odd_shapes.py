"""Shapes whose rows are not a multiple of 8 elements (the reference accepts
any static shape; TMA needs 16-byte row strides): the plan reserves
workspace for a zero-padded copy of such an operand and the run repacks it."""
from __future__ import annotations

import numpy as np
import pytest

import mini_triton_nvgpu_v1_b200 as tb
from conftest import make_inputs


def _plan(m, n, k, **kw):
    kw.setdefault("exact_tile", m % kw["block_m"] == 0 and n % kw["block_n"] == 0 and k % kw["block_k"] == 0)
    return tb.MatmulPlan(tb.KernelConfig(m=m, n=n, k=k, **kw))


def test_packing_space_in_the_workspace():
    t = dict(block_m=64, block_n=64, block_k=16)
    assert _plan(64, 64, 32, **t).workspace_bytes == 0
    assert _plan(100, 64, 36, **t).workspace_bytes == 100 * 40 * 2            # A: 36 -> 40
    assert _plan(64, 90, 32, **t).workspace_bytes == 32 * 96 * 2              # B: 90 -> 96
    p = _plan(100, 90, 36, **t)                                              # both, 256-aligned parts
    assert p.workspace_bytes == ((100 * 40 * 2 + 255) // 256) * 256 + 36 * 96 * 2
    sk = _plan(128, 90, 1000, split_k=4, reduction_mode="split_k_serial", **t)
    part = 4 * 128 * 90 * 4
    assert sk.workspace_bytes == ((part + 255) // 256) * 256 + 1000 * 96 * 2
    # column-major A packs along m
    assert _plan(37, 64, 32, a_col_major=True, **t).workspace_bytes == 32 * 40 * 2


CASES = [
    ((100, 90, 36), dict(block_m=64, block_n=64, block_k=16), "rr"),
    ((33, 17, 9), dict(block_m=128, block_n=64, block_k=16), "rr"),
    ((300, 250, 1000), dict(block_m=256, block_n=256, block_k=64, split_k=4,
                            reduction_mode="split_k_serial"), "rr"),
    ((37, 45, 50), dict(block_m=128, block_n=128, block_k=32), "cc"),
    ((130, 70, 99), dict(block_m=128, block_n=128, block_k=32), "cr"),
]


@pytest.mark.gpu
@pytest.mark.parametrize("shape,knobs,layout", CASES, ids=[f"{c[0]}{c[2]}" for c in CASES])
def test_odd_shapes_match_oracle(cuda, shape, knobs, layout):
    import torch
    import oracle
    m, n, k = shape
    A, B, Cin = make_inputs(m, n, k, 71, "uniform")
    tA = torch.from_numpy(np.ascontiguousarray(A.T)).to(cuda).t() if layout[0] == "c" else torch.from_numpy(A).to(cuda)
    tB = torch.from_numpy(np.ascontiguousarray(B.T)).to(cuda).t() if layout[1] == "c" else torch.from_numpy(B).to(cuda)
    tC = torch.from_numpy(Cin).to(cuda)
    tb.matmul(tA, tB, tC, exact_tile=False, **knobs)
    err = float(np.abs(tC.cpu().numpy() - oracle.matmul_ref(A, B, Cin)).max())
    assert err <= oracle.tolerance(k), err


@pytest.mark.gpu
def test_misaligned_base_pointer_is_repacked(cuda):
    """An A view starting 1 element into its buffer (2-byte aligned) on an
    odd-K plan is repacked; on an aligned-shape plan it is rejected."""
    import torch
    import oracle
    m, n, k = 64, 64, 36
    A, B, Cin = make_inputs(m, n, k, 72, "uniform")
    buf = torch.zeros(m * k + 1, dtype=torch.float16, device=cuda)
    buf[1:] = torch.from_numpy(A.reshape(-1)).to(cuda)
    tA = buf[1:].view(m, k)
    tC = torch.from_numpy(Cin).to(cuda)
    tb.matmul(tA, torch.from_numpy(B).to(cuda), tC, block_m=64, block_n=64, block_k=16, exact_tile=False)
    assert float(np.abs(tC.cpu().numpy() - oracle.matmul_ref(A, B, Cin)).max()) <= oracle.tolerance(k)
    buf2 = torch.zeros(64 * 32 + 1, dtype=torch.float16, device=cuda)
    with pytest.raises(tb.TBError, match="reserve workspace"):
        tb.matmul(buf2[1:].view(64, 32), torch.zeros(32, 64, dtype=torch.float16, device=cuda),
                  torch.zeros(64, 64, device=cuda), block_m=64, block_n=64, block_k=32)
