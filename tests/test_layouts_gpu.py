"""Transposed operand storage (column-major A and/or B, read directly by
TMA/UMMA as MN-major A / K-major B) against the CPU oracle, across the tile
families, ragged edges, padded leading dimensions and split-K."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import make_inputs

pytestmark = pytest.mark.gpu

KNOBS = [
    ((256, 192, 320), dict(block_m=128, block_n=64, block_k=64)),
    ((512, 384, 256), dict(block_m=128, block_n=128, block_k=64, group_m=2)),
    ((1024, 1024, 512), dict(block_m=128, block_n=256, block_k=64)),
    # one-CTA 128 × 256 hardware tile (group of 3 rows: no pairing)
    ((640, 360, 512), dict(block_m=128, block_n=256, block_k=64, group_m=3, exact_tile=False)),
    ((1024, 1024, 512), dict(block_m=256, block_n=256, block_k=64, group_m=8)),
    ((1000, 744, 520), dict(block_m=256, block_n=128, block_k=64, exact_tile=False)),
    ((96, 80, 40), dict(block_m=64, block_n=64, block_k=16, exact_tile=False)),
    ((512, 512, 4096), dict(block_m=256, block_n=256, block_k=64, split_k=8,
                            reduction_mode="split_k_serial")),
    ((1000, 1200, 520), dict(block_m=256, block_n=512, block_k=64, exact_tile=False)),
]


def _col_major(x: np.ndarray, pad: int, dev):
    """x as a column-major CUDA view (unit row stride), leading dim rows+pad."""
    import torch
    rows, cols = x.shape
    buf = torch.zeros(cols, rows + pad, dtype=torch.float16, device=dev)
    buf[:, :rows] = torch.from_numpy(np.ascontiguousarray(x.T)).to(dev)
    return buf[:, :rows].t()


@pytest.mark.parametrize("a_col,b_col", [(False, False), (True, False), (False, True), (True, True)],
                         ids=["rr", "cr", "rc", "cc"])
@pytest.mark.parametrize("shape,knobs", KNOBS, ids=[f"{s[0]}x{s[1]}x{s[2]}_{k['block_m']}x{k['block_n']}"
                                                   + ("_sk" if "split_k" in k else "") for s, k in KNOBS])
def test_layouts_match_oracle(cuda, shape, knobs, a_col, b_col):
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    import oracle
    m, n, k = shape
    A, B, Cin = make_inputs(m, n, k, 61, "uniform")
    tA = _col_major(A, 8, cuda) if a_col else torch.from_numpy(A).to(cuda)
    tB = _col_major(B, 16, cuda) if b_col else torch.from_numpy(B).to(cuda)
    assert (tA.stride(0) == 1) == a_col and (tB.stride(0) == 1) == b_col
    tC = torch.from_numpy(Cin).to(cuda)
    tb.matmul(tA, tB, tC, **knobs)
    err = float(np.abs(tC.cpu().numpy() - oracle.matmul_ref(A, B, Cin)).max())
    assert err <= oracle.tolerance(k), err


def test_layout_leading_dimension_rules(cuda):
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    p = tb.MatmulPlan(tb.KernelConfig(m=256, n=128, k=64, block_m=128, block_n=128, block_k=64,
                                      a_col_major=True), 0)
    assert p.info["a_layout"] == "col_major"
    A = torch.zeros(64, 256, dtype=torch.float16, device=cuda)
    B = torch.zeros(64, 128, dtype=torch.float16, device=cuda)
    C = torch.zeros(256, 128, device=cuda)
    with pytest.raises(tb.TBError, match="leading dimensions"):
        p.run_ptr(A.data_ptr(), 64, B.data_ptr(), 128, C.data_ptr(), 128)  # lda < m
    p.run_ptr(A.data_ptr(), 256, B.data_ptr(), 128, C.data_ptr(), 128)
