"""GPU: seeded random knob sets and shapes (ragged edges, every tile family,
split-K in both modes, persistent walks, transposed operands, f16 output,
beta = 0, fused epilogue expressions) against the CPU oracle. Each case is
small enough for the oracle to finish in milliseconds."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import make_inputs

pytestmark = pytest.mark.gpu


def _cases(count=240, seed=1234, big=False, fusing=False):
    rng = np.random.default_rng(seed)
    out = []
    while len(out) < count:
        bm = int(rng.choice([64, 128, 256]))
        bn = int(rng.choice([64, 128, 256, 512]))
        bk = int(rng.choice([16, 32, 64]))
        hi = 3000 if big else 700
        m, n, k = (int(x) for x in rng.integers(1, hi, 3))
        if fusing:  # enough 128-class programs for the 2 × 2 / horizontal fusions
            bm, bn = int(rng.choice([128, 256])), 128
            # even tile counts (ragged last tiles) so both fusions can apply
            m = 2 * bm * int(rng.integers(8, 15)) - int(rng.integers(0, bm))
            n = 256 * int(rng.integers(8, 15)) - int(rng.integers(0, 128))
            k = int(rng.integers(64, 600))
        k = max(k, 16)
        kn = dict(block_m=bm, block_n=bn, block_k=bk, exact_tile=False,
                  group_m=int(rng.choice([2, 4, 6, 8])) if fusing else int(rng.integers(1, 9)))
        mode = "plain" if fusing else rng.choice(["plain", "persistent", "serial", "parallel"])
        if mode == "persistent":
            kn.update(persistent=True, num_ctas=int(rng.integers(1, 200)))
        elif mode in ("serial", "parallel"):
            kn.update(split_k=int(rng.integers(2, 6)), reduction_mode=f"split_k_{mode}")
        out_dtype = "f32" if mode == "parallel" else str(rng.choice(["f32", "f16"]))
        beta = 1 if mode == "parallel" else int(rng.integers(0, 2))
        ex = {}
        if mode != "parallel" and rng.random() < 0.3:
            ex = dict(activation=str(rng.choice(["relu", "silu", "gelu_tanh"])), bias=True)
        layout = (bool(rng.random() < 0.25), bool(rng.random() < 0.25))
        out.append(((m, n, k), kn, out_dtype, beta, ex, layout))
    return out


# many small cases, then fewer multi-wave ones (several tiles per CTA)
CASES = _cases() + _cases(40, seed=777, big=True) + _cases(24, seed=4242, fusing=True)


def _view(x: np.ndarray, col_major: bool, dev):
    import torch
    if not col_major:
        return torch.from_numpy(x).to(dev)
    return torch.from_numpy(np.ascontiguousarray(x.T)).to(dev).t()


@pytest.mark.parametrize("case", CASES, ids=[f"{i}" for i in range(len(CASES))])
def test_random_config_matches_oracle(cuda, case):
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    import oracle
    (m, n, k), kn, out_dtype, beta, ex, (a_col, b_col) = case
    # TMA reads rows with 16-byte strides: a column-major operand needs its
    # leading dimension (m or k) to be a multiple of 8 — else keep row-major
    a_col = a_col and m % 8 == 0
    b_col = b_col and k % 8 == 0
    A, B, Cin = make_inputs(m, n, k, 7 + m + n + k, "uniform")
    if out_dtype == "f16":
        Cin = Cin.astype(np.float16).astype(np.float32)
    bias = np.random.default_rng(m * n).standard_normal(n).astype(np.float32) if ex.get("bias") else None
    tC = torch.from_numpy(Cin.astype(np.float16) if out_dtype == "f16" else Cin).to(cuda)
    tA, tB = _view(A, a_col, cuda), _view(B, b_col, cuda)
    tbias = None if bias is None else torch.from_numpy(bias).to(cuda)
    if (m + n + k) % 3 == 0:
        # every third case through a dynamic-shape plan (all dims open)
        cfg = tb.KernelConfig(m=None, n=None, k=None, c_dtype=out_dtype, beta=beta, bias=bias is not None,
                              activation=ex.get("activation"), a_col_major=a_col, b_col_major=b_col, **kn)
        tb.DynamicMatmulPlan(cfg, cuda.index or 0).run(tA, tB, tC, bias=tbias)
    else:
        tb.matmul(tA, tB, tC, beta=beta, bias=tbias, activation=ex.get("activation"), **kn)
    torch.cuda.synchronize()
    assert tb.device_status() == 0
    want = oracle.apply_epilogue(oracle.matmul_ref(A, B, Cin if beta else None, beta=beta), bias,
                                 ex.get("activation"), None)
    got = tC.float().cpu().numpy()
    tol = oracle.tolerance(k) * 1.15 + 1e-5
    if out_dtype == "f16":
        tol += float(np.abs(np.spacing(want.astype(np.float16))).max())
    err = float(np.abs(got - want).max())
    assert err <= tol, (case, err, tol)
