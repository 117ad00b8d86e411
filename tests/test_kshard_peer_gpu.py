"""GPU, 2 ranks (one process per GPU; skipped with fewer than 2 GPUs): the
fused K-sharded GEMM + reduce-scatter over NVLink (PeerKShard) against the
CPU oracle and against the NCCL-collective version of the same partition."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, m, n, k, knobs):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        import mini_triton_nvgpu_v1_b200 as tb
        from mini_triton_nvgpu_v1_b200 import parallel as par
        import oracle
        dev = torch.device("cuda", rank)
        rng = np.random.default_rng(41)
        A = rng.uniform(-1, 1, (m, k)).astype(np.float16)
        B = rng.uniform(-1, 1, (k, n)).astype(np.float16)
        Cin = rng.standard_normal((m, n)).astype(np.float32)
        k0, kr = par.k_shard(k, world, rank, knobs["block_k"])
        r0, mr = par.row_shard(m, world, rank)
        tA = torch.from_numpy(A[:, k0:k0 + kr].copy()).to(dev)
        tB = torch.from_numpy(B[k0:k0 + kr].copy()).to(dev)
        rows = torch.from_numpy(Cin[r0:r0 + mr].copy()).to(dev)
        comm = par.PeerKShard(rows)
        plan = tb.MatmulPlan(tb.KernelConfig(m=m, n=n, k=kr, **knobs), rank)
        for _ in range(2):  # C += A·B twice
            comm.run(plan, tA, tB)
        assert comm.check() == 0
        got = rows.cpu().numpy()
        once = oracle.matmul_ref(A, B, Cin)
        want = oracle.matmul_ref(A, B, once)[r0:r0 + mr]
        err = float(np.abs(got - want).max())
        # the NCCL-collective version of the same partition
        rows2 = torch.from_numpy(Cin[r0:r0 + mr].copy()).to(dev)
        par.matmul_kshard(tA, tB, rows2, **{kk: v for kk, v in knobs.items()
                                           if kk not in ("split_k", "reduction_mode")})
        err2 = float(np.abs(rows2.cpu().numpy() - once[r0:r0 + mr]).max())
        comm.close()
        # the C ABI's NCCL path (tb_matmul_run_kshard_nccl), into a strided view of C rows
        wide = torch.zeros(mr, n + 8, device=dev)
        wide[:, :n] = torch.from_numpy(Cin[r0:r0 + mr].copy()).to(dev)
        rows3 = wide[:, :n]
        nc = par.NcclKShard(rows3)
        for _ in range(2):
            nc.run(plan, tA, tB)
        torch.cuda.synchronize()
        nc.close()
        err3 = float(np.abs(rows3.cpu().numpy() - want).max())
        assert float(wide[:, n:].abs().max()) == 0.0          # nothing written past n
        q.put((rank, max(err, err3), err2, oracle.tolerance(k)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shape,knobs", [
    ((512, 512, 8192), dict(block_m=256, block_n=256, block_k=64, split_k=4,
                            reduction_mode="split_k_parallel")),
    ((512, 384, 4096), dict(block_m=128, block_n=128, block_k=64)),
    # 256 × 200 rows per rank is not a whole number of 16 KB chunks: atomics path
    ((512, 200, 2048), dict(block_m=128, block_n=128, block_k=64, exact_tile=False)),
    # ragged K slices, 1-CTA tiles, three split parts per rank
    ((768, 264, 3000), dict(block_m=128, block_n=128, block_k=32, split_k=3,
                            reduction_mode="split_k_parallel", exact_tile=False)),
])
def test_two_rank_fused_kshard(cuda, shape, knobs):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, *shape, knobs)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, err2, tol in res:
        assert err <= 2 * tol, (rank, err)
        assert err2 <= tol, (rank, err2)


def _nshard_worker(rank, world, q, m, n, k, knobs):
    import torch
    torch.cuda.set_device(rank)
    import mini_triton_nvgpu_v1_b200 as tb
    from mini_triton_nvgpu_v1_b200 import parallel as par
    import oracle
    dev = torch.device("cuda", rank)
    rng = np.random.default_rng(43)
    A = rng.uniform(-1, 1, (m, k)).astype(np.float16)
    B = rng.uniform(-1, 1, (k, n)).astype(np.float16)
    Cin = rng.standard_normal((m, n)).astype(np.float32)
    sh = par.NShard(tb.KernelConfig(m=m, n=n, k=k, **knobs), rank, world, rank)
    c0, nc = sh.col0, sh.ncols
    tA = torch.from_numpy(A).to(dev)
    tB = torch.from_numpy(B[:, c0:c0 + nc].copy()).to(dev)
    tC = torch.from_numpy(Cin[:, c0:c0 + nc].copy()).to(dev)
    sh.run(tA, tB, tC)
    torch.cuda.synchronize()
    want = oracle.matmul_ref(A, B, Cin)[:, c0:c0 + nc]
    q.put((rank, c0, nc, float(np.abs(tC.cpu().numpy() - want).max()), oracle.tolerance(k)))


@pytest.mark.parametrize("shape,knobs", [
    ((1024, 2304, 1024), dict(block_m=256, block_n=256, block_k=64)),
    ((520, 1000, 700), dict(block_m=128, block_n=128, block_k=64, exact_tile=False)),
])
def test_two_rank_nshard(cuda, shape, knobs):
    """tb_matmul_run_nshard on two GPUs, one process each, no collective: the
    two column slices cover C once and each matches the oracle."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_nshard_worker, args=(r, 2, q, *shape, knobs)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][1] == 0 and res[0][2] + res[1][2] == shape[1] and res[1][1] == res[0][2]
    for rank, c0, nc, err, tol in res:
        assert err <= tol, (rank, err)
