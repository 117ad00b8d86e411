"""CPU, world_size 2 (gloo): the multi-GPU partitions' host logic with the
CPU oracle as the local GEMM. The sharded results must equal the single-rank
oracle result (N-shard: bit for bit — same k order per element; K-shard:
within f32 reassociation of the partial sums)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mini_triton_nvgpu_v1_b200 import parallel as par


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_matmul(A, B, C, beta=1, **_):
    import oracle
    out = oracle.matmul_ref(A.numpy(), B.numpy(), C.numpy() if beta else None, beta=beta)
    C.copy_(torch.from_numpy(out))
    return C


def _inputs(m, n, k, seed=5):
    rng = np.random.default_rng(seed)
    A = rng.uniform(-1, 1, (m, k)).astype(np.float16)
    B = rng.uniform(-1, 1, (k, n)).astype(np.float16)
    C = rng.standard_normal((m, n)).astype(np.float32)
    return A, B, C


def _worker(rank, world, port, kind, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle
        m, n, k = 96, 80, 160
        A, B, C = _inputs(m, n, k)
        if kind == "nshard":
            n0, nr = par.column_shard(n, world, rank, block_n=16)
            Cl = torch.from_numpy(C[:, n0:n0 + nr].copy())
            par.matmul_nshard(torch.from_numpy(A), torch.from_numpy(B[:, n0:n0 + nr].copy()), Cl,
                              local_matmul=_oracle_matmul)
            parts = [None] * world
            dist.all_gather_object(parts, (n0, Cl.numpy()))
            full = np.concatenate([p for _, p in sorted(parts, key=lambda t: t[0])], axis=1)
            ref = oracle.matmul_ref(A, B, C)
            q.put((rank, bool(np.array_equal(full, ref)), 0.0))
        else:
            k0, kr = par.k_shard(k, world, rank, block_k=32)
            r0, mr = par.row_shard(m, world, rank)
            rows = torch.from_numpy(C[r0:r0 + mr].copy())
            par.matmul_kshard(torch.from_numpy(A[:, k0:k0 + kr].copy()),
                              torch.from_numpy(B[k0:k0 + kr].copy()), rows,
                              local_matmul=_oracle_matmul)
            ref = oracle.matmul_ref(A, B, C)[r0:r0 + mr]
            err = float(np.abs(rows.numpy() - ref).max())
            q.put((rank, err <= 1e-4, err))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["nshard", "kshard"])
def test_two_rank_partitions(kind):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, kind, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in results), results


def test_balanced_shard_covers_exactly():
    for total, world, align in [(8192, 8, 256), (1000, 3, 64), (80, 2, 16), (7, 4, 8), (65536, 8, 64)]:
        spans = [par.balanced_shard(total, world, r, align) for r in range(world)]
        cur = 0
        for s, sz in spans:
            assert s == cur and sz >= 0
            assert s % align == 0 or s == total
            cur += sz
        assert cur == total


def test_shard_argument_errors():
    with pytest.raises(ValueError):
        par.balanced_shard(10, 2, 2)
    with pytest.raises(ValueError):
        par.row_shard(10, 3, 0)
