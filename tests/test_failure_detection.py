"""Failure detection without a GPU fault.

GPU: a bounded device-side wait on a flag nothing sets expires, the kernel
records TB_ERR_DEVICE_TIMEOUT in the status word the host reads, and the
context stays usable (a GEMM afterwards is correct). CPU: argument and state
errors of the multi-GPU host path, and a rank that fails before a collective
makes the others fail with an error instead of hanging (gloo, short timeout).
"""
from __future__ import annotations

import ctypes as C
import datetime
import os
import socket

import numpy as np
import pytest

from conftest import make_inputs


@pytest.mark.gpu
def test_expired_device_wait_is_reported_and_context_survives(cuda):
    import torch
    import mini_triton_nvgpu_v1_b200 as tb
    import oracle
    from mini_triton_nvgpu_v1_b200 import _capi
    lib = _capi.load()
    assert tb.device_status() == 0
    assert lib.tb_selftest_bounded_wait(None, 2_000_000) == 0        # ~1 ms of SM clocks
    with pytest.raises(tb.TBError) as e:
        tb.device_status()
    assert e.value.code == _capi.TB_ERR_DEVICE_TIMEOUT
    assert tb.device_status() == 0                                     # read-and-clear
    A, B, Cin = make_inputs(256, 256, 128, 81, "uniform")
    tC = torch.from_numpy(Cin).to(cuda)
    tb.matmul(torch.from_numpy(A).to(cuda), torch.from_numpy(B).to(cuda), tC, block_m=128,
              block_n=128, block_k=64)
    assert tb.device_status() == 0
    assert float(np.abs(tC.cpu().numpy() - oracle.matmul_ref(A, B, Cin)).max()) <= oracle.tolerance(128)


def test_selftest_budget_is_validated():
    from mini_triton_nvgpu_v1_b200 import _capi
    lib = _capi.load()
    assert lib.tb_selftest_bounded_wait(None, 0) == _capi.TB_ERR_INVALID_ARGUMENT
    assert lib.tb_selftest_bounded_wait(None, 3_000_000_000) == _capi.TB_ERR_INVALID_ARGUMENT


def test_peer_comm_host_errors():
    from mini_triton_nvgpu_v1_b200 import _capi
    lib = _capi.load()
    h = _capi.tb_peer_handle()
    comm = C.c_void_p()
    assert lib.tb_peer_comm_create(0, 9, C.c_void_p(0x1000), 64, 64, 64, C.byref(comm), C.byref(h)) \
        == _capi.TB_ERR_INVALID_ARGUMENT
    assert lib.tb_peer_comm_create(2, 2, C.c_void_p(0x1000), 64, 64, 64, C.byref(comm), C.byref(h)) \
        == _capi.TB_ERR_INVALID_ARGUMENT
    assert lib.tb_peer_comm_create(0, 2, None, 64, 64, 64, C.byref(comm), C.byref(h)) \
        == _capi.TB_ERR_INVALID_ARGUMENT
    assert lib.tb_peer_barrier(None, None) == _capi.TB_ERR_INVALID_ARGUMENT
    assert lib.tb_matmul_run_kshard_peer(None, None, None, 0, None, 0, None) == _capi.TB_ERR_INVALID_ARGUMENT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, port, q):
    import torch
    import torch.distributed as dist
    from mini_triton_nvgpu_v1_b200 import parallel as par
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves between steps, without joining the collective
    try:
        A = torch.zeros(64, 32, dtype=torch.float16)
        B = torch.zeros(32, 64, dtype=torch.float16)
        rows = torch.zeros(32, 64)

        def local(A, B, C, beta=1, **_):
            C.zero_()
            return C
        par.matmul_kshard(A, B, rows, local_matmul=local)
        q.put((0, "no error"))
    except Exception as e:  # the collective must fail, not hang
        q.put((0, type(e).__name__))


def test_a_rank_that_leaves_makes_the_collective_fail_not_hang():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    rank0, outcome = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert procs[1].exitcode == 0
    assert rank0 == 0 and outcome != "no error", outcome
