"""Multi-GPU partitions of one tb.matmul (one process per GPU).

The reference is single-GPU; these are the two partitions its hot path
admits on one B200 box:

* N-column sharding (large square shapes): rank r owns columns
  [n0_r, n0_r + n_r) of B and C, A is replicated, and each rank runs the
  single-GPU op on its slice — no communication.
* K sharding (skinny / split-K shapes): rank r owns A[:, K_r] and B[K_r, :],
  computes the partial P_r = A_r·B_r in f32, and a reduce-scatter (sum) over
  the ranks leaves rank r with rows [m0_r, m0_r + m_r) of Σ_r P_r, to which it
  adds its rows of C_in. This is the split-K reduction of the reference
  (ReductionPlan.cpp:137-192) with the split parts on different GPUs.

`local_matmul` lets the host logic run with any local GEMM (the CPU oracle
in gloo tests); the default is this package's sm_100a kernel.
"""
from __future__ import annotations

from typing import Callable, Optional


def balanced_shard(total: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """[start, start + size) of `rank`'s share of `total` items, in units of
    `align` (the last rank takes the ragged remainder)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if align <= 0:
        raise ValueError("align must be positive")
    units = (total + align - 1) // align
    base, extra = divmod(units, world)
    u0 = rank * base + min(rank, extra)
    u1 = u0 + base + (1 if rank < extra else 0)
    start = min(total, u0 * align)
    end = min(total, u1 * align)
    return start, end - start


def column_shard(n: int, world: int, rank: int, block_n: int) -> tuple[int, int]:
    """Columns of B/C owned by `rank` under N-sharding, whole program tiles
    (block_n) per rank so every rank runs the same tile shape."""
    return balanced_shard(n, world, rank, align=block_n)


def k_shard(k: int, world: int, rank: int, block_k: int) -> tuple[int, int]:
    """K range of `rank` under K-sharding, whole block_k tiles, which also
    keeps every A column offset a multiple of 16 elements (TMA alignment)."""
    return balanced_shard(k, world, rank, align=block_k)


def row_shard(m: int, world: int, rank: int) -> tuple[int, int]:
    """Rows of C that `rank` receives from the reduce-scatter (equal slices;
    m must divide by world)."""
    if m % world:
        raise ValueError("K-sharded tb.matmul needs m divisible by the world size")
    return rank * (m // world), m // world


def _default_local_matmul():
    from . import matmul
    return matmul


def matmul_nshard(A, B_local, C_local, local_matmul: Optional[Callable] = None, **knobs):
    """N-sharded tb.matmul: C_local ← C_local + A·B_local (no collective)."""
    f = local_matmul or _default_local_matmul()
    return f(A, B_local, C_local, **knobs)


class NShard:
    """N-column sharded tb.matmul through the C ABI (tb_matmul_run_nshard):
    `cfg` describes the WHOLE m × n × k problem; rank `rank` of `world` runs
    its columns [col0, col0 + ncols) (whole block_n tiles, balanced) with the
    same knobs. No collective."""

    def __init__(self, cfg, rank: int, world: int, device: Optional[int] = None):
        import ctypes as C
        from . import MatmulPlan, _check, _load_lib
        self._lib = _load_lib()
        self._check = _check
        self.plan = MatmulPlan(cfg, device)
        self.rank, self.world = rank, world
        c0, nc = C.c_int64(0), C.c_int64(0)
        _check(self._lib.tb_matmul_nshard_columns(self.plan._h, rank, world, C.byref(c0), C.byref(nc)))
        self.col0, self.ncols = c0.value, nc.value
        ws = C.c_size_t(0)
        _check(self._lib.tb_matmul_nshard_workspace_bytes(self.plan._h, rank, world, C.byref(ws)))
        self.workspace_bytes = ws.value

    def run_ptr(self, a_ptr: int, lda: int, b_ptr: int, ldb: int, c_ptr: int, ldc: int,
                ws_ptr: int = 0, ws_bytes: int = 0, stream: int = 0, bias_ptr: int = 0) -> None:
        """b_ptr / c_ptr address column col0 of B and C (this rank's slices)."""
        import ctypes as C
        self._check(self._lib.tb_matmul_run_nshard(
            self.plan._h, self.rank, self.world, C.c_void_p(a_ptr), lda, C.c_void_p(b_ptr), ldb,
            C.c_void_p(c_ptr), ldc, C.c_void_p(bias_ptr or None), C.c_void_p(ws_ptr or None), ws_bytes,
            C.c_void_p(stream or None)))

    def run(self, A, B_cols, C_cols, workspace=None, stream=None, bias_cols=None) -> None:
        """A [m, k]; B_cols [k, ncols] and C_cols [m, ncols]: this rank's
        slices (or column views of full matrices), unit minor stride."""
        import torch
        if tuple(B_cols.shape) != (self.plan.cfg.k, self.ncols) or \
                tuple(C_cols.shape) != (self.plan.cfg.m, self.ncols):
            raise ValueError(f"rank {self.rank} owns {self.ncols} columns from {self.col0}")
        ws_ptr, ws_bytes = 0, 0
        if self.workspace_bytes:
            if workspace is None:
                workspace = torch.empty(self.workspace_bytes, dtype=torch.uint8, device=C_cols.device)
            ws_ptr, ws_bytes = workspace.data_ptr(), workspace.numel()
        s = stream if stream is not None else torch.cuda.current_stream(C_cols.device)
        self.run_ptr(A.data_ptr(), A.stride(0), B_cols.data_ptr(), B_cols.stride(0), C_cols.data_ptr(),
                     C_cols.stride(0), ws_ptr, ws_bytes, s.cuda_stream,
                     0 if bias_cols is None else bias_cols.data_ptr())


def matmul_kshard(A_local, B_local, C_rows, group=None, local_matmul: Optional[Callable] = None,
                  partial=None, **knobs):
    """K-sharded tb.matmul with a reduce-scatter.

    A_local: [m, k_r] (this rank's K columns of A), B_local: [k_r, n],
    C_rows: [m / world, n] f32 — this rank's rows of C, updated in place to
    C_in + Σ_r A_r·B_r. `partial` ([m, n] f32 scratch) is allocated when
    omitted. Returns C_rows."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    m, n = A_local.shape[0], B_local.shape[1]
    if C_rows.shape != (m // world, n) or m % world:
        raise ValueError("C_rows must be this rank's [m / world, n] slice")
    if partial is None:
        partial = torch.empty(m, n, dtype=torch.float32, device=C_rows.device)
    f = local_matmul or _default_local_matmul()
    f(A_local, B_local, partial, beta=0, **knobs)
    recv = torch.empty_like(C_rows)
    dist.reduce_scatter_tensor(recv, partial, op=dist.ReduceOp.SUM, group=group)
    C_rows.add_(recv)
    return C_rows


class PeerKShard:
    """K-sharded tb.matmul whose reduce-scatter is fused into the GEMM (the C
    ABI's tb_matmul_run_kshard_peer): each rank's epilogue adds its partial
    tiles straight into the owning rank's rows of C over NVLink.

    C_rows: this rank's [m / world, n] f32 rows of C (CUDA memory, unit minor
    stride); it is registered once and updated in place by every run. The
    constructor is collective (it exchanges CUDA IPC handles through
    `group`, any torch.distributed backend)."""

    def __init__(self, C_rows, group=None):
        import ctypes as C
        import torch.distributed as dist
        from . import _capi, _load_lib, _check
        self._lib = _load_lib()
        self._check = _check
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if C_rows.dtype.itemsize != 4 or C_rows.stride(1) != 1 or not C_rows.is_cuda:
            raise ValueError("C_rows must be an f32 CUDA tensor with unit minor stride")
        self.C_rows = C_rows
        self.rows_per_rank, self.n = C_rows.shape
        self._h = C.c_void_p()
        mine = _capi.tb_peer_handle()
        _check(self._lib.tb_peer_comm_create(self.rank, self.world, C.c_void_p(C_rows.data_ptr()),
                                             self.rows_per_rank, self.n, C_rows.stride(0),
                                             C.byref(self._h), C.byref(mine)))
        blobs = [None] * self.world
        dist.all_gather_object(blobs, bytes(mine), group=group)
        arr = (_capi.tb_peer_handle * self.world)()
        for r, b in enumerate(blobs):
            C.memmove(C.byref(arr[r]), b, C.sizeof(_capi.tb_peer_handle))
        _check(self._lib.tb_peer_comm_connect(self._h, arr))

    def run(self, plan, A_local, B_local, stream=None):
        """C_rows ← C_rows + Σ_ranks A_local·B_local restricted to these rows.
        `plan`: MatmulPlan of the local problem (m × n × k_local)."""
        import ctypes as C
        import torch
        s = stream if stream is not None else torch.cuda.current_stream(A_local.device)
        self._check(self._lib.tb_matmul_run_kshard_peer(
            plan._h, self._h, C.c_void_p(A_local.data_ptr()), A_local.stride(0),
            C.c_void_p(B_local.data_ptr()), B_local.stride(0), C.c_void_p(s.cuda_stream or None)))

    def barrier(self, stream=None):
        import ctypes as C
        import torch
        s = stream if stream is not None else torch.cuda.current_stream(self.C_rows.device)
        self._check(self._lib.tb_peer_barrier(self._h, C.c_void_p(s.cuda_stream or None)))

    def check(self, stream=None) -> int:
        """Synchronises; raises TBError(TB_ERR_DEVICE_TIMEOUT) if a barrier gave up."""
        import ctypes as C
        import torch
        s = stream if stream is not None else torch.cuda.current_stream(self.C_rows.device)
        raw = C.c_uint32(0)
        self._check(self._lib.tb_peer_comm_status(self._h, C.c_void_p(s.cuda_stream or None), C.byref(raw)))
        return raw.value

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            self._lib.tb_peer_comm_destroy(self._h)
            self._h = None


class NcclKShard:
    """K-sharded tb.matmul through the C ABI's NCCL path
    (tb_matmul_run_kshard_nccl): each rank's K-slice GEMM runs into an f32
    staging copy of C, then one ncclReduceScatter leaves every rank its rows.

    C_rows: this rank's [m / world, n] f32 rows of C (CUDA memory, unit minor
    stride), updated in place by every run. The constructor is collective: rank
    0 makes the NCCL unique id and `group` (any torch.distributed backend)
    carries it to the others."""

    def __init__(self, C_rows, group=None):
        import ctypes as C
        import torch.distributed as dist
        from . import _check, _load_lib
        self._lib = _load_lib()
        self._check = _check
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if C_rows.dtype.itemsize != 4 or C_rows.stride(1) != 1 or not C_rows.is_cuda:
            raise ValueError("C_rows must be an f32 CUDA tensor with unit minor stride")
        self.C_rows = C_rows
        uid = C.create_string_buffer(128)
        if self.rank == 0:
            _check(self._lib.tb_nccl_unique_id(uid))
        box = [bytes(uid.raw)]
        dist.broadcast_object_list(box, src=0 if group is None else dist.get_global_rank(group, 0),
                                   group=group)
        self._h = C.c_void_p()
        _check(self._lib.tb_nccl_comm_create(self.rank, self.world, box[0], C.byref(self._h)))
        self._ws = None

    def run(self, plan, A_local, B_local, stream=None):
        """C_rows ← C_rows + Σ_ranks A_local·B_local restricted to these rows
        (beta = 1 plans; beta = 0 gives the sum alone). `plan`: MatmulPlan of
        the local problem (m × n × k_local)."""
        import ctypes as C
        import torch
        need = int(self._lib.tb_matmul_kshard_nccl_workspace_bytes(plan._h, self.world,
                                                                    self.C_rows.stride(0)))
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.C_rows.device)
        s = stream if stream is not None else torch.cuda.current_stream(A_local.device)
        lda = A_local.stride(1) if plan.cfg.a_col_major else A_local.stride(0)
        ldb = B_local.stride(1) if plan.cfg.b_col_major else B_local.stride(0)
        self._check(self._lib.tb_matmul_run_kshard_nccl(
            plan._h, self._h, C.c_void_p(A_local.data_ptr()), lda, C.c_void_p(B_local.data_ptr()), ldb,
            C.c_void_p(self.C_rows.data_ptr()), self.C_rows.stride(0), C.c_void_p(self._ws.data_ptr()),
            self._ws.numel(), C.c_void_p(s.cuda_stream or None)))

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            self._lib.tb_nccl_comm_destroy(self._h)
            self._h = None
