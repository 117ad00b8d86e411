"""B200-native `tb.matmul`: f16 × f16 → f32 (or f16) GEMM with the
reference's C-accumulate semantics, ``C = C_in + A·B``, and its knobs.

The host-side mirror of the reference operator surface::

    tb.matmul %A, %B, %C {block_m, block_n, block_k, group_m, exact_tile}
    module attributes {tb.num-warps, tb.requested-stages, tb.split-k,
                       tb.reduction-mode, tb.persistent, tb.num-ctas}

(include/tb/IR/TBOps.td:32-58, include/tb/Analysis/TargetInfo.h:17-21,
include/tb/Analysis/ProgramMappingPlan.h:14-17) is :func:`matmul` — it updates
``C`` in place, exactly as the lowered kernel updates its C memref. Knobs are
validated with the reference's rules and messages (:class:`TBError`).

Everything runs through ``libtbgemm.so`` (sm_100a CUDA); torch is used only for
device memory and streams.
"""
from __future__ import annotations

import ctypes as C
import json
from dataclasses import dataclass, field, asdict
from typing import Optional

from . import _capi
from ._capi import (TB_F16, TB_F32, TB_REDUCTION_SPLIT_K_PARALLEL, TB_REDUCTION_SPLIT_K_SERIAL,
                    TB_REDUCTION_UNSET)

_lib_handle = None


def _load_lib():
    """Loads libtbgemm.so on first use (raises ImportError if it is missing:
    there is no CPU fallback)."""
    global _lib_handle
    if _lib_handle is None:
        _lib_handle = _capi.load()
    return _lib_handle


class _LazyLib:
    def __getattr__(self, name):
        return getattr(_load_lib(), name)


_lib = _LazyLib()

__all__ = ["KernelConfig", "MatmulPlan", "DynamicMatmulPlan", "TBError", "matmul", "plan_for", "version", "lib"]

_REDUCTION = {None: TB_REDUCTION_UNSET, "": TB_REDUCTION_UNSET,
              "split_k_serial": TB_REDUCTION_SPLIT_K_SERIAL,
              "split_k_parallel": TB_REDUCTION_SPLIT_K_PARALLEL}


def lib() -> C.CDLL:
    return _load_lib()


def version() -> str:
    return _lib.tb_version().decode()


class TBError(RuntimeError):
    """A tbStatus other than TB_OK; ``.code`` is the status, the message is
    the library's (reference-worded where the rule is the reference's)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{_capi.STATUS_NAMES.get(code, code)}: {message}")
        self.code = code
        self.message = message


def _check(code: int) -> None:
    if code != _capi.TB_OK:
        raise TBError(code, _lib.tb_last_error().decode())


@dataclass(frozen=True)
class KernelConfig:
    """The knobs of one tb.matmul (KernelConfig.h:22-37 plus the module
    attributes). Defaults are the reference's attribute defaults."""
    m: int
    n: int
    k: int
    block_m: int
    block_n: int
    block_k: int
    group_m: int = 8
    exact_tile: bool = True
    num_warps: int = 4
    num_stages: int = 2
    split_k: int = 1
    reduction_mode: Optional[str] = None
    persistent: bool = False
    num_ctas: int = 1
    programs_per_tile: int = 0
    c_dtype: str = "f32"
    beta: int = 1
    # fused epilogue expressions (applied after the full sum, in this order)
    bias: bool = False                 # runs pass a length-n f32 bias
    activation: Optional[str] = None   # "relu" | "silu" | "gelu_tanh"
    clamp: Optional[tuple] = None      # (lo, hi)
    # operand storage: column-major A (m × k, lda >= m) / B (k × n, ldb >= k)
    a_col_major: bool = False
    b_col_major: bool = False
    # bitwise-repeatable runs: no stream-K tail (partial tiles reduce-added into C)
    deterministic: bool = False

    def to_desc(self) -> _capi.tb_matmul_desc:
        d = _capi.tb_matmul_desc()
        _check(_lib.tb_matmul_desc_init(C.byref(d)))
        # None leaves a dim open ("?"): only dynamic plans accept it
        d.m, d.n, d.k = (_capi.TB_DIM_DYNAMIC if x is None else x for x in (self.m, self.n, self.k))
        d.block_m, d.block_n, d.block_k = self.block_m, self.block_n, self.block_k
        d.group_m = self.group_m
        d.exact_tile = 1 if self.exact_tile else 0
        d.num_warps = self.num_warps
        d.num_stages = self.num_stages
        d.split_k = self.split_k
        if self.reduction_mode not in _REDUCTION:
            d.reduction_mode = 99  # rejected by the plan with the reference's message
        else:
            d.reduction_mode = _REDUCTION[self.reduction_mode]
        d.persistent = 1 if self.persistent else 0
        d.num_ctas = self.num_ctas
        d.programs_per_tile = self.programs_per_tile
        d.a_dtype = TB_F16
        d.b_dtype = TB_F16
        d.c_dtype = {"f32": TB_F32, "f16": TB_F16, "bf16": _capi.TB_BF16}.get(self.c_dtype, 99)
        d.beta = int(self.beta)
        d.bias = 1 if self.bias else 0
        d.activation = _capi.ACTIVATIONS.get(self.activation, 99)
        if self.clamp is not None:
            d.clamp = 1
            d.clamp_lo, d.clamp_hi = float(self.clamp[0]), float(self.clamp[1])
        d.a_col_major = 1 if self.a_col_major else 0
        d.b_col_major = 1 if self.b_col_major else 0
        d.deterministic = 1 if self.deterministic else 0
        return d


class MatmulPlan:
    """A validated plan (C ABI ``tb_matmul_plan``). ``device=None`` plans for
    a B200 without touching CUDA (host-only checks)."""

    def __init__(self, cfg: KernelConfig, device: Optional[int] = None):
        self.cfg = cfg
        self._h = C.c_void_p()
        desc = cfg.to_desc()
        _check(_lib.tb_matmul_plan_create(C.byref(desc), -1 if device is None else int(device),
                                          C.byref(self._h)))
        self.device = device
        self.info = self._describe()

    def __del__(self):
        h = getattr(self, "_h", None)
        lib_ = _lib_handle  # may already be None during interpreter shutdown
        if h is not None and h.value and lib_ is not None:
            lib_.tb_matmul_plan_destroy(h)
            self._h = C.c_void_p()

    def _describe(self) -> dict:
        need = C.c_size_t(0)
        _lib.tb_matmul_plan_describe(self._h, None, 0, C.byref(need))
        buf = C.create_string_buffer(need.value)
        _check(_lib.tb_matmul_plan_describe(self._h, buf, need.value, C.byref(need)))
        return json.loads(buf.value.decode())

    @property
    def workspace_bytes(self) -> int:
        return int(_lib.tb_matmul_workspace_bytes(self._h))

    @property
    def total_programs(self) -> int:
        return int(self.info["total_programs"])

    def program_work(self, pid: int) -> tuple[int, int, int, int, int]:
        """(tile_m, tile_n, split_part, k_tile_begin, k_tile_count) of `pid`."""
        w = _capi.tb_program_work()
        _check(_lib.tb_matmul_program_work(self._h, int(pid), C.byref(w)))
        return (w.tile_m, w.tile_n, w.split_part, w.k_tile_begin, w.k_tile_count)

    def run_ptr(self, a_ptr: int, lda: int, b_ptr: int, ldb: int, c_ptr: int, ldc: int,
                ws_ptr: int = 0, ws_bytes: int = 0, stream: int = 0, bias_ptr: int = 0) -> None:
        """Raw-pointer launch (device addresses)."""
        if bias_ptr or self.cfg.bias:
            _check(_lib.tb_matmul_run_epilogue(self._h, C.c_void_p(a_ptr), lda, C.c_void_p(b_ptr), ldb,
                                               C.c_void_p(c_ptr), ldc, C.c_void_p(bias_ptr or None),
                                               C.c_void_p(ws_ptr or None), ws_bytes,
                                               C.c_void_p(stream or None)))
            return
        _check(_lib.tb_matmul_run(self._h, C.c_void_p(a_ptr), lda, C.c_void_p(b_ptr), ldb,
                                  C.c_void_p(c_ptr), ldc, C.c_void_p(ws_ptr or None), ws_bytes,
                                  C.c_void_p(stream or None)))

    def run(self, A, B, Cm, workspace=None, stream=None, bias=None) -> None:
        """C ← beta·C + A·B in place, on torch CUDA tensors."""
        import torch
        _check_tensors(self.cfg, A, B, Cm)
        ws_ptr, ws_bytes = 0, 0
        need = self.workspace_bytes
        if need:
            if workspace is None:
                workspace = torch.empty(need, dtype=torch.uint8, device=Cm.device)
            ws_ptr, ws_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
        s = stream if stream is not None else torch.cuda.current_stream(Cm.device)
        bias_ptr = 0
        if bias is not None:
            if bias.dtype != torch.float32 or bias.numel() != self.cfg.n or not bias.is_contiguous() \
                    or not bias.is_cuda:
                raise TBError(_capi.TB_ERR_INVALID_ARGUMENT, "bias must be a contiguous f32 CUDA vector of n")
            bias_ptr = bias.data_ptr()
        lda = A.stride(1) if self.cfg.a_col_major else A.stride(0)
        ldb = B.stride(1) if self.cfg.b_col_major else B.stride(0)
        self.run_ptr(A.data_ptr(), lda, B.data_ptr(), ldb, Cm.data_ptr(),
                     Cm.stride(0), ws_ptr, ws_bytes, s.cuda_stream, bias_ptr)


class DynamicMatmulPlan:
    """A plan whose problem dims may be left open (``None`` in the
    KernelConfig, ``memref<?x…>`` in the reference spelling, which the
    reference rejects). Knobs are validated once here; each ``run`` takes its
    shape from the tensors, and the library derives and caches the concrete
    plan of each shape (C ABI ``tb_matmul_plan_create_dynamic``)."""

    def __init__(self, cfg: KernelConfig, device: Optional[int] = None):
        self.cfg = cfg
        self._h = C.c_void_p()
        desc = cfg.to_desc()
        _check(_lib.tb_matmul_plan_create_dynamic(C.byref(desc), -1 if device is None else int(device),
                                                  C.byref(self._h)))
        self.device = device

    def __del__(self):
        h = getattr(self, "_h", None)
        lib_ = _lib_handle
        if h is not None and h.value and lib_ is not None:
            lib_.tb_matmul_plan_destroy(h)
            self._h = C.c_void_p()

    @property
    def info(self) -> dict:
        return MatmulPlan._describe(self)

    def workspace_bytes(self, m: int, n: int, k: int) -> int:
        out = C.c_size_t(0)
        _check(_lib.tb_matmul_workspace_bytes_dynamic(self._h, m, n, k, C.byref(out)))
        return int(out.value)

    def shape_info(self, m: int, n: int, k: int) -> dict:
        """Plan facts of the concrete plan for m×n×k."""
        h = C.c_void_p()
        _check(_lib.tb_matmul_plan_for_shape(self._h, m, n, k, C.byref(h)))
        try:
            need = C.c_size_t(0)
            _lib.tb_matmul_plan_describe(h, None, 0, C.byref(need))
            buf = C.create_string_buffer(need.value)
            _check(_lib.tb_matmul_plan_describe(h, buf, need.value, C.byref(need)))
            return json.loads(buf.value.decode())
        finally:
            _lib.tb_matmul_plan_destroy(h)

    def run(self, A, B, Cm, workspace=None, stream=None, bias=None) -> None:
        """C ← beta·C + A·B in place for the tensors' own m, n, k."""
        import torch
        m, k = A.shape
        n = B.shape[1]
        _check_tensors(self.cfg, A, B, Cm, shape=(m, n, k))
        ws_ptr, ws_bytes = 0, 0
        need = self.workspace_bytes(m, n, k)
        if need:
            if workspace is None:
                workspace = torch.empty(need, dtype=torch.uint8, device=Cm.device)
            ws_ptr, ws_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
        if bias is not None and (bias.dtype != torch.float32 or bias.numel() != n
                                 or not bias.is_contiguous() or not bias.is_cuda):
            raise TBError(_capi.TB_ERR_INVALID_ARGUMENT, "bias must be a contiguous f32 CUDA vector of n")
        s = stream if stream is not None else torch.cuda.current_stream(Cm.device)
        lda = A.stride(1) if self.cfg.a_col_major else A.stride(0)
        ldb = B.stride(1) if self.cfg.b_col_major else B.stride(0)
        _check(_lib.tb_matmul_run_dynamic(self._h, m, n, k, A.data_ptr(), lda, B.data_ptr(), ldb,
                                          Cm.data_ptr(), Cm.stride(0),
                                          None if bias is None else bias.data_ptr(),
                                          ws_ptr or None, ws_bytes, s.cuda_stream or None))


def _check_tensors(cfg: KernelConfig, A, B, Cm, shape=None) -> None:
    import torch
    if A.dtype != torch.float16 or B.dtype != torch.float16:
        raise TBError(_capi.TB_ERR_INVALID_ARGUMENT,
                      "stage1 currently supports fp16 x fp16 -> fp32 matmul kernels")
    want_c = torch.float32 if cfg.c_dtype == "f32" else torch.float16
    if Cm.dtype != want_c:
        raise TBError(_capi.TB_ERR_INVALID_ARGUMENT, f"C must be {want_c}")
    for t, name, col in ((A, "A", cfg.a_col_major), (B, "B", cfg.b_col_major), (Cm, "C", False)):
        if t.dim() != 2:
            raise TBError(_capi.TB_ERR_INVALID_ARGUMENT, "tb.matmul currently requires rank-2 memrefs")
        if not t.is_cuda:
            raise TBError(_capi.TB_ERR_INVALID_ARGUMENT, f"{name} must be a CUDA tensor")
        if t.stride(0 if col else 1) != 1:
            raise TBError(_capi.TB_ERR_UNSUPPORTED,
                          f"{name} must have a unit stride along its {'rows' if col else 'columns'}")
    m, n, k = shape if shape is not None else (cfg.m, cfg.n, cfg.k)
    if tuple(A.shape) != (m, k) or tuple(B.shape) != (k, n) or tuple(Cm.shape) != (m, n):
        raise TBError(_capi.TB_ERR_INVALID_ARGUMENT, "operand shapes disagree with the plan")


_PLAN_CACHE: dict = {}


def plan_for(cfg: KernelConfig, device: Optional[int]) -> MatmulPlan:
    key = (cfg, device)
    p = _PLAN_CACHE.get(key)
    if p is None:
        p = MatmulPlan(cfg, device)
        if len(_PLAN_CACHE) > 256:
            _PLAN_CACHE.clear()
        _PLAN_CACHE[key] = p
    return p


def matmul(A, B, Cm, *, block_m: int = 128, block_n: int = 256, block_k: int = 64,
           group_m: int = 8, exact_tile: Optional[bool] = None, num_warps: int = 4,
           num_stages: int = 2, split_k: int = 1, reduction_mode: Optional[str] = None,
           persistent: bool = False, num_ctas: int = 1, beta: int = 1, workspace=None,
           stream=None, bias=None, activation: Optional[str] = None, clamp=None,
           deterministic: bool = False):
    """``tb.matmul %A, %B, %C {…}``: C ← C + A·B in place (beta=1, the
    reference semantics) or C ← A·B (beta=0). A [m,k] f16, B [k,n] f16,
    C [m,n] f32 (or f16, this build's extension). Returns C.

    ``exact_tile=None`` picks True when the tile divides the problem.
    ``bias`` (f32, length n), ``activation`` ("relu" | "silu" | "gelu_tanh")
    and ``clamp`` ((lo, hi)) are fused epilogue expressions applied, in that
    order, to the complete sum before the output conversion.
    ``deterministic=True`` keeps every tile's sum in one fixed order (no
    stream-K tail), so repeated runs are bitwise equal."""
    import torch
    # Fast path: everything that decides the plan and the leading dimensions
    # is in the key, so a hit skips validation and plan construction.
    key = (A.shape, B.shape, Cm.shape, A.stride(), B.stride(), Cm.stride(), A.dtype, B.dtype,
           Cm.dtype, A.device, B.device, Cm.device, block_m, block_n, block_k, group_m, exact_tile,
           num_warps, num_stages, split_k, reduction_mode, persistent, num_ctas, beta,
           bias is None, activation, None if clamp is None else tuple(clamp), deterministic)
    hit = _FAST.get(key)
    if hit is None:
        m, k = A.shape
        n = B.shape[1]
        # transposed views (unit stride along rows) select the column-major layout
        a_col = A.stride(1) != 1 and A.stride(0) == 1
        b_col = B.stride(1) != 1 and B.stride(0) == 1
        ex = exact_tile
        if ex is None:
            ex = (m % block_m == 0 and n % block_n == 0 and k % block_k == 0)
        cfg = KernelConfig(m=m, n=n, k=k, block_m=block_m, block_n=block_n, block_k=block_k,
                           group_m=group_m, exact_tile=ex, num_warps=num_warps,
                           num_stages=num_stages, split_k=split_k, reduction_mode=reduction_mode,
                           persistent=persistent, num_ctas=num_ctas,
                           c_dtype="f16" if Cm.dtype == torch.float16 else "f32", beta=beta,
                           bias=bias is not None, activation=activation,
                           clamp=tuple(clamp) if clamp is not None else None,
                           a_col_major=a_col, b_col_major=b_col, deterministic=deterministic)
        plan = plan_for(cfg, Cm.device.index if Cm.is_cuda else None)
        _check_tensors(cfg, A, B, Cm)
        # the bound C entry points and the device index ride along, so a hit
        # costs a dict lookup, three data_ptr() calls and one ctypes call
        hit = (plan, A.stride(1) if a_col else A.stride(0), B.stride(1) if b_col else B.stride(0),
               Cm.stride(0), plan.workspace_bytes, _lib.tb_matmul_run, _lib.tb_matmul_run_epilogue,
               Cm.device.index)
        if len(_FAST) > 1024:
            _FAST.clear()
        _FAST[key] = hit
    plan, lda, ldb, ldc, need, run, run_epilogue, dev_index = hit
    ws_ptr, ws_bytes = 0, 0
    if need:
        if workspace is None:
            workspace = torch.empty(need, dtype=torch.uint8, device=Cm.device)
        ws_ptr, ws_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    if stream is not None:
        sp = stream.cuda_stream
    else:  # the current stream of C's device, as a raw handle
        sp = torch._C._cuda_getCurrentRawStream(dev_index)
    if bias is not None:
        if bias.dtype != torch.float32 or bias.numel() != Cm.shape[1] or not bias.is_contiguous() \
                or not bias.is_cuda:
            raise TBError(_capi.TB_ERR_INVALID_ARGUMENT, "bias must be a contiguous f32 CUDA vector of n")
        code = run_epilogue(plan._h, A.data_ptr(), lda, B.data_ptr(), ldb, Cm.data_ptr(), ldc,
                            bias.data_ptr(), ws_ptr or None, ws_bytes, sp or None)
    else:
        code = run(plan._h, A.data_ptr(), lda, B.data_ptr(), ldb, Cm.data_ptr(), ldc, ws_ptr or None,
                   ws_bytes, sp or None)
    if code:
        _check(code)
    return Cm


_FAST: dict = {}


def device_status(stream=None) -> int:
    """Synchronises and returns/clears the kernels' device status word;
    raises TBError(TB_ERR_DEVICE_TIMEOUT) when a bounded wait gave up."""
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    raw = C.c_uint32(0)
    code = _lib.tb_device_status(C.c_void_p(s.cuda_stream or None), C.byref(raw))
    _check(code)
    return raw.value
