/*
 * tb_gemm.h — C ABI of the B200-native `tb.matmul` GEMM.
 *
 * The reference (zrqnwu/mini_triton_nvgpu_v1) has no runtime library: its
 * operator surface is the MLIR op
 *
 *     tb.matmul %A, %B, %C {block_m, block_n, block_k, group_m, exact_tile}
 *
 * (include/tb/IR/TBOps.td:32-58) plus the module attributes tb.num-warps,
 * tb.requested-stages (include/tb/Analysis/TargetInfo.h:17-21), tb.split-k,
 * tb.reduction-mode, tb.persistent, tb.programs-per-tile
 * (include/tb/Analysis/ProgramMappingPlan.h:14-17) and tb.num-ctas
 * (TargetInfo.h:20). `tb-opt` lowers that op into one kernel
 * `kernel_tb_kernel_0(A, B, C)` that computes C = C_in + A·B in place
 * (lib/Transforms/LowerPipelineToNVGPU.cpp:994-999, :2507-2583).
 *
 * This header replaces that whole chain with three steps:
 *   tb_matmul_desc  — the knobs, same names and meaning as the attributes;
 *   tb_matmul_plan  — validated knobs + program mapping (replaces
 *                     verifySupportedKernelConfig, deriveProgramMappingPlan,
 *                     deriveReductionPlan, derivePersistentWorkPlan);
 *   tb_matmul_run   — one stream-ordered launch of the sm_100a kernels
 *                     (replaces the generated kernel and its launch).
 *
 * Ownership: the caller owns every device buffer and the stream. A plan owns
 * host metadata only; it is immutable after creation and may be shared by
 * threads. Every call returns a tbStatus; tb_last_error() gives the message of
 * the calling thread's last failure (messages mirror the reference's
 * diagnostics where the rule is the reference's).
 */
#ifndef TB_GEMM_H_
#define TB_GEMM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum tbStatus {
  TB_OK = 0,
  TB_ERR_INVALID_ARGUMENT = 1, /* knob or argument rejected by validation */
  TB_ERR_UNSUPPORTED = 2,      /* legal for the reference, outside this build */
  TB_ERR_CUDA = 3,             /* a CUDA runtime/driver call failed */
  TB_ERR_DEVICE_TIMEOUT = 4,   /* a bounded device-side wait gave up */
  TB_ERR_WORKSPACE = 5,        /* workspace missing or too small */
  TB_ERR_NCCL = 6              /* NCCL unavailable or a collective failed */
} tbStatus;

/* Element types (memref element types of A, B and C). */
typedef enum tbDtype { TB_F16 = 0, TB_F32 = 1, TB_BF16 = 2 } tbDtype;

/* tb.reduction-mode (ProgramMappingPlan.h:37-41). UNSET means the attribute
 * is absent, which the reference resolves to split_k_serial
 * (lib/Analysis/ProgramMappingPlan.cpp:415-418). */
typedef enum tbReductionMode {
  TB_REDUCTION_UNSET = 0,
  TB_REDUCTION_SPLIT_K_SERIAL = 1,   /* fp32 workspace + fixed-order reduction */
  TB_REDUCTION_SPLIT_K_PARALLEL = 2  /* f32 atomic accumulation into C */
} tbReductionMode;

/* Knobs of one tb.matmul. Field names follow the reference attributes. */
typedef struct tb_matmul_desc {
  int64_t m, n, k;                 /* A: m×k, B: k×n, C: m×n; TB_DIM_DYNAMIC
                                      (dynamic plans only) leaves one open */
  int64_t block_m, block_n, block_k; /* TBOps.td:42-44 */
  int64_t group_m;                 /* TBOps.td:45, default 8 */
  int32_t exact_tile;              /* TBOps.td:46, default 1 */
  int64_t num_warps;               /* "tb.num-warps" (required) */
  int64_t num_stages;              /* "tb.requested-stages" (required) */
  int64_t split_k;                 /* "tb.split-k", default 1 */
  int32_t reduction_mode;          /* "tb.reduction-mode", tbReductionMode */
  int32_t persistent;              /* "tb.persistent", default 0 */
  int64_t num_ctas;                /* "tb.num-ctas", default 1 */
  int64_t programs_per_tile;       /* "tb.programs-per-tile", 0 = absent */
  int32_t a_dtype, b_dtype;        /* must be TB_F16 */
  int32_t c_dtype;                 /* TB_F32 (reference) or TB_F16 (extension) */
  int32_t beta;                    /* 1: C = C_in + A·B (reference); 0: C = A·B */
  /* Fused epilogue expressions, applied in this order after the full sum
   * (the kinds EpiloguePlan.h:61-75 declares — LoadBias/Add, Activation,
   * Clamp, Convert — which the reference never emits):
   *   v = A·B + beta·C_in; v += bias[col]; v = act(v); v = clamp(v, lo, hi);
   *   C = convert(v, c_dtype).
   * Not available with split_k_parallel (partials are summed in C). */
  int32_t bias;                    /* 1: runs take a length-n f32 bias (per column) */
  int32_t activation;              /* tbActivation */
  int32_t clamp;                   /* 1: clamp to [clamp_lo, clamp_hi] */
  float clamp_lo, clamp_hi;
  /* Operand storage (the reference takes row-major A and B only; these select
   * the transposed layouts, read directly by TMA/UMMA without a copy):
   * a_col_major: A is m × k column-major, lda >= m (A^T row-major);
   * b_col_major: B is k × n column-major, ldb >= k (B^T row-major). */
  int32_t a_col_major, b_col_major;
  /* 1: bitwise-repeatable runs. By default (0) a plain f32-output plan whose
   * work items leave the last wave of SMs partly idle (after at least one
   * whole wave) spreads the K work of its last items evenly over the SMs
   * (a stream-K tail: partial tiles reduce-added into C; results within the
   * f32 tolerance, summation order not fixed). No counterpart in the
   * reference. */
  int32_t deterministic;
} tb_matmul_desc;

/* An open ("?") problem dim, for tb_matmul_plan_create_dynamic; the value
 * MLIR gives a dynamic memref dim (ShapedType::kDynamic = INT64_MIN). */
#define TB_DIM_DYNAMIC INT64_MIN

typedef enum tbActivation {
  TB_ACT_NONE = 0,
  TB_ACT_RELU = 1,
  TB_ACT_SILU = 2,      /* v · sigmoid(v) */
  TB_ACT_GELU_TANH = 3  /* tanh approximation of GELU (Hendrycks & Gimpel) */
} tbActivation;

typedef struct tb_matmul_plan tb_matmul_plan;

/* Work assigned to one program id (LowerPipelineToNVGPU.cpp:279-357). */
typedef struct tb_program_work {
  int64_t tile_m, tile_n, split_part;
  int64_t k_tile_begin, k_tile_count; /* in block_k tiles */
} tb_program_work;

/* Fills the defaults the reference applies to absent attributes:
 * group_m=8, exact_tile=1, split_k=1, num_ctas=1, persistent=0,
 * f16·f16→f32, beta=1. Replaces the attribute defaults of TBOps.td:45-46 and
 * ProgramMappingPlan.cpp:331-340. */
tbStatus tb_matmul_desc_init(tb_matmul_desc* desc);

/* Validates `desc` and derives the program mapping. `device` < 0 plans for a
 * B200 (148 SMs) without touching CUDA, for host-only use; otherwise the SM
 * count of `device` is queried. Replaces verifySupportedKernelConfig
 * (lib/Analysis/KernelConfig.cpp:202-246), deriveProgramMappingPlan
 * (lib/Analysis/ProgramMappingPlan.cpp:329-458), deriveReductionPlan
 * (lib/Analysis/ReductionPlan.cpp:137-192), derivePersistentWorkPlan
 * (lib/Analysis/PersistentWorkPlan.cpp:91-131) and the mapping checks of
 * validateLoweringContract (LowerPipelineToNVGPU.cpp:678-815). */
tbStatus tb_matmul_plan_create(const tb_matmul_desc* desc, int device,
                               tb_matmul_plan** plan);

tbStatus tb_matmul_plan_destroy(tb_matmul_plan* plan);

/* Bytes of device workspace `tb_matmul_run` needs (nonzero only for
 * split_k_serial, which keeps S fp32 partials of C). Replaces the global
 * scratch of ReductionPlan (scratchBytes, ReductionPlan.cpp:164-166). */
size_t tb_matmul_workspace_bytes(const tb_matmul_plan* plan);

/* Writes a JSON object describing the plan (the reference's structural plan
 * facts — mapping_kind, swizzle_kind, total_programs, reduction kind,
 * resident_programs, warp_grid, … — and this build's launch facts) into buf.
 * Replaces the plan attributes tb-opt prints (checked by the reference's
 * test/Transforms FileCheck tests). Returns TB_ERR_INVALID_ARGUMENT
 * when len is too small; *needed receives the size including the NUL. */
tbStatus tb_matmul_plan_describe(const tb_matmul_plan* plan, char* buf,
                                 size_t len, size_t* needed);

/* The work of program `pid` (0 <= pid < total_programs). Host restatement of
 * buildProgramWorkAssignment + buildSplitKGroupActivePredicate
 * (LowerPipelineToNVGPU.cpp:279-357); the device kernels use the same code. */
tbStatus tb_matmul_program_work(const tb_matmul_plan* plan, int64_t pid,
                                tb_program_work* work);

/* Runs C = beta·C_in + A·B in place on `stream` (a cudaStream_t; NULL = the
 * legacy default stream). A is m×k row-major with row stride lda (elements),
 * B is k×n row-major with stride ldb, C is m×n row-major with stride ldc, of
 * c_dtype. TMA reads rows with 16-byte strides from 16-byte aligned bases;
 * when the plan's row length is not a multiple of 8 elements, operands that
 * break that rule are first copied, zero-padded, into the workspace.
 * `workspace` must hold tb_matmul_workspace_bytes(plan) bytes (may be NULL
 * when that is 0). Replaces kernel_tb_kernel_0(A, B, C) and its launch
 * (LowerPipelineToNVGPU.cpp:2678-2711; tools/bench_stage1_fair.py:67-74). */
tbStatus tb_matmul_run(const tb_matmul_plan* plan, const void* A, int64_t lda,
                       const void* B, int64_t ldb, void* C, int64_t ldc,
                       void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free variant of tb_matmul_run. It has no counterpart in the
 * reference. It is for callers that must not allocate device memory while
 * they run — an inference engine's plugin that executes inside a memory plan
 * fixed ahead of time, a process whose device memory is reserved up front, or
 * code on a path where an allocator call (and the synchronisation it can
 * bring) is not allowed. Those callers still pass A, B and C.
 *
 * Scratch (the split_k_serial partial planes) comes from one fixed 16 MiB
 * (16777216-byte) array inside the library, which every GPU that loads the
 * library holds until the process exits; a plan needing more returns
 * TB_ERR_WORKSPACE without launching. No cudaMalloc/cudaFree or other
 * allocating routine is called. The first call on a device looks the array's
 * device address up (once per device); make that first call before any
 * stream capture. The address is kept for the life of the process: after a
 * cudaDeviceReset on that device it is stale, so do not call this entry
 * point on a device that was reset. All calls share the one array: two calls whose kernels
 * overlap on the GPU (different streams, or different host threads) race on
 * it. Nothing in it needs to start at zero — each call writes every partial
 * before it reads it. */
tbStatus tb_matmul_run_no_alloc(const tb_matmul_plan* plan, const void* A,
                                int64_t lda, const void* B, int64_t ldb,
                                void* C, int64_t ldc, void* stream);

/* ---- N-column sharded runs (one process per GPU, no collective) ----
 * The reference is single-GPU; its op splits along N with no exchange. For a
 * plan of the whole m × n × k problem, rank r of `world` owns columns
 * [col0, col0 + ncols) of B and C: whole block_n program tiles, balanced
 * over the ranks. A is replicated. Each rank runs the op on its slice, a
 * tb.matmul of m × ncols × k with the plan's knobs; every element gets the
 * value the one-GPU run gives it (same program tile, same K order).
 * Replaces, per rank, kernel_tb_kernel_0(A, B, C) on the rank's columns
 * (LowerPipelineToNVGPU.cpp:2678-2711). */
tbStatus tb_matmul_nshard_columns(const tb_matmul_plan* plan, int rank, int world,
                                  int64_t* col0, int64_t* ncols);
/* Workspace bytes of this rank's slice run (0 unless split_k_serial or a
 * repacked operand needs some). */
tbStatus tb_matmul_nshard_workspace_bytes(const tb_matmul_plan* plan, int rank,
                                          int world, size_t* bytes);
/* B_cols / C_cols address column col0 of B and C (row strides ldb, ldc):
 * either this rank's own k × ncols and m × ncols slices, or B + col0 and
 * C + col0 of full matrices. bias_cols: the slice's ncols bias values
 * (NULL unless desc.bias). Row-major B only. A rank with no columns
 * (world > column tiles) returns TB_OK without launching. */
tbStatus tb_matmul_run_nshard(const tb_matmul_plan* plan, int rank, int world,
                              const void* A, int64_t lda, const void* B_cols,
                              int64_t ldb, void* C_cols, int64_t ldc,
                              const float* bias_cols, void* workspace,
                              size_t workspace_bytes, void* stream);

/* ---- K-sharded runs over NVLink peer memory (one process per GPU) ----
 * The reference is single-GPU; its split-K reduction (ReductionPlan.cpp:137-192,
 * atomic executor LowerPipelineToNVGPU.cpp:1862-1912) becomes a cross-GPU
 * reduce-scatter here. Rank r owns rows [r·m/W, (r+1)·m/W) of C and runs the
 * plan of its K slice (m × n × k_r, f32 C, split_k_parallel or no split).
 * The GEMM reduces its split parts into a private staging buffer; one more
 * kernel adds each staged element once into its owner's rows over NVLink
 * (peer-mapped memory), between two device-side barriers, so C_rows ends as
 * C_rows_in + Σ_r A_r·B_r on every owner. */
typedef struct tb_peer_handle {
  unsigned char rows_ipc[64];  /* CUDA IPC handle of the allocation holding C rows */
  int64_t rows_offset;         /* offset of the C rows inside that allocation */
  unsigned char flags_ipc[64]; /* CUDA IPC handle of the rank's barrier flags */
} tb_peer_handle;
typedef struct tb_peer_comm tb_peer_comm;

/* my_rows: this rank's rows_per_rank × n f32 rows of C (row stride ldc,
 * cudaMalloc'd memory, e.g. a torch tensor). Fills *my_handle, which every
 * rank must pass to tb_peer_comm_connect in rank order. */
tbStatus tb_peer_comm_create(int rank, int world, void* my_rows,
                             int64_t rows_per_rank, int64_t n, int64_t ldc,
                             tb_peer_comm** comm, tb_peer_handle* my_handle);
tbStatus tb_peer_comm_connect(tb_peer_comm* comm, const tb_peer_handle* all);
/* Stream-ordered barrier across the ranks (bounded device-side wait). */
tbStatus tb_peer_barrier(tb_peer_comm* comm, void* stream);
/* K-sharded GEMM, then barrier → add into the owners' rows → barrier.
 * Collective: every rank calls it with the same plan shape. */
tbStatus tb_matmul_run_kshard_peer(const tb_matmul_plan* plan, tb_peer_comm* comm,
                                   const void* A, int64_t lda, const void* B,
                                   int64_t ldb, void* stream);
/* Synchronises `stream`; TB_ERR_DEVICE_TIMEOUT if a barrier wait gave up.
 * A timed-out comm is failed for good: its later barrier and scatter kernels
 * return at once (so the other ranks time out too), and runs and barriers on
 * it are refused; destroy it and create a new one. */
tbStatus tb_peer_comm_status(tb_peer_comm* comm, void* stream, uint32_t* raw);
tbStatus tb_peer_comm_destroy(tb_peer_comm* comm);

/* ---- K-sharded runs with an NCCL reduce-scatter (one process per GPU) ----
 * The same partition as tb_matmul_run_kshard_peer, with the cross-GPU sum
 * done by ncclReduceScatter: rank r runs its K slice (plan: m × n × k_r, f32
 * C, any reduction mode) into an f32 staging copy of C held in `workspace`
 * (its own rows seeded with C_in when beta = 1, the rest zero), then the
 * staging buffers are reduce-scattered so C_rows (rank r's m/W rows, row
 * stride ldc) ends as C_rows_in + Σ_r A_r·B_r. Replaces the split-K reduction
 * of ReductionPlan.cpp:137-192 / LowerPipelineToNVGPU.cpp:1862-1912 across
 * GPUs. NCCL is loaded at run time (libnccl.so.2); TB_ERR_NCCL when absent.
 * The communicator is this library's (tb_nccl_comm_create from a unique id
 * that rank 0 makes and the caller distributes). */
typedef struct tb_nccl_comm tb_nccl_comm;
tbStatus tb_nccl_unique_id(unsigned char id[128]);
tbStatus tb_nccl_comm_create(int rank, int world, const unsigned char id[128],
                             tb_nccl_comm** comm);
tbStatus tb_nccl_comm_destroy(tb_nccl_comm* comm);
/* Workspace bytes of tb_matmul_run_kshard_nccl (staging + plan workspace). */
size_t tb_matmul_kshard_nccl_workspace_bytes(const tb_matmul_plan* plan, int world,
                                             int64_t ldc);
/* Collective: every rank calls it with plans of the same m × n. */
tbStatus tb_matmul_run_kshard_nccl(const tb_matmul_plan* plan, tb_nccl_comm* comm,
                                   const void* A, int64_t lda, const void* B,
                                   int64_t ldb, void* C_rows, int64_t ldc,
                                   void* workspace, size_t workspace_bytes,
                                   void* stream);

/* tb_matmul_run with the bias of a plan made with desc.bias = 1 (`bias`:
 * n f32 values, one per column of C; NULL when the plan has no bias). */
tbStatus tb_matmul_run_epilogue(const tb_matmul_plan* plan, const void* A,
                                int64_t lda, const void* B, int64_t ldb,
                                void* C, int64_t ldc, const float* bias,
                                void* workspace, size_t workspace_bytes,
                                void* stream);

/* ---- Dynamic shapes ----
 * The reference accepts static memref shapes only (deriveSourceKernelConfig,
 * lib/Analysis/KernelConfig.cpp:98-103 — tb_matmul_plan_create rejects a
 * TB_DIM_DYNAMIC dim with the same message). A dynamic plan validates its
 * knobs once; each run names m, n and k, which must equal the desc's static
 * dims where those are given. The concrete per-shape plan (mapping, hardware
 * tile, grid, workspace) is derived on a shape's first run and cached inside
 * the plan (thread-safe; bounded to 256 shapes). Static-plan entry points
 * (tb_matmul_run, tb_matmul_run_no_alloc, tb_matmul_program_work,
 * tb_matmul_run_kshard_peer) reject a dynamic plan; tb_matmul_workspace_bytes
 * returns 0 for it. No counterpart in the reference. */
tbStatus tb_matmul_plan_create_dynamic(const tb_matmul_desc* desc, int device,
                                       tb_matmul_plan** plan);
/* Workspace bytes of one shape of a dynamic plan (monotone in m, n and k). */
tbStatus tb_matmul_workspace_bytes_dynamic(const tb_matmul_plan* plan, int64_t m,
                                           int64_t n, int64_t k, size_t* bytes);
/* tb_matmul_run_epilogue for shape m×n×k (bias: NULL unless desc.bias). */
tbStatus tb_matmul_run_dynamic(const tb_matmul_plan* plan, int64_t m, int64_t n,
                               int64_t k, const void* A, int64_t lda, const void* B,
                               int64_t ldb, void* C, int64_t ldc, const float* bias,
                               void* workspace, size_t workspace_bytes, void* stream);
/* A new static plan equal to the dynamic plan's concrete plan for m×n×k
 * (destroy it with tb_matmul_plan_destroy). */
tbStatus tb_matmul_plan_for_shape(const tb_matmul_plan* plan, int64_t m, int64_t n,
                                  int64_t k, tb_matmul_plan** shape_plan);

/* One-call convenience: desc → plan → run → destroy. */
tbStatus tb_matmul(const tb_matmul_desc* desc, const void* A, int64_t lda,
                   const void* B, int64_t ldb, void* C, int64_t ldc,
                   void* workspace, size_t workspace_bytes, void* stream);

/* Reads and clears the device status word the kernels set when a bounded
 * wait gives up (TB_ERR_DEVICE_TIMEOUT) — synchronises `stream`. The reference
 * has no device-side failure detection; this has no counterpart there. */
tbStatus tb_device_status(void* stream, uint32_t* raw_status);

/* Failure-detection self-test: launches one warp that waits, bounded by
 * `budget_cycles` SM clocks (at most 2e9), on an mbarrier nothing arrives on,
 * using the GEMM kernels' bounded-wait and status-recording code. Afterwards
 * tb_device_status() reports TB_ERR_DEVICE_TIMEOUT (site 5) and the context
 * stays usable. No counterpart in the reference. */
tbStatus tb_selftest_bounded_wait(void* stream, uint64_t budget_cycles);

/* Message of the calling thread's most recent failure ("" if none). */
const char* tb_last_error(void);

/* Library version string. */
const char* tb_version(void);

#ifdef __cplusplus
}
#endif

#endif /* TB_GEMM_H_ */
