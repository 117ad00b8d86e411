// tb_peer.cu — K-sharded tb.matmul with the reduce-scatter fused into the
// GEMM, over NVLink peer memory (one process per GPU).
//
// Rank r holds A[:, K_r] and B[K_r, :] and owns rows [r·m/W, (r+1)·m/W) of C.
// A run is two kernels: the GEMM of the rank's K slice, whose split parts
// reduce-add (TMA, at L2) into a private m × n staging buffer, and a scatter
// kernel that adds every staged element once into its owner's rows over
// NVLink and re-zeroes staging, with the opening and closing cross-rank
// barriers inside it (one NVLink transfer per element instead of one per
// split part, and no separate collective). This is the reference's
// split-K reduction (ReductionPlan.cpp:137-192, atomic executor
// LowerPipelineToNVGPU.cpp:1862-1912) with the split parts on different GPUs.
//
// Ordering between ranks uses a flag word per rank (library-owned device
// memory, shared through CUDA IPC): a barrier kernel adds 1 to every rank's
// flag (system-scope atomics over NVLink) and waits, bounded, until its own
// flag reaches world × phase. The scatter opens with one such barrier (no
// rank adds into rows an owner is still using) and closes with another
// (every owner has all additions when its run completes on its stream).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <new>
#include <string>

#include "tb_plan.h"

namespace {

constexpr int kMaxWorld = 8;
constexpr long long kBarrierBudgetCycles = 2000000000LL;  // ≈1 s

struct FlagArgs {
  unsigned int* flags[kMaxWorld];  // every rank's flag word (peer-mapped)
  unsigned int* status;            // this rank's status word (0 = ok)
  int world;
  int rank;
  unsigned int target;
};

// thread s < world signals rank s; thread 0 then waits for its own flag.
__global__ void tb_peer_barrier_kernel(FlagArgs a) {
  // A comm whose earlier wait timed out is poisoned: the ranks' flag counts
  // no longer agree, so a barrier could pass early. Do nothing; the ranks
  // still waiting on this one time out and poison their comms in turn.
  if (*(volatile unsigned int*)a.status != 0) return;
  const int t = threadIdx.x;
  if (t < a.world) {
    __threadfence_system();
    atomicAdd_system(a.flags[t], 1u);
  }
  __syncthreads();
  if (t == 0) {
    volatile unsigned int* mine = a.flags[a.rank];
    const long long t0 = clock64();
    while ((int)(*mine - a.target) < 0) {
      if (clock64() - t0 > kBarrierBudgetCycles) {
        atomicCAS(a.status, 0u, (unsigned)TB_ERR_DEVICE_TIMEOUT);
        break;
      }
      __nanosleep(64);
    }
    __threadfence_system();
  }
}

// Sends this rank's locally reduced partial C (staging, m × n, L2-resident)
// to the owners: element (r, c) is added to rank r / rows_per_rank's row
// r % rows_per_rank (vector f32 atomics, over NVLink for peers), and staging is
// zeroed for the next run. The last block to finish then performs the
// closing barrier: it signals every rank and waits (bounded) for all signals.
struct ScatterArgs {
  float* staging;
  float* rows[kMaxWorld];
  unsigned int* flags[kMaxWorld];
  unsigned int* status;
  unsigned int* done;  // block-completion counter (own memory, starts at 0)
  int64_t n, ldc;
  int rows_per_rank, world, rank;
  int bulk;  // ldc == n: owner rows are contiguous, move 16 KB chunks with bulk reductions
  unsigned int open_target, target;
};

__device__ __forceinline__ void wait_flag(const ScatterArgs& a, unsigned int target) {
  volatile unsigned int* mine = a.flags[a.rank];
  const long long t0 = clock64();
  while ((int)(*mine - target) < 0) {
    if (clock64() - t0 > kBarrierBudgetCycles) {
      atomicCAS(a.status, 0u, (unsigned)TB_ERR_DEVICE_TIMEOUT);
      break;
    }
    __nanosleep(64);
  }
  __threadfence_system();
}

__global__ void __launch_bounds__(256) tb_peer_scatter_kernel(ScatterArgs a) {
  if (*(volatile unsigned int*)a.status != 0) return;  // poisoned comm (see the barrier kernel)
  // Opening barrier: this rank's stream has reached the scatter, so its own
  // rows are free to receive; tell every rank, then wait until all ranks are.
  if (blockIdx.x == 0 && threadIdx.x == 0)
    for (int s = 0; s < a.world; ++s) atomicAdd_system(a.flags[s], 1u);
  // Launched as a programmatic dependent of the GEMM: staging is complete
  // only after this wait.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) wait_flag(a, a.open_target);
  __syncthreads();
  const int64_t nvec = (int64_t)a.rows_per_rank * a.world * a.n / 4;
  float4* st = reinterpret_cast<float4*>(a.staging);
  if (a.bulk) {
    // chunk of 1024 float4 (16 KB): one bulk f32 add into the owner's rows
    __shared__ __align__(128) float4 chunk[1024];
    const int64_t per_owner = (int64_t)a.rows_per_rank * a.n / 4;  // multiple of 1024
    for (int64_t c0 = (int64_t)blockIdx.x * 1024; c0 < nvec; c0 += (int64_t)gridDim.x * 1024) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t i = c0 + u * 256 + threadIdx.x;
        chunk[u * 256 + threadIdx.x] = st[i];
        st[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncthreads();
      if (threadIdx.x == 0) {
        const int owner = (int)(c0 / per_owner);
        float4* dst = reinterpret_cast<float4*>(a.rows[owner]) + (c0 - owner * per_owner);
        asm volatile(
            "cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(dst),
            "r"(static_cast<uint32_t>(__cvta_generic_to_shared(chunk))), "r"(16384u)
            : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        // The bulk add ran in the async proxy: order it before this thread's
        // generic-proxy flag and counter atomics that publish completion.
        asm volatile("fence.proxy.async.global;" ::: "memory");
      }
      __syncthreads();
    }
  } else
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nvec;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i * 4;
    const int64_t r = e / a.n, c = e % a.n;
    const float4 v = st[i];
    st[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    const int owner = (int)(r / a.rows_per_rank);
    float* dst = a.rows[owner] + (r - (int64_t)owner * a.rows_per_rank) * a.ldc + c;
    atomicAdd(reinterpret_cast<float4*>(dst), v);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned int prev = atomicAdd(a.done, 1u);
    if (prev == gridDim.x - 1) {
      *a.done = 0;
      for (int s = 0; s < a.world; ++s) atomicAdd_system(a.flags[s], 1u);
      wait_flag(a, a.target);
    }
  }
}

PFN_cuMemGetAddressRange_v3020 g_range = nullptr;
std::once_flag g_range_once;

tbStatus cuda_fail(const char* what, cudaError_t e) {
  return tb_fail(TB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

struct tb_peer_comm {
  int rank, world, device;
  int64_t rows_per_rank, n, ldc;
  void* rows[kMaxWorld];          // C rows of every rank (own pointer for self)
  void* opened[kMaxWorld];        // IPC mappings to close (rows bases)
  unsigned int* flag_base;        // own allocation: [flag, status, done, …]
  float* staging;                 // m × n f32, locally reduced partial (zero between runs)
  unsigned int* flags[kMaxWorld];
  void* flag_opened[kMaxWorld];
  unsigned int phase;
  bool connected;
  bool failed;  // a barrier wait timed out: the flag counts disagree, runs are refused
};

extern "C" tbStatus tb_peer_comm_create(int rank, int world, void* my_rows, int64_t rows_per_rank,
                                        int64_t n, int64_t ldc, tb_peer_comm** out,
                                        tb_peer_handle* my_handle) {
  tb_clear_error();
  if (!out || !my_handle || !my_rows)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "comm, handle and C rows must not be NULL");
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "need 1 <= world <= 8 and 0 <= rank < world");
  if (rows_per_rank <= 0 || n <= 0 || ldc < n)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "rows_per_rank, n must be positive and ldc >= n");
  std::call_once(g_range_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  });
  if (!g_range) return tb_fail(TB_ERR_CUDA, "cuMemGetAddressRange unavailable");
  tb_peer_comm* c = new (std::nothrow) tb_peer_comm();
  if (!c) return tb_fail(TB_ERR_INVALID_ARGUMENT, "out of host memory");
  c->rank = rank;
  c->world = world;
  c->rows_per_rank = rows_per_rank;
  c->n = n;
  c->ldc = ldc;
  cudaGetDevice(&c->device);
  cudaError_t e = cudaMalloc(&c->flag_base, 256);
  if (e != cudaSuccess) { delete c; return cuda_fail("cudaMalloc(flags)", e); }
  e = cudaMemset(c->flag_base, 0, 256);
  std::memset(my_handle, 0, sizeof(*my_handle));
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->flag_base);
  if (e != cudaSuccess) { cudaFree(c->flag_base); delete c; return cuda_fail("flags IPC export", e); }
  std::memcpy(my_handle->flags_ipc, &h, sizeof(h));
  // C rows may live inside a larger allocation (a caching allocator block):
  // export the allocation and the offset into it.
  CUdeviceptr base = 0;
  size_t size = 0;
  if (g_range(&base, &size, (CUdeviceptr)my_rows) != CUDA_SUCCESS) {
    cudaFree(c->flag_base);
    delete c;
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "C rows are not device memory from cudaMalloc");
  }
  e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) { cudaFree(c->flag_base); delete c; return cuda_fail("C rows IPC export", e); }
  std::memcpy(my_handle->rows_ipc, &h, sizeof(h));
  my_handle->rows_offset = (int64_t)((CUdeviceptr)my_rows - base);
  const size_t stage_bytes = (size_t)rows_per_rank * world * n * sizeof(float);
  e = cudaMalloc(&c->staging, stage_bytes);
  if (e == cudaSuccess) e = cudaMemset(c->staging, 0, stage_bytes);
  if (e != cudaSuccess) { cudaFree(c->flag_base); delete c; return cuda_fail("cudaMalloc(staging)", e); }
  c->rows[rank] = my_rows;
  c->flags[rank] = c->flag_base;
  *out = c;
  return TB_OK;
}

extern "C" tbStatus tb_peer_comm_connect(tb_peer_comm* c, const tb_peer_handle* all) {
  tb_clear_error();
  if (!c || !all) return tb_fail(TB_ERR_INVALID_ARGUMENT, "comm and handles must not be NULL");
  if (c->connected) return tb_fail(TB_ERR_INVALID_ARGUMENT, "comm is already connected");
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, all[r].rows_ipc, sizeof(h));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail("C rows IPC import", e);
    c->opened[r] = p;
    c->rows[r] = static_cast<char*>(p) + all[r].rows_offset;
    std::memcpy(&h, all[r].flags_ipc, sizeof(h));
    e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail("flags IPC import", e);
    c->flag_opened[r] = p;
    c->flags[r] = static_cast<unsigned int*>(p);
  }
  c->connected = true;
  return TB_OK;
}

extern "C" tbStatus tb_peer_barrier(tb_peer_comm* c, void* stream) {
  if (!c || !c->connected) return tb_fail(TB_ERR_INVALID_ARGUMENT, "comm is not connected");
  if (c->failed)
    return tb_fail(TB_ERR_DEVICE_TIMEOUT, "this comm is failed: a peer barrier wait timed out earlier");
  FlagArgs a;
  std::memset(&a, 0, sizeof(a));
  for (int r = 0; r < c->world; ++r) a.flags[r] = c->flags[r];
  a.status = c->flag_base + 1;
  a.world = c->world;
  a.rank = c->rank;
  c->phase += 1;
  a.target = (unsigned int)c->world * c->phase;
  tb_peer_barrier_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TB_OK : cuda_fail("tb_peer_barrier launch", e);
}

extern "C" tbStatus tb_matmul_run_kshard_peer(const tb_matmul_plan* plan, tb_peer_comm* c,
                                              const void* A, int64_t lda, const void* B,
                                              int64_t ldb, void* stream) {
  tb_clear_error();
  if (!plan || !c || !c->connected)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "plan and a connected comm are required");
  if (c->failed)
    return tb_fail(TB_ERR_DEVICE_TIMEOUT, "this comm is failed: a peer barrier wait timed out earlier");
  if (plan->dynamic)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "K-sharded runs take a plan with static dims");
  if (plan->desc.m != c->rows_per_rank * c->world || plan->desc.n != c->n)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "plan m must be world * rows_per_rank and n the comm's n");
  if (plan->epilogue == kEpiWorkspace)
    return tb_fail(TB_ERR_UNSUPPORTED, "K-sharded runs reduce split parts with split_k_parallel, "
                                       "not split_k_serial");
  if (plan->desc.bias || plan->desc.activation != TB_ACT_NONE || plan->desc.clamp)
    return tb_fail(TB_ERR_UNSUPPORTED, "K-sharded runs sum partials across GPUs: fused epilogue "
                                       "expressions are not available");
  if (plan->desc.c_dtype != TB_F32 || c->n % 4 != 0 || c->ldc % 4 != 0)
    return tb_fail(TB_ERR_UNSUPPORTED, "K-sharded runs need f32 C and n, ldc multiples of 4");
  // 1. local GEMM of this K slice (touches only this rank's private staging,
  //    so it needs no barrier); split parts reduce into zeroed staging
  tbStatus st;
  tb_matmul_plan local = *plan;
  local.desc.beta = 1;  // staging starts at zero: C_in + Σ = Σ, and no memset
  st = tb_launch(&local, A, lda, B, ldb, c->staging, c->n, nullptr, 0, stream);
  if (st != TB_OK) return st;
  // 2. opening barrier, one NVLink transfer per element to its owner, closing
  //    barrier — one kernel, launched to overlap the GEMM's tail
  ScatterArgs a;
  std::memset(&a, 0, sizeof(a));
  a.staging = c->staging;
  for (int r = 0; r < c->world; ++r) {
    a.rows[r] = static_cast<float*>(c->rows[r]);
    a.flags[r] = c->flags[r];
  }
  a.status = c->flag_base + 1;
  a.done = c->flag_base + 2;
  a.n = c->n;
  a.ldc = c->ldc;
  a.rows_per_rank = (int)c->rows_per_rank;
  a.world = c->world;
  a.rank = c->rank;
  a.bulk = c->ldc == c->n && (c->rows_per_rank * c->n) % 4096 == 0;
  c->phase += 1;
  a.open_target = (unsigned int)c->world * c->phase;
  c->phase += 1;
  a.target = (unsigned int)c->world * c->phase;
  int dev_sms = 148;
  cudaDeviceGetAttribute(&dev_sms, cudaDevAttrMultiProcessorCount, c->device);
  const int64_t nvec = c->rows_per_rank * c->world * c->n / 4;
  int blocks = a.bulk ? (int)std::min<int64_t>(nvec / 1024, (int64_t)dev_sms * 2)
                      : (int)std::min<int64_t>((nvec + 255) / 256, (int64_t)dev_sms * 4);
  if (blocks < 1) blocks = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, tb_peer_scatter_kernel, a);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? TB_OK : cuda_fail("tb_peer_scatter launch", e);
}

extern "C" tbStatus tb_peer_comm_status(tb_peer_comm* c, void* stream, uint32_t* raw) {
  if (!c) return tb_fail(TB_ERR_INVALID_ARGUMENT, "comm must not be NULL");
  cudaError_t e = cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail("cudaStreamSynchronize", e);
  unsigned int v = 0;
  e = cudaMemcpy(&v, c->flag_base + 1, sizeof(v), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail("cudaMemcpy(status)", e);
  if (raw) *raw = v;
  if (v) {
    c->failed = true;
    return tb_fail(TB_ERR_DEVICE_TIMEOUT,
                   "a peer barrier wait timed out; this comm is failed (destroy it and build a new one)");
  }
  return TB_OK;
}

extern "C" tbStatus tb_peer_comm_destroy(tb_peer_comm* c) {
  if (!c) return TB_OK;
  for (int r = 0; r < kMaxWorld; ++r) {
    if (c->opened[r]) cudaIpcCloseMemHandle(c->opened[r]);
    if (c->flag_opened[r]) cudaIpcCloseMemHandle(c->flag_opened[r]);
  }
  cudaFree(c->flag_base);
  cudaFree(c->staging);
  delete c;
  return TB_OK;
}
