// tb_peer.cu — K-sharded tb.matmul with the reduce-scatter fused into the
// GEMM, over NVLink peer memory (one process per GPU).
//
// Rank r holds A[:, K_r] and B[K_r, :] and owns rows [r·m/W, (r+1)·m/W) of C.
// Every rank's GEMM epilogue reduce-adds each finished f32 [32 × 32] chunk
// straight into the owning rank's C rows with a TMA reduction through a
// peer-mapped tensor map, so the partial sums never make a round trip
// through a workspace or a separate collective. This is the reference's
// split-K reduction (ReductionPlan.cpp:137-192, atomic executor
// LowerPipelineToNVGPU.cpp:1862-1912) with the split parts on different GPUs.
//
// Ordering between ranks uses a flag word per rank (library-owned device
// memory, shared through CUDA IPC): a barrier kernel adds 1 to every rank's
// flag (system-scope atomics over NVLink) and waits, bounded, until its own
// flag reaches world × phase. A run is barrier → GEMM → barrier, so no rank
// adds into C rows an owner is still using, and every owner sees all
// additions when its run completes on its stream.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

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
  unsigned int* flag_base;        // own allocation: [flag, status, …]
  unsigned int* flags[kMaxWorld];
  void* flag_opened[kMaxWorld];
  unsigned int phase;
  bool connected;
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
  if (plan->desc.m != c->rows_per_rank * c->world || plan->desc.n != c->n)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "plan m must be world * rows_per_rank and n the comm's n");
  tbStatus st = tb_peer_barrier(c, stream);
  if (st != TB_OK) return st;
  st = tb_launch_peer_reduce(plan, A, lda, B, ldb, c->rows, c->world, c->rows_per_rank, c->ldc, stream);
  if (st != TB_OK) return st;
  return tb_peer_barrier(c, stream);
}

extern "C" tbStatus tb_peer_comm_status(tb_peer_comm* c, void* stream, uint32_t* raw) {
  if (!c) return tb_fail(TB_ERR_INVALID_ARGUMENT, "comm must not be NULL");
  cudaError_t e = cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail("cudaStreamSynchronize", e);
  unsigned int v = 0;
  e = cudaMemcpy(&v, c->flag_base + 1, sizeof(v), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail("cudaMemcpy(status)", e);
  if (raw) *raw = v;
  if (v) return tb_fail(TB_ERR_DEVICE_TIMEOUT, "a peer barrier wait timed out");
  return TB_OK;
}

extern "C" tbStatus tb_peer_comm_destroy(tb_peer_comm* c) {
  if (!c) return TB_OK;
  for (int r = 0; r < kMaxWorld; ++r) {
    if (c->opened[r]) cudaIpcCloseMemHandle(c->opened[r]);
    if (c->flag_opened[r]) cudaIpcCloseMemHandle(c->flag_opened[r]);
  }
  cudaFree(c->flag_base);
  delete c;
  return TB_OK;
}
