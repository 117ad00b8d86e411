// tb_nccl.cpp — K-sharded tb.matmul with the reduce-scatter done by NCCL.
//
// The reference is single-GPU; its split-K reduction (ReductionPlan.cpp:137-192,
// atomic executor LowerPipelineToNVGPU.cpp:1862-1912) becomes, across GPUs, a
// reduce-scatter of per-rank partial products. This is the library-collective
// form of that step (tb_matmul_run_kshard_peer in tb_peer.cu is the fused
// NVLink form): each rank runs its K slice into an f32 staging copy of C
// (its own rows seeded with C_in, the rest zero), then ncclReduceScatter sums
// the staging buffers and leaves each rank its rows.
//
// NCCL is opened at run time (dlopen of libnccl.so.2, which is the copy the
// process already loaded if torch or the caller brought one), so the library
// links without it and only these entry points need it.

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>

#include "tb_plan.h"

namespace {

struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*reduce_scatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                                 cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      api.why = std::string("libnccl.so.2 not found: ") + dlerror();
      return;
    }
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.reduce_scatter = reinterpret_cast<decltype(api.reduce_scatter)>(dlsym(h, "ncclReduceScatter"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.reduce_scatter &&
             api.error_string;
    if (!api.ok) api.why = "libnccl.so.2 lacks an entry point this library uses";
  });
  return api;
}

tbStatus nccl_fail(const char* what, ncclResult_t r) {
  return tb_fail(TB_ERR_NCCL, std::string(what) + ": " + nccl().error_string(r));
}

tbStatus cuda_fail(const char* what, cudaError_t e) {
  return tb_fail(TB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace

struct tb_nccl_comm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
};

extern "C" tbStatus tb_nccl_unique_id(unsigned char id[128]) {
  tb_clear_error();
  if (!id) return tb_fail(TB_ERR_INVALID_ARGUMENT, "id must not be NULL");
  if (!nccl().ok) return tb_fail(TB_ERR_NCCL, nccl().why);
  ncclUniqueId u;
  const ncclResult_t r = nccl().get_unique_id(&u);
  if (r != ncclSuccess) return nccl_fail("ncclGetUniqueId", r);
  static_assert(sizeof(u) == 128, "ncclUniqueId is 128 bytes");
  std::memcpy(id, &u, sizeof(u));
  return TB_OK;
}

extern "C" tbStatus tb_nccl_comm_create(int rank, int world, const unsigned char id[128],
                                        tb_nccl_comm** out) {
  tb_clear_error();
  if (!out || !id) return tb_fail(TB_ERR_INVALID_ARGUMENT, "id and comm must not be NULL");
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "rank must be in [0, world)");
  if (!nccl().ok) return tb_fail(TB_ERR_NCCL, nccl().why);
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  auto* c = new (std::nothrow) tb_nccl_comm();
  if (!c) return tb_fail(TB_ERR_INVALID_ARGUMENT, "out of host memory");
  const ncclResult_t r = nccl().comm_init_rank(&c->comm, world, u, rank);
  if (r != ncclSuccess) {
    delete c;
    return nccl_fail("ncclCommInitRank", r);
  }
  c->rank = rank;
  c->world = world;
  *out = c;
  return TB_OK;
}

extern "C" tbStatus tb_nccl_comm_destroy(tb_nccl_comm* c) {
  tb_clear_error();
  if (!c) return TB_OK;
  tbStatus st = TB_OK;
  if (c->comm) {
    const ncclResult_t r = nccl().comm_destroy(c->comm);
    if (r != ncclSuccess) st = nccl_fail("ncclCommDestroy", r);
  }
  delete c;
  return st;
}

// Workspace: [staging m × n f32][contiguous receive rows when ldc != n][plan workspace].
static size_t kshard_ws(const tb_matmul_plan* p, int world, int64_t ldc, size_t* recv_off,
                        size_t* plan_off) {
  const size_t staging = align256((size_t)p->desc.m * (size_t)p->desc.n * sizeof(float));
  const size_t rows = (size_t)(p->desc.m / world);
  const size_t recv = ldc == p->desc.n ? 0 : align256(rows * (size_t)p->desc.n * sizeof(float));
  *recv_off = staging;
  *plan_off = staging + recv;
  return staging + recv + p->workspace_bytes;
}

extern "C" size_t tb_matmul_kshard_nccl_workspace_bytes(const tb_matmul_plan* plan, int world,
                                                        int64_t ldc) {
  if (!plan || plan->dynamic || world < 1) return 0;
  size_t a, b;
  return kshard_ws(plan, world, ldc, &a, &b);
}

extern "C" tbStatus tb_matmul_run_kshard_nccl(const tb_matmul_plan* plan, tb_nccl_comm* c,
                                              const void* A, int64_t lda, const void* B, int64_t ldb,
                                              void* C_rows, int64_t ldc, void* workspace,
                                              size_t workspace_bytes, void* stream_v) {
  tb_clear_error();
  if (!plan || !c || !c->comm) return tb_fail(TB_ERR_INVALID_ARGUMENT, "plan and comm are required");
  if (plan->dynamic)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "K-sharded runs take a plan with static dims");
  const tb_matmul_desc& d = plan->desc;
  if (d.c_dtype != TB_F32)
    return tb_fail(TB_ERR_UNSUPPORTED, "K-sharded runs accumulate f32 partials: C must be f32");
  if (d.bias || d.activation != TB_ACT_NONE || d.clamp)
    return tb_fail(TB_ERR_UNSUPPORTED,
                   "epilogue expressions apply to the complete sum, not to per-rank partials");
  if (d.m % c->world != 0)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "m must be a multiple of the world size");
  if (!C_rows || ldc < d.n) return tb_fail(TB_ERR_INVALID_ARGUMENT, "C rows and ldc >= n are required");
  size_t recv_off, plan_off;
  const size_t need = kshard_ws(plan, c->world, ldc, &recv_off, &plan_off);
  if (!workspace || workspace_bytes < need)
    return tb_fail(TB_ERR_WORKSPACE, "K-sharded NCCL run needs " + std::to_string(need) +
                                         " workspace bytes (tb_matmul_kshard_nccl_workspace_bytes)");
  if (!nccl().ok) return tb_fail(TB_ERR_NCCL, nccl().why);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  auto* ws = static_cast<unsigned char*>(workspace);
  float* staging = reinterpret_cast<float*>(ws);
  const int64_t rows = d.m / c->world;
  const size_t row_bytes = (size_t)d.n * sizeof(float);
  // Staging starts as zero with this rank's rows holding C_in (beta = 1), so
  // the sum over ranks adds C_in exactly once.
  cudaError_t e = cudaMemsetAsync(staging, 0, (size_t)d.m * row_bytes, stream);
  if (e != cudaSuccess) return cuda_fail("cudaMemsetAsync", e);
  if (d.beta) {
    e = cudaMemcpy2DAsync(staging + (size_t)c->rank * rows * d.n, row_bytes, C_rows,
                          (size_t)ldc * sizeof(float), row_bytes, (size_t)rows, cudaMemcpyDeviceToDevice,
                          stream);
    if (e != cudaSuccess) return cuda_fail("cudaMemcpy2DAsync", e);
  }
  tbStatus st = tb_launch(plan, A, lda, B, ldb, staging, d.n, ws + plan_off, workspace_bytes - plan_off,
                          stream_v);
  if (st != TB_OK) return st;
  float* recv = ldc == d.n ? static_cast<float*>(C_rows) : reinterpret_cast<float*>(ws + recv_off);
  const ncclResult_t r = nccl().reduce_scatter(staging, recv, (size_t)rows * d.n, ncclFloat32, ncclSum,
                                               c->comm, stream);
  if (r != ncclSuccess) return nccl_fail("ncclReduceScatter", r);
  if (recv != C_rows) {
    e = cudaMemcpy2DAsync(C_rows, (size_t)ldc * sizeof(float), recv, row_bytes, row_bytes, (size_t)rows,
                          cudaMemcpyDeviceToDevice, stream);
    if (e != cudaSuccess) return cuda_fail("cudaMemcpy2DAsync", e);
  }
  return TB_OK;
}
