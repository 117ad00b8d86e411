// tb_dynamic.cpp — plans with dynamic ("?") problem dims.
//
// The reference requires static memref shapes: deriveSourceKernelConfig
// rejects `memref<?x…>` (lib/Analysis/KernelConfig.cpp:98-103), so one
// compiled kernel serves exactly one M×N×K. Here a plan may leave any of m, n,
// k open (TB_DIM_DYNAMIC in the descriptor). Its knobs are validated once, at creation,
// on a probe shape; every run then names its shape, and the concrete plan for
// that shape (mapping, hardware tile, grid, workspace) is derived on first use
// and kept in a per-plan cache. The kernels are the same ones a static plan
// launches; only host-side plan derivation moves from creation to first run.

#include <cstring>
#include <mutex>
#include <new>
#include <sstream>
#include <unordered_map>

#include "tb_plan.h"

struct TbShapeKey {
  int64_t m, n, k;
  bool operator==(const TbShapeKey& o) const { return m == o.m && n == o.n && k == o.k; }
};
struct TbShapeKeyHash {
  size_t operator()(const TbShapeKey& x) const {
    uint64_t h = (uint64_t)x.m * 0x9E3779B97F4A7C15ull;
    h ^= (uint64_t)x.n + 0x7F4A7C159E3779B9ull + (h << 6) + (h >> 2);
    h ^= (uint64_t)x.k + 0x94D049BB133111EBull + (h << 6) + (h >> 2);
    return (size_t)h;
  }
};

struct TbShapeCache {
  // Bounded: when full, the cache starts over. Runs hold a shared_ptr to the
  // concrete plan they launch, so dropping entries never frees one in use.
  static constexpr size_t kMaxShapes = 256;
  std::mutex mu;
  std::unordered_map<TbShapeKey, std::shared_ptr<const tb_matmul_plan>, TbShapeKeyHash> plans;
  uint64_t derived = 0;  // concrete plans derived so far (misses)
};

namespace {

bool is_open(int64_t dim) { return dim == TB_DIM_DYNAMIC; }

// Concrete plan of `plan` for m×n×k (from the cache, derived on a miss).
tbStatus shape_plan(const tb_matmul_plan* plan, int64_t m, int64_t n, int64_t k,
                    std::shared_ptr<const tb_matmul_plan>* out) {
  if (!plan) return tb_fail(TB_ERR_INVALID_ARGUMENT, "plan must not be NULL");
  if (!plan->dynamic)
    return tb_fail(TB_ERR_INVALID_ARGUMENT,
                   "this plan has static dims: run it with tb_matmul_run");
  const tb_matmul_desc& d = plan->desc;
  if ((!is_open(d.m) && m != d.m) || (!is_open(d.n) && n != d.n) ||
      (!is_open(d.k) && k != d.k))
    return tb_fail(TB_ERR_INVALID_ARGUMENT,
                   "run shape " + std::to_string(m) + "x" + std::to_string(n) + "x" +
                       std::to_string(k) + " differs from the plan's static dims");
  TbShapeCache& c = *plan->shapes;
  const TbShapeKey key{m, n, k};
  {
    std::lock_guard<std::mutex> lock(c.mu);
    auto it = c.plans.find(key);
    if (it != c.plans.end()) {
      *out = it->second;
      return TB_OK;
    }
  }
  // Derive outside the lock (pure host arithmetic); a racing thread may
  // derive the same shape too, and the first insert wins.
  tb_matmul_desc sd = d;
  sd.m = m;
  sd.n = n;
  sd.k = k;
  auto p = std::make_shared<tb_matmul_plan>();
  tbStatus st = tb_plan_build(sd, plan->device, plan->num_sms, p.get());
  if (st != TB_OK) return st;
  std::lock_guard<std::mutex> lock(c.mu);
  if (c.plans.size() >= TbShapeCache::kMaxShapes) c.plans.clear();
  auto ins = c.plans.emplace(key, std::move(p));
  if (ins.second) ++c.derived;
  *out = ins.first->second;
  return TB_OK;
}

}  // namespace

extern "C" tbStatus tb_matmul_plan_create_dynamic(const tb_matmul_desc* desc, int device,
                                                  tb_matmul_plan** out) {
  tb_clear_error();
  if (!desc || !out) return tb_fail(TB_ERR_INVALID_ARGUMENT, "desc and plan must not be NULL");
  *out = nullptr;
  // Validate every knob once on a probe shape that each rule accepts for
  // shape reasons (two tiles per open dim, divisible for exact_tile, K
  // covering every split part); the rules left are then the knobs' own.
  tb_matmul_desc probe = *desc;
  if (is_open(probe.m)) probe.m = 2 * (probe.block_m > 0 ? probe.block_m : 1);
  if (is_open(probe.n)) probe.n = 2 * (probe.block_n > 0 ? probe.block_n : 1);
  if (is_open(probe.k))
    probe.k = 2 * (probe.block_k > 0 ? probe.block_k : 1) * (probe.split_k > 1 ? probe.split_k : 1);
  tb_matmul_plan* probe_plan = nullptr;
  tbStatus st = tb_matmul_plan_create(&probe, device, &probe_plan);
  if (st != TB_OK) return st;
  probe_plan->desc = *desc;
  if (is_open(desc->m)) probe_plan->desc.m = TB_DIM_DYNAMIC;
  if (is_open(desc->n)) probe_plan->desc.n = TB_DIM_DYNAMIC;
  if (is_open(desc->k)) probe_plan->desc.k = TB_DIM_DYNAMIC;
  probe_plan->dynamic = true;
  probe_plan->shapes = std::make_shared<TbShapeCache>();
  *out = probe_plan;
  return TB_OK;
}

extern "C" tbStatus tb_matmul_workspace_bytes_dynamic(const tb_matmul_plan* plan, int64_t m,
                                                      int64_t n, int64_t k, size_t* bytes) {
  tb_clear_error();
  if (!bytes) return tb_fail(TB_ERR_INVALID_ARGUMENT, "bytes must not be NULL");
  *bytes = 0;
  std::shared_ptr<const tb_matmul_plan> sp;
  tbStatus st = shape_plan(plan, m, n, k, &sp);
  if (st != TB_OK) return st;
  *bytes = sp->workspace_bytes;
  return TB_OK;
}

extern "C" tbStatus tb_matmul_run_dynamic(const tb_matmul_plan* plan, int64_t m, int64_t n,
                                          int64_t k, const void* A, int64_t lda, const void* B,
                                          int64_t ldb, void* C, int64_t ldc, const float* bias,
                                          void* workspace, size_t workspace_bytes,
                                          void* stream) {
  tb_clear_error();
  std::shared_ptr<const tb_matmul_plan> sp;
  tbStatus st = shape_plan(plan, m, n, k, &sp);
  if (st != TB_OK) return st;
  return tb_launch_ex(sp.get(), A, lda, B, ldb, C, ldc, bias, workspace, workspace_bytes, stream);
}

extern "C" tbStatus tb_matmul_plan_for_shape(const tb_matmul_plan* plan, int64_t m, int64_t n,
                                             int64_t k, tb_matmul_plan** out) {
  tb_clear_error();
  if (!out) return tb_fail(TB_ERR_INVALID_ARGUMENT, "plan must not be NULL");
  *out = nullptr;
  std::shared_ptr<const tb_matmul_plan> sp;
  tbStatus st = shape_plan(plan, m, n, k, &sp);
  if (st != TB_OK) return st;
  tb_matmul_plan* copy = new (std::nothrow) tb_matmul_plan(*sp);
  if (!copy) return tb_fail(TB_ERR_INVALID_ARGUMENT, "out of host memory");
  *out = copy;
  return TB_OK;
}

// JSON facts of a dynamic plan (the shape-dependent ones are per run).
std::string tb_describe_dynamic(const tb_matmul_plan* plan) {
  const tb_matmul_desc& d = plan->desc;
  auto dim = [](int64_t x) { return x == TB_DIM_DYNAMIC ? std::string("null") : std::to_string(x); };
  size_t cached = 0;
  uint64_t derived = 0;
  {
    std::lock_guard<std::mutex> lock(plan->shapes->mu);
    cached = plan->shapes->plans.size();
    derived = plan->shapes->derived;
  }
  std::ostringstream o;
  o << "{\"dynamic\": true, ";
  o << "\"problem\": [" << dim(d.m) << ", " << dim(d.n) << ", " << dim(d.k) << "], ";
  o << "\"tile\": [" << d.block_m << ", " << d.block_n << ", " << d.block_k << "], ";
  o << "\"exact_tile\": " << (d.exact_tile ? "true" : "false") << ", ";
  o << "\"num_warps\": " << d.num_warps << ", ";
  o << "\"requested_stages\": " << d.num_stages << ", ";
  o << "\"warp_grid\": [" << plan->warp_grid_m << ", " << plan->warp_grid_n << "], ";
  o << "\"group_m\": " << d.group_m << ", ";
  o << "\"split_k\": " << (d.split_k > 1 ? d.split_k : 1) << ", ";
  o << "\"reduction_kind\": \"" << plan->reduction_kind << "\", ";
  o << "\"persistent\": " << (d.persistent ? "true" : "false") << ", ";
  o << "\"num_ctas\": " << plan->num_ctas << ", ";
  o << "\"num_sms\": " << plan->num_sms << ", ";
  o << "\"beta\": " << d.beta << ", ";
  o << "\"a_layout\": \"" << (d.a_col_major ? "col_major" : "row_major") << "\", ";
  o << "\"b_layout\": \"" << (d.b_col_major ? "col_major" : "row_major") << "\", ";
  o << "\"shapes_cached\": " << cached << ", ";
  o << "\"shapes_derived\": " << derived << "}";
  return o.str();
}
