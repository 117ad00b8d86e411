// tb_shard.cpp — N-column sharded runs (one process per GPU, no collective).
//
// The reference is single-GPU. Its op C = C_in + A·B splits along N with
// no exchange: rank r of W owns columns [col0_r, col0_r + ncols_r) of B and C
// (whole block_n program tiles, balanced over the ranks, the last ranks
// taking one tile fewer), A is replicated, and each rank runs the
// single-GPU op on its slice — a tb.matmul of m × ncols_r × k with the same
// knobs. Host-only: the per-shard plan is derived on each call (integer
// arithmetic, no allocation on the device) and launched by tb_launch_ex.

#include <string>

#include "tb_plan.h"

namespace {

// [col0, col0 + ncols) of `rank`: balanced in block_n units (the first
// `extra` ranks take one tile more).
void shard_columns(const tb_matmul_desc& d, int rank, int world, int64_t* col0, int64_t* ncols) {
  const int64_t units = (d.n + d.block_n - 1) / d.block_n;
  const int64_t base = units / world, extra = units % world;
  const int64_t u0 = rank * base + (rank < extra ? rank : extra);
  const int64_t u1 = u0 + base + (rank < extra ? 1 : 0);
  const int64_t c0 = u0 * d.block_n < d.n ? u0 * d.block_n : d.n;
  const int64_t c1 = u1 * d.block_n < d.n ? u1 * d.block_n : d.n;
  *col0 = c0;
  *ncols = c1 - c0;
}

tbStatus check_args(const tb_matmul_plan* plan, int rank, int world) {
  if (!plan) return tb_fail(TB_ERR_INVALID_ARGUMENT, "plan must not be NULL");
  if (plan->dynamic)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "N-sharded runs take a plan with static dims");
  if (world < 1 || rank < 0 || rank >= world)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "rank must be in [0, world) and world >= 1");
  return TB_OK;
}

// The plan of this rank's slice: the same knobs on m × ncols × k.
tbStatus shard_plan(const tb_matmul_plan* plan, int64_t ncols, tb_matmul_plan* out) {
  tb_matmul_desc d = plan->desc;
  d.n = ncols;
  return tb_plan_build(d, plan->device, plan->num_sms, out);
}

}  // namespace

extern "C" tbStatus tb_matmul_nshard_columns(const tb_matmul_plan* plan, int rank, int world,
                                             int64_t* col0, int64_t* ncols) {
  tb_clear_error();
  tbStatus st = check_args(plan, rank, world);
  if (st != TB_OK) return st;
  if (!col0 || !ncols) return tb_fail(TB_ERR_INVALID_ARGUMENT, "col0 and ncols must not be NULL");
  shard_columns(plan->desc, rank, world, col0, ncols);
  return TB_OK;
}

extern "C" tbStatus tb_matmul_nshard_workspace_bytes(const tb_matmul_plan* plan, int rank, int world,
                                                     size_t* bytes) {
  tb_clear_error();
  tbStatus st = check_args(plan, rank, world);
  if (st != TB_OK) return st;
  if (!bytes) return tb_fail(TB_ERR_INVALID_ARGUMENT, "bytes must not be NULL");
  int64_t c0 = 0, nc = 0;
  shard_columns(plan->desc, rank, world, &c0, &nc);
  *bytes = 0;
  if (nc == 0) return TB_OK;
  tb_matmul_plan sp;
  st = shard_plan(plan, nc, &sp);
  if (st != TB_OK) return st;
  *bytes = sp.workspace_bytes;
  return TB_OK;
}

extern "C" tbStatus tb_matmul_run_nshard(const tb_matmul_plan* plan, int rank, int world,
                                         const void* A, int64_t lda, const void* B_cols,
                                         int64_t ldb, void* C_cols, int64_t ldc,
                                         const float* bias_cols, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  tb_clear_error();
  tbStatus st = check_args(plan, rank, world);
  if (st != TB_OK) return st;
  if (plan->desc.b_col_major)
    return tb_fail(TB_ERR_UNSUPPORTED,
                   "N-sharded runs take row-major B (a column slice of a column-major B is a "
                   "row range: pass it to tb_matmul_run as its own plan)");
  int64_t c0 = 0, nc = 0;
  shard_columns(plan->desc, rank, world, &c0, &nc);
  if (nc == 0) return TB_OK;  // more ranks than column tiles: nothing to do here
  tb_matmul_plan sp;
  st = shard_plan(plan, nc, &sp);
  if (st != TB_OK) return st;
  return tb_launch_ex(&sp, A, lda, B_cols, ldb, C_cols, ldc, bias_cols, workspace, workspace_bytes,
                      stream);
}
