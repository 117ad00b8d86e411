/* Plain-C caller of libtbgemm.so (built and run by tests/test_capi_c_caller.py):
 * what a C/C++ program that used the reference's generated kernel links
 * against. Host-only calls (device = -1), so it runs without a GPU. */
#include <stdio.h>
#include <string.h>

#include "tb_gemm.h"

int main(void) {
  tb_matmul_desc d;
  if (tb_matmul_desc_init(&d) != TB_OK) return 1;
  d.m = 192; d.n = 128; d.k = 32;
  d.block_m = 64; d.block_n = 64; d.block_k = 32;
  d.group_m = 2; d.num_warps = 4; d.num_stages = 2;
  tb_matmul_plan* plan = NULL;
  if (tb_matmul_plan_create(&d, -1, &plan) != TB_OK) {
    printf("plan failed: %s\n", tb_last_error());
    return 2;
  }
  char buf[4096];
  size_t need = 0;
  if (tb_matmul_plan_describe(plan, buf, sizeof buf, &need) != TB_OK) return 3;
  printf("%s\n", buf);
  tb_program_work w;
  for (int64_t pid = 0; pid < 6; ++pid) {
    if (tb_matmul_program_work(plan, pid, &w) != TB_OK) return 4;
    printf("pid %lld -> tile (%lld, %lld)\n", (long long)pid, (long long)w.tile_m, (long long)w.tile_n);
  }
  tb_matmul_plan_destroy(plan);
  /* a knob the reference rejects: same status class and message */
  d.block_m = 40;
  if (tb_matmul_plan_create(&d, -1, &plan) != TB_ERR_INVALID_ARGUMENT) return 5;
  printf("rejected: %s\n", tb_last_error());
  /* N-shard: columns of each of 3 ranks for 8192 columns of 256-wide tiles */
  tb_matmul_desc big;
  tb_matmul_desc_init(&big);
  big.m = 8192; big.n = 8192; big.k = 8192;
  big.block_m = 256; big.block_n = 256; big.block_k = 64;
  big.num_warps = 4; big.num_stages = 4;
  if (tb_matmul_plan_create(&big, -1, &plan) != TB_OK) return 6;
  for (int r = 0; r < 3; ++r) {
    int64_t c0 = 0, nc = 0;
    size_t ws = 1;
    if (tb_matmul_nshard_columns(plan, r, 3, &c0, &nc) != TB_OK) return 7;
    if (tb_matmul_nshard_workspace_bytes(plan, r, 3, &ws) != TB_OK) return 8;
    printf("nshard rank %d: columns %lld + %lld, workspace %zu\n", r, (long long)c0, (long long)nc, ws);
  }
  if (tb_matmul_nshard_columns(plan, 3, 3, NULL, NULL) != TB_ERR_INVALID_ARGUMENT) return 9;
  tb_matmul_plan_destroy(plan);
  printf("version: %s\n", tb_version());
  return 0;
}
