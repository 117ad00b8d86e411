// tb_plan.h — the immutable plan behind the C ABI's opaque tb_matmul_plan.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <memory>
#include <string>

#include "../../include/tb_gemm.h"
#include "tb_mapping.h"

// Kernel family selected by the plan (the hardware CTA tile; the program tile
// is block_m × block_n and may be smaller, with the rest masked).
enum TbKernelTile : int32_t {
  kTile128x64 = 0,
  kTile128x128 = 1,
  kTile128x256 = 2,
  kTile256x128 = 3,  // CTA pair (cta_group::2)
  kTile256x256 = 4,  // CTA pair (cta_group::2)
  kTile256x512 = 5,  // CTA pair, two N = 256 MMAs per K step, one accumulator
};

enum TbEpilogue : int32_t {
  kEpiStore = 0,      // C = beta·C_in + acc
  kEpiWorkspace = 1,  // ws[part] = acc   (split_k_serial)
  kEpiAtomic = 2,     // C += acc atomically (split_k_parallel)
};

struct TbShapeCache;  // tb_dynamic.cpp

struct tb_matmul_plan {
  tb_matmul_desc desc;
  // Dynamic plan: desc.m/n/k equal to TB_DIM_DYNAMIC are left open ("?" dims) and every run
  // names its shape; the concrete per-shape plans live in `shapes`. All the
  // facts below are then those of a probe shape and are not used for launch.
  bool dynamic = false;
  std::shared_ptr<TbShapeCache> shapes;
  int device;
  int num_sms;

  // --- reference plan facts (ProgramMappingPlan / ReductionPlan /
  //     PersistentWorkPlan / EncodingPlan) ---
  tb::MappingArgs map;
  std::string mapping_kind;    // "tile" | "grouped_tile" | "split_k" | "persistent_tile"
  std::string launch_order;    // "row_major" | "grouped_m" | "persistent"
  std::string swizzle_kind;    // "none" | "grouped_m"
  std::string reduction_kind;  // "none" | "split_k_serial" | "split_k_atomic"
  std::string mainline_kind;   // "single_tile" | "grouped_tile" | "split_k" | "persistent_tile_loop"
  int64_t launch_group_count;
  int64_t group_tile_span_n;
  int64_t programs_per_tile;
  int64_t num_ctas;            // after the reference's clamps
  int64_t resident_programs;   // persistent: min(num_ctas, numSms)
  int64_t warp_grid_m, warp_grid_n;

  // --- this build's launch facts ---
  int32_t kernel_tile;         // TbKernelTile
  // Program fusion: programs whose tiles are adjacent run as one hardware
  // work item (same programs, same results; tb::item_first_pid): 1 =
  // vertical pair (grouped order, even group),
  // 2 = horizontal pair (row-major / persistent order), 3 = horizontal pair
  // in grouped order (pids p and p + group rows), 4 = 2 × 2 block (grouped
  // order, even group and tile counts), 0 = none.
  int32_t fuse;
  int64_t work_items;          // total_programs / programs per item (1, 2 or 4), or × sub-tiles
  int32_t sub_m, sub_n;        // hardware tiles per program along M / N (programs larger than a tile)
  // Tail balancing (tb_choose_tail_split, a stream-K tail): walk positions
  // [0, dp_items) run whole work items; the last tail_items items form one
  // run of tail_items · tail_fills ring fills split evenly over tail_slots
  // slots, each slot taking up to tail_segs segments (parts of one item; a
  // partial one is reduce-added into C). positions = dp_items +
  // tail_segs · tail_slots.
  int64_t dp_items, tail_items, tail_slots, tail_segs, tail_fills, positions;
  // Latency kernel (tb_gemm_small_kernel): one-CTA tiles at most 128 wide,
  // every work item at most 128 K elements, row-major operands, at most
  // four items per CTA.
  bool small;
  int32_t cta_m, cta_n;        // hardware tile (cta_m = 256: a CTA pair)
  int32_t ctas_per_tile;       // 1 or 2
  int32_t stages;              // shared-memory ring depth
  int32_t kb;                  // K elements per ring stage (64 or 128)
  int32_t epilogue;            // TbEpilogue
  int64_t grid;                // CTAs launched
  size_t smem_bytes;
  int32_t tmem_cols;
  size_t workspace_bytes;       // partial_bytes + pack_a_bytes + pack_b_bytes (256-aligned parts)
  size_t partial_bytes;         // split_k_serial f32 partials, at offset 0
  size_t pack_a_offset, pack_a_bytes;  // zero-padded copy of A when its rows are not TMA-aligned
  size_t pack_b_offset, pack_b_bytes;  // same for B
};

// Defined in tb_launch.cu.
tbStatus tb_launch_ex(const tb_matmul_plan* plan, const void* A, int64_t lda, const void* B,
                      int64_t ldb, void* C, int64_t ldc, const float* bias, void* workspace,
                      size_t workspace_bytes, void* stream);
tbStatus tb_launch(const tb_matmul_plan* plan, const void* A, int64_t lda,
                   const void* B, int64_t ldb, void* C, int64_t ldc,
                   void* workspace, size_t workspace_bytes, void* stream);
size_t tb_kernel_smem_bytes(int32_t kernel_tile, int32_t stages);
int32_t tb_kernel_max_stages(int32_t kernel_tile);
int32_t tb_kernel_kb(int32_t kernel_tile);
size_t tb_small_smem_bytes(int32_t cta_n, int32_t c_dtype);

// Derives a concrete plan for `d` (validated) into *out; tb_plan.cpp.
tbStatus tb_plan_build(const tb_matmul_desc& d, int device, int num_sms, tb_matmul_plan* out);

// JSON facts of a dynamic plan; tb_dynamic.cpp.
std::string tb_describe_dynamic(const tb_matmul_plan* plan);

// Chooses the stream-K tail for `items` equal work items of `fills` ring
// fills on `slots` resident slots (tb_plan.cpp); *tail_items = 0: none.
void tb_choose_tail_split(int64_t items, int64_t slots, int64_t fills, int64_t* dp_items,
                          int64_t* tail_items, int64_t* tail_segs);

// Thread-local error message helpers (tb_plan.cpp).
tbStatus tb_fail(tbStatus code, const std::string& msg);
void tb_clear_error();
