// tb_mapping.h — program-id → work mapping shared by the host plan and the
// sm_100a kernels. A "program" is the reference's unit of work (one
// `gpu.func` instance per pid); here resident CTAs walk the program list.
//
// The formulas restate the reference's runtime mapping:
//   * tile / grouped_tile / persistent_tile:
//       buildProgramWorkAssignment, LowerPipelineToNVGPU.cpp:283-304
//   * split_k: LowerPipelineToNVGPU.cpp:305-316
//   * K range of a split part, in block_k tiles:
//       buildSplitKGroupActivePredicate, LowerPipelineToNVGPU.cpp:325-357
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define TB_HD __host__ __device__ __forceinline__
#else
#define TB_HD inline
#endif

namespace tb {

enum MappingKind : int32_t {
  kMapTile = 0,
  kMapGroupedTile = 1,
  kMapSplitK = 2,
  kMapPersistentTile = 3,
};

// Plain-old-data copy of the mapping facts the kernels need.
struct MappingArgs {
  int32_t kind;
  int32_t tiles_m, tiles_n, tiles_k;   // problem tiles in block units
  int32_t group_span_m;                // groupTileSpanM
  int32_t programs_per_group;          // programsPerLaunchGroup
  int32_t split_k;
  int32_t total_programs;
};

struct Work {
  int32_t tile_m, tile_n, part;
  int32_t kt_begin, kt_count;  // K range in block_k tiles
};

TB_HD Work program_work(const MappingArgs& a, int32_t pid) {
  Work w;
  if (a.kind == kMapSplitK) {
    const int32_t group = pid / a.programs_per_group;
    const int32_t in_group = pid % a.programs_per_group;
    w.tile_m = group;
    w.tile_n = in_group / a.split_k;
    w.part = in_group % a.split_k;
    const int32_t base = a.tiles_k / a.split_k;
    const int32_t extra = a.tiles_k % a.split_k;
    w.kt_begin = w.part * base + (w.part < extra ? w.part : extra);
    w.kt_count = base + (w.part < extra ? 1 : 0);
  } else {
    const int32_t group = pid / a.programs_per_group;
    const int32_t first_m = group * a.group_span_m;
    const int32_t left_m = a.tiles_m - first_m;
    const int32_t size_m = a.group_span_m < left_m ? a.group_span_m : left_m;
    const int32_t in_group = pid % a.programs_per_group;
    w.tile_m = first_m + in_group % size_m;
    w.tile_n = in_group / size_m;
    w.part = 0;
    w.kt_begin = 0;
    w.kt_count = a.tiles_k;
  }
  return w;
}

// ---- hardware walk order ----------------------------------------------
// The order in which resident CTAs take work items (a program, or two or
// four programs when the plan fuses them; see item_first_pid). Which CTA runs a program, and when, does not change its
// result: each program still computes the reference's tile over its K range.
// The order only decides what shares L2 at a time.
//   kWalkRowGroups (row-major tile / persistent mappings): the reference's
//     persistent CTAs take pids c, c + R, ..., so every concurrent wave spans
//     a full tile row and re-reads each B panel from DRAM per tile row. Items
//     are walked in groups of kWalkRows item rows, column by column.
//   kWalkSerpentine (grouped mapping): GROUP_M order, every other group
//     walked from its last column back, so a group's first programs reuse the
//     B panels the previous group read last.
enum WalkMode : int32_t { kWalkIdentity = 0, kWalkRowGroups = 1, kWalkSerpentine = 2 };
constexpr int32_t kWalkRows = 8;

TB_HD int32_t walk_mode(const MappingArgs& a, int32_t fuse) {
  if (a.kind == kMapGroupedTile) return kWalkSerpentine;
  if ((a.kind == kMapTile || a.kind == kMapPersistentTile) && a.tiles_m > 1 &&
      a.tiles_n / (fuse == 2 ? 2 : 1) > 1)
    return kWalkRowGroups;
  return kWalkIdentity;
}

// Work item taken at position `w` of the walk.
TB_HD int32_t walk_item(const MappingArgs& a, int32_t fuse, int32_t mode, int32_t w) {
  if (mode == kWalkSerpentine) {
    const int32_t per = fuse == 1 || fuse == 3 ? 2 : fuse == 4 ? 4 : 1;  // programs per item
    const int32_t ppg = a.programs_per_group / per;        // items per full group
    const int32_t g = w / ppg;
    if ((g & 1) == 0) return w;
    const int32_t first = g * a.group_span_m;
    const int32_t left = a.tiles_m - first;
    const int32_t rows = left < a.group_span_m ? left : a.group_span_m;
    const int32_t size = fuse == 1 || fuse == 4 ? rows / 2 : rows;  // items per item column
    const int32_t ncols = fuse == 3 || fuse == 4 ? a.tiles_n / 2 : a.tiles_n;
    const int32_t in = w - g * ppg;
    return g * ppg + (ncols - 1 - in / size) * size + in % size;
  }
  if (mode == kWalkRowGroups) {
    const int32_t cols = a.tiles_n / (fuse == 2 ? 2 : 1);
    const int32_t span = kWalkRows * cols;
    const int32_t first = (w / span) * kWalkRows;
    const int32_t left = a.tiles_m - first;
    const int32_t size = left < kWalkRows ? left : kWalkRows;
    const int32_t in = w % span;
    return (first + in % size) * cols + in / size;
  }
  return w;
}

// First program of work item `item`: fuse 1 = pids 2i, 2i+1 (vertical pair,
// grouped order), 2 = pids 2i, 2i+1 (horizontal pair, row-major order),
// 3 = pids p and p + rows (horizontal pair in grouped order: one row of a
// group in columns 2c and 2c + 1, rows = the group's height), 4 = a 2 × 2
// block in grouped order: pids p, p + 1 (vertical pair in column 2c) and
// p + rows, p + rows + 1 (the same pair in column 2c + 1; rows even). Items
// are numbered group by group, column pair by column pair, down the rows, as
// the programs are.
TB_HD int32_t item_first_pid(const MappingArgs& a, int32_t fuse, int32_t item) {
  if (fuse != 3 && fuse != 4) return fuse ? 2 * item : item;
  const int32_t per = fuse == 4 ? 4 : 2;
  const int32_t group = (per * item) / a.programs_per_group;
  const int32_t first = group * a.group_span_m;
  const int32_t left = a.tiles_m - first;
  const int32_t rows = left < a.group_span_m ? left : a.group_span_m;
  const int32_t wi = item - group * (a.programs_per_group / per);
  if (fuse == 3) return group * a.programs_per_group + 2 * (wi / rows) * rows + wi % rows;
  const int32_t half = rows / 2;
  return group * a.programs_per_group + 2 * (wi / half) * rows + 2 * (wi % half);
}

}  // namespace tb
