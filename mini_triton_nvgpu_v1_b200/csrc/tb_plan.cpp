// tb_plan.cpp — knob validation and program mapping behind the C ABI.
//
// Host-only C++: the rules and the error messages restate the reference's
// compile-time analyses so that a knob set the reference rejects is rejected
// here with the same words:
//   verifySupportedKernelConfig   lib/Analysis/KernelConfig.cpp:202-246
//   deriveProgramMappingPlan      lib/Analysis/ProgramMappingPlan.cpp:329-458
//   validateProgramMappingPlan    lib/Analysis/ProgramMappingPlan.cpp:219-324
//   deriveReductionPlan           lib/Analysis/ReductionPlan.cpp:137-192
//   derivePersistentWorkPlan      lib/Analysis/PersistentWorkPlan.cpp:91-131
//   deriveWarpGrid                lib/Analysis/EncodingPlan.cpp:283-321
//   selectedMainlineKind          lib/Analysis/ResourceClosurePlan.cpp:154-161
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <new>
#include <sstream>
#include <string>

#include "tb_plan.h"

namespace {

thread_local std::string g_last_error;

constexpr int kDefaultB200Sms = 148;
constexpr int64_t kMaxWarpsPerCta = 8;  // TargetInfo.cpp:126

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

const char* dtype_name(int32_t t) {
  switch (t) {
    case TB_F16: return "f16";
    case TB_F32: return "f32";
    case TB_BF16: return "bf16";
  }
  return "?";
}

// deriveWarpGrid (EncodingPlan.cpp:283-321) for the m16n8k16 instruction
// shape: the most square warp tile wins; ties prefer more warps along the
// longer block edge.
bool derive_warp_grid(int64_t num_warps, int64_t bm, int64_t bn, int64_t* gm,
                      int64_t* gn) {
  const int64_t im = 16, in = 8;
  int64_t best_m = -1, best_n = -1;
  int64_t best = std::numeric_limits<int64_t>::max();
  for (int64_t wm = 1; wm <= num_warps; ++wm) {
    if (num_warps % wm != 0) continue;
    const int64_t wn = num_warps / wm;
    if (bm % wm != 0 || bn % wn != 0) continue;
    const int64_t tm = bm / wm, tn = bn / wn;
    if (tm % im != 0 || tn % in != 0) continue;
    const int64_t score = std::llabs(tm - tn);
    if (score < best || (score == best && ((bm >= bn && wm > best_m) ||
                                           (bm < bn && wn > best_n)))) {
      best = score;
      best_m = wm;
      best_n = wn;
    }
  }
  if (best_m <= 0 || best_n <= 0) return false;
  *gm = best_m;
  *gn = best_n;
  return true;
}

}  // namespace

void tb_choose_tail_split(int64_t items, int64_t slots, int64_t fills, int64_t* dp_items,
                          int64_t* tail_items, int64_t* tail_segs) {
  // Cost model in ring fills per slot (every item has `fills` fills). The
  // whole waves before the last full one keep their items whole; the rest
  // (one full wave plus the partial one, L items) is cut into `slots` equal
  // runs of consecutive fills — a run starts and ends inside items, so a
  // slot works on up to three segments, the partial ones reduce-added into
  // C. Each segment beyond a slot's first is charged kSegCost fills (its
  // start and its partial-tile reduce-add). The tail is taken only when it
  // shortens the modelled makespan by 5 % or more. (Measured on one B200:
  // cutting every item of the 8-way slice of 8192³ into 4 K pieces instead
  // lost 5 %; the stream-K run bounds the partial segments to two per slot.)
  constexpr int64_t kSegCost = 8;
  *dp_items = items;
  *tail_items = 0;
  *tail_segs = 0;
  if (slots <= 1 || items <= 0 || items % slots == 0 || fills < 16) return;
  const int64_t whole = (items + slots - 1) / slots * fills;
  const int64_t d = std::max<int64_t>(0, items / slots - 1) * slots;
  const int64_t L = items - d;
  const int64_t U = L * fills;
  int64_t segs = 1;
  for (int64_t p = 0; p < slots; ++p) {
    const int64_t u0 = p * U / slots, u1 = (p + 1) * U / slots;
    if (u1 > u0) segs = std::max<int64_t>(segs, (u1 - 1) / fills - u0 / fills + 1);
  }
  // Runs shorter than kMinRun fills are all start-up and reduce-add: keep
  // such problems whole (e.g. 1024³ on 74 pairs would give 3–4 fills a slot).
  constexpr int64_t kMinRun = 32;
  const int64_t run = (U + slots - 1) / slots;
  const int64_t t = d / slots * fills + run + kSegCost * (segs - 1);
  // With no whole wave before it (d = 0) the tail measured slower: every
  // slot then starts mid-item from the first fill, so the CTAs that share an
  // A or B panel slice no longer read it at the same time (8192 × 1024 ×
  // 8192 on 74 pairs: 124.8 µs against 113.2 µs whole; with a whole wave
  // first, 8192 × 2048 × 8192: 213 against 229 µs).
  if (d > 0 && run >= kMinRun && t < whole - whole * 5 / 100 && d + segs * slots <= std::numeric_limits<int32_t>::max()) {
    *dp_items = d;
    *tail_items = L;
    *tail_segs = segs;
  }
}

tbStatus tb_fail(tbStatus code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

void tb_clear_error() { g_last_error.clear(); }

extern "C" const char* tb_last_error(void) { return g_last_error.c_str(); }

extern "C" const char* tb_version(void) { return "tbgemm 0.1 (sm_100a tcgen05)"; }

extern "C" tbStatus tb_matmul_desc_init(tb_matmul_desc* d) {
  if (!d) return tb_fail(TB_ERR_INVALID_ARGUMENT, "desc must not be NULL");
  std::memset(d, 0, sizeof(*d));
  d->group_m = 8;         // TBOps.td:45 DefaultValuedAttr<I64Attr, "8">
  d->exact_tile = 1;      // TBOps.td:46 DefaultValuedAttr<BoolAttr, "true">
  d->split_k = 1;         // ProgramMappingPlan.cpp:333
  d->num_ctas = 1;        // ProgramMappingPlan.cpp:331
  d->persistent = 0;
  d->programs_per_tile = 0;
  d->reduction_mode = TB_REDUCTION_UNSET;
  d->a_dtype = TB_F16;
  d->b_dtype = TB_F16;
  d->c_dtype = TB_F32;
  d->beta = 1;
  d->num_warps = 4;
  d->num_stages = 2;
  d->bias = 0;
  d->activation = TB_ACT_NONE;
  d->clamp = 0;
  d->clamp_lo = 0.f;
  d->clamp_hi = 0.f;
  d->a_col_major = 0;
  d->b_col_major = 0;
  d->deterministic = 0;
  return TB_OK;
}

static tbStatus validate_kernel_config(const tb_matmul_desc& d) {
  // KernelConfig.cpp:204-207. f16 C is this build's extension.
  if (d.a_dtype != TB_F16 || d.b_dtype != TB_F16 ||
      (d.c_dtype != TB_F32 && d.c_dtype != TB_F16))
    return tb_fail(TB_ERR_INVALID_ARGUMENT,
                   "stage1 currently supports fp16 x fp16 -> fp32 matmul kernels");
  if (d.m == TB_DIM_DYNAMIC || d.n == TB_DIM_DYNAMIC || d.k == TB_DIM_DYNAMIC)  // KernelConfig.cpp:98-103
    return tb_fail(TB_ERR_INVALID_ARGUMENT,
                   "stage1 supported envelope currently requires static rank-2 memrefs to "
                   "derive problem shape coverage");
  if (d.m <= 0 || d.n <= 0 || d.k <= 0)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "problem M/N/K must be positive");
  if (d.block_m <= 0 || d.block_n <= 0 || d.block_k <= 0)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "block M/N/K must be positive");
  if (d.block_m % 16 != 0 || d.block_n % 8 != 0 || d.block_k % 16 != 0)
    return tb_fail(TB_ERR_INVALID_ARGUMENT,
                   "stage1 requires block_m % 16 == 0, block_n % 8 == 0 and "
                   "block_k % 16 == 0 for mma.sync m16n8k16 legality");
  if (d.num_stages < 2 || d.num_stages > 4)
    return tb_fail(TB_ERR_INVALID_ARGUMENT,
                   "stage1 currently supports num_stages in [2, 4]");
  if (d.num_warps <= 0)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "num_warps must be positive");
  if (d.group_m <= 0)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "group_m must be positive");
  if (d.exact_tile && ((d.m % d.block_m) != 0 || (d.n % d.block_n) != 0 ||
                       (d.k % d.block_k) != 0))
    return tb_fail(TB_ERR_INVALID_ARGUMENT,
                   "exact_tile=true requires problem M/N/K to be divisible by "
                   "block M/N/K");
  return TB_OK;
}

extern "C" tbStatus tb_matmul_plan_create(const tb_matmul_desc* desc, int device,
                                          tb_matmul_plan** out) {
  tb_clear_error();
  if (!desc || !out)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "desc and plan must not be NULL");
  *out = nullptr;
  const tb_matmul_desc& d = *desc;
  tbStatus st = validate_kernel_config(d);
  if (st != TB_OK) return st;

  int num_sms = kDefaultB200Sms;
  if (device >= 0) {
    int n = 0;
    cudaError_t e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess)
      return tb_fail(TB_ERR_CUDA, std::string("cudaDeviceGetAttribute: ") +
                                      cudaGetErrorString(e));
    num_sms = n;
  }
  tb_matmul_plan* heap = new (std::nothrow) tb_matmul_plan();
  if (!heap) return tb_fail(TB_ERR_INVALID_ARGUMENT, "out of host memory");
  st = tb_plan_build(d, device, num_sms, heap);
  if (st != TB_OK) {
    delete heap;
    return st;
  }
  *out = heap;
  return TB_OK;
}

tbStatus tb_plan_build(const tb_matmul_desc& d, int device, int num_sms, tb_matmul_plan* out) {
  tbStatus st = validate_kernel_config(d);
  if (st != TB_OK) return st;
  tb_matmul_plan& p = *out;
  p.desc = d;
  p.device = device;
  p.num_sms = num_sms;

  // ---- deriveProgramMappingPlan (ProgramMappingPlan.cpp:329-458) ----
  const int64_t tiles_m = ceil_div(d.m, d.block_m);
  const int64_t tiles_n = ceil_div(d.n, d.block_n);
  const int64_t tiles_k = ceil_div(d.k, d.block_k);
  int64_t group_m = std::max<int64_t>(1, d.group_m);
  int64_t span_m = 1, span_n = tiles_n;
  int64_t ppg = span_m * span_n;
  int64_t launch_groups = tiles_m;
  int64_t total = tiles_m * tiles_n;
  const int64_t split_k = std::max<int64_t>(d.split_k, 1);  // :361
  int64_t num_ctas = d.num_ctas;
  int64_t programs_per_tile = 1;

  if (d.persistent && split_k != 1)
    return tb_fail(TB_ERR_INVALID_ARGUMENT,
                   "stage1 does not allow persistent and split-k in the same "
                   "program mapping contract yet");
  if (num_ctas <= 0)
    return tb_fail(TB_ERR_INVALID_ARGUMENT,
                   "module attr `tb.num-ctas` must be positive");
  if (d.programs_per_tile > 0) programs_per_tile = d.programs_per_tile;
  if (d.reduction_mode != TB_REDUCTION_UNSET &&
      d.reduction_mode != TB_REDUCTION_SPLIT_K_SERIAL &&
      d.reduction_mode != TB_REDUCTION_SPLIT_K_PARALLEL)
    return tb_fail(TB_ERR_INVALID_ARGUMENT,
                   "module attr `tb.reduction-mode` must be `split_k_serial` or "
                   "`split_k_parallel`");

  int32_t kind;
  std::string reduction = "none";
  if (d.persistent) {
    kind = tb::kMapPersistentTile;
    p.mapping_kind = "persistent_tile";
    p.launch_order = "persistent";
    p.swizzle_kind = "none";
    group_m = 1;
    span_m = 1;
    span_n = tiles_n;
    ppg = span_n;
    launch_groups = tiles_m;
    total = tiles_m * tiles_n;
    programs_per_tile = 1;
    num_ctas = std::min<int64_t>(num_ctas, total);
  } else if (split_k > 1) {
    kind = tb::kMapSplitK;
    p.mapping_kind = "split_k";
    p.launch_order = "row_major";
    p.swizzle_kind = "none";
    group_m = 1;
    span_m = 1;
    span_n = tiles_n * split_k;
    ppg = span_n;
    launch_groups = tiles_m;
    total = tiles_m * tiles_n * split_k;
    programs_per_tile = split_k;
    if (d.reduction_mode == TB_REDUCTION_SPLIT_K_PARALLEL)
      reduction = "split_k_atomic";      // ReductionPlan.cpp:176-182
    else
      reduction = "split_k_serial";      // ReductionPlan.cpp:169-175
  } else if (group_m > 1 && tiles_m > 1 && tiles_n > 1) {
    kind = tb::kMapGroupedTile;
    p.mapping_kind = "grouped_tile";
    p.launch_order = "grouped_m";
    p.swizzle_kind = "grouped_m";
    span_m = group_m;
    span_n = tiles_n;
    ppg = span_m * span_n;
    launch_groups = ceil_div(tiles_m, group_m);
    total = tiles_m * tiles_n;
  } else {
    kind = tb::kMapTile;
    p.mapping_kind = "tile";
    p.launch_order = "row_major";
    p.swizzle_kind = "none";
    group_m = 1;
    span_m = 1;
    span_n = tiles_n;
    ppg = span_n;
    launch_groups = tiles_m;
    total = tiles_m * tiles_n;
  }
  // ProgramMappingPlan.cpp:446-449: the target's limit is 8 warps per CTA
  // (maxWarpsPerCTA, TargetInfo.cpp:126), checked whenever the SM count is known.
  if (num_sms > 0 && d.num_warps > kMaxWarpsPerCta)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "num_warps exceeds target max warps per CTA");
  if (d.persistent && num_ctas > num_sms) num_ctas = num_sms;  // :450-453

  if (total > std::numeric_limits<int32_t>::max() ||
      tiles_k > std::numeric_limits<int32_t>::max())
    return tb_fail(TB_ERR_UNSUPPORTED, "program count exceeds 2^31-1");

  // deriveWarpGrid failure is a layout-plan error in the reference.
  int64_t wgm = 0, wgn = 0;
  if (!derive_warp_grid(d.num_warps, d.block_m, d.block_n, &wgm, &wgn))
    return tb_fail(TB_ERR_INVALID_ARGUMENT,
                   "failed to derive a legal warp grid from module num-warps, "
                   "block shape and mma instruction shape");

  p.map.kind = kind;
  p.map.tiles_m = (int32_t)tiles_m;
  p.map.tiles_n = (int32_t)tiles_n;
  p.map.tiles_k = (int32_t)tiles_k;
  p.map.group_span_m = (int32_t)span_m;
  p.map.programs_per_group = (int32_t)ppg;
  p.map.split_k = (int32_t)split_k;
  p.map.total_programs = (int32_t)total;
  p.reduction_kind = reduction;
  p.launch_group_count = launch_groups;
  p.group_tile_span_n = span_n;
  p.programs_per_tile = programs_per_tile;
  p.num_ctas = num_ctas;
  p.resident_programs = d.persistent ? std::max<int64_t>(1, std::min<int64_t>(num_ctas, num_sms)) : 1;
  p.warp_grid_m = wgm;
  p.warp_grid_n = wgn;
  if (d.persistent) p.mainline_kind = "persistent_tile_loop";
  else if (split_k > 1) p.mainline_kind = "split_k";
  else if (kind == tb::kMapGroupedTile) p.mainline_kind = "grouped_tile";
  else p.mainline_kind = "single_tile";

  // ---- this build's hardware tile: tcgen05 M=128 on one CTA, or M=256 on a
  //      CTA pair (cta_group::2); N ∈ {64, 128, 256, 512} ----
  // A program tile larger than every hardware tile (block_m > 256 or
  // block_n > 512; KernelConfig.cpp:217-221 only asks for multiples of 16 /
  // 8) runs as sub_m × sub_n hardware work items that together cover it;
  // each computes its part of the program's tile over the program's K range.
  const bool big = d.block_m > 256 || d.block_n > 512;
  // Consecutive program ids in grouped order are vertically adjacent tiles
  // (LowerPipelineToNVGPU.cpp:283-304: tile_m advances fastest inside a
  // group), and in row-major / persistent order horizontally adjacent. When
  // every such pair is aligned, two programs share one hardware tile (half
  // the operand traffic per FLOP); a 32-bit program walk stays the same.
  p.fuse = 0;
  if (!big && split_k == 1 && total % 2 == 0) {
    // 2 × 2 blocks of programs no larger than 128 × 128 make one 256 × 256
    // pair tile (measured 4096³ with 128 × 128 programs: 119 → 112 µs), when
    // every CTA pair still gets a work item.
    if (kind == tb::kMapGroupedTile && span_m % 2 == 0 && tiles_m % 2 == 0 && tiles_n % 2 == 0 &&
        2 * d.block_m <= 256 && 2 * d.block_n <= 256 && d.block_n > 64 &&
        total / 4 >= std::max<int64_t>(1, num_sms / 2))
      p.fuse = 4;
    else if (kind == tb::kMapGroupedTile && span_m % 2 == 0 && tiles_m % 2 == 0 && 2 * d.block_m <= 256)
      p.fuse = 1;
    // 256-row programs at most 128 wide, side by side in grouped order, make
    // one 256 × 256 pair tile (4096³ with 256 × 128 programs: 134 → 108 µs)
    else if (kind == tb::kMapGroupedTile && tiles_n % 2 == 0 && d.block_m > 128 &&
             2 * d.block_n <= 256 && d.block_n > 64 && total / 2 >= std::max<int64_t>(1, num_sms / 2))
      p.fuse = 3;
    else if ((kind == tb::kMapTile || kind == tb::kMapPersistentTile) && tiles_n % 2 == 0 &&
             2 * d.block_n <= 256)
      p.fuse = 2;
  }
  p.work_items = p.fuse == 4 ? total / 4 : p.fuse ? total / 2 : total;
  const int64_t eff_bm = d.block_m * (p.fuse == 1 || p.fuse == 4 ? 2 : 1);
  const int64_t eff_bn = d.block_n * (p.fuse >= 2 ? 2 : 1);
  p.sub_m = p.sub_n = 1;
  if (big) {
    // Pair tiles for programs taller than 128 rows, else one-CTA 128-row
    // tiles; the widest tile no wider than the program (256 × 512 only for
    // programs at most 512 wide, where it covers the width in one item).
    if (d.block_m > 128) {
      p.cta_m = 256;
      p.ctas_per_tile = 2;
      if (d.block_n <= 128) { p.kernel_tile = kTile256x128; p.cta_n = 128; }
      else if (d.block_n <= 256 || d.block_n > 512) { p.kernel_tile = kTile256x256; p.cta_n = 256; }
      else { p.kernel_tile = kTile256x512; p.cta_n = 512; }
    } else {
      p.cta_m = 128;
      p.ctas_per_tile = 1;
      p.kernel_tile = kTile128x256;
      p.cta_n = 256;
    }
    p.sub_m = (int32_t)ceil_div(d.block_m, p.cta_m);
    p.sub_n = (int32_t)ceil_div(d.block_n, p.cta_n);
    if (total * p.sub_m * p.sub_n > std::numeric_limits<int32_t>::max())
      return tb_fail(TB_ERR_UNSUPPORTED, "hardware work items exceed 2^31-1");
    p.work_items = total * p.sub_m * p.sub_n;
  } else if (eff_bn > 256) {  // 256 × 512 CTA pair (256 < block_n <= 512)
    // Pairing never builds a 256 × 512 tile: its single accumulator leaves
    // the epilogue exposed (measured 5 % slower than 256 × 256 at 8192³).
    p.cta_m = 256;
    p.ctas_per_tile = 2;
    p.kernel_tile = kTile256x512;
    p.cta_n = 512;
  } else if (eff_bm <= 128) {
    p.cta_m = 128;
    p.ctas_per_tile = 1;
    if (eff_bn <= 64) { p.kernel_tile = kTile128x64; p.cta_n = 64; }
    else if (eff_bn <= 128) { p.kernel_tile = kTile128x128; p.cta_n = 128; }
    else { p.kernel_tile = kTile128x256; p.cta_n = 256; }
  } else {
    p.cta_m = 256;
    p.ctas_per_tile = 2;
    if (eff_bn <= 128) { p.kernel_tile = kTile256x128; p.cta_n = 128; }
    else { p.kernel_tile = kTile256x256; p.cta_n = 256; }
  }
  // The ring is as deep as shared memory allows and never shallower than
  // tb.requested-stages.
  p.stages = std::max<int32_t>((int32_t)d.num_stages, tb_kernel_max_stages(p.kernel_tile));
  p.smem_bytes = tb_kernel_smem_bytes(p.kernel_tile, p.stages);
  p.kb = tb_kernel_kb(p.kernel_tile);
  // two accumulators (epilogue/mainloop overlap), or one that fills TMEM
  p.tmem_cols = std::min<int32_t>(2 * p.cta_n, 512);

  if (d.activation < TB_ACT_NONE || d.activation > TB_ACT_GELU_TANH)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "unknown epilogue activation");
  if (d.clamp && !(d.clamp_lo <= d.clamp_hi))
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "epilogue clamp needs clamp_lo <= clamp_hi");
  const bool exprs = d.bias || d.activation != TB_ACT_NONE || d.clamp;
  if (exprs && split_k > 1 && d.reduction_mode == TB_REDUCTION_SPLIT_K_PARALLEL)
    return tb_fail(TB_ERR_UNSUPPORTED,
                   "fused epilogue expressions need the complete sum: use split_k_serial "
                   "(split_k_parallel adds partials into C)");
  if (split_k > 1) {
    if (d.reduction_mode == TB_REDUCTION_SPLIT_K_PARALLEL) {
      if (d.c_dtype != TB_F32)
        return tb_fail(TB_ERR_UNSUPPORTED,
                       "split_k_parallel accumulates with f32 atomics; f16 C "
                       "needs split_k_serial");
      p.epilogue = kEpiAtomic;
      p.workspace_bytes = 0;
    } else {
      p.epilogue = kEpiWorkspace;
      p.workspace_bytes = (size_t)split_k * (size_t)d.m * (size_t)d.n * sizeof(float);
    }
  } else {
    p.epilogue = kEpiStore;
    p.workspace_bytes = 0;
  }
  // Operands whose contiguous rows are not a multiple of 8 elements (16 bytes)
  // cannot be read by TMA in place: reserve room for a zero-padded copy.
  {
    auto align256 = [](size_t x) { return (x + 255) & ~(size_t)255; };
    const int64_t a_rows = d.a_col_major ? d.k : d.m, a_cols = d.a_col_major ? d.m : d.k;
    const int64_t b_rows = d.b_col_major ? d.n : d.k, b_cols = d.b_col_major ? d.k : d.n;
    p.partial_bytes = p.workspace_bytes;
    p.pack_a_bytes = a_cols % 8 ? (size_t)a_rows * (size_t)((a_cols + 7) / 8 * 8) * 2 : 0;
    p.pack_b_bytes = b_cols % 8 ? (size_t)b_rows * (size_t)((b_cols + 7) / 8 * 8) * 2 : 0;
    p.pack_a_offset = align256(p.partial_bytes);
    p.pack_b_offset = p.pack_a_offset + align256(p.pack_a_bytes);
    if (p.pack_b_bytes) p.workspace_bytes = p.pack_b_offset + p.pack_b_bytes;
    else if (p.pack_a_bytes) p.workspace_bytes = p.pack_a_offset + p.pack_a_bytes;
    else p.workspace_bytes = p.partial_bytes;
  }
  // Resident program slots: one per SM, or one per SM pair for CTA pairs.
  const int64_t slots = std::max<int64_t>(1, num_sms / p.ctas_per_tile);
  const int64_t resident = d.persistent ? std::min<int64_t>(p.resident_programs, slots) : slots;
  // Tail balancing: when the work items leave the last wave of resident
  // slots partly idle (e.g. 128 items of 256 × 256 on 74 CTA pairs), the
  // last items are cut into K pieces that fill the idle slots.
  p.dp_items = p.work_items;
  p.tail_items = 0;
  p.tail_segs = 0;
  p.tail_slots = 0;
  p.tail_fills = 0;
  const bool exact_hw = d.block_m * (p.fuse == 1 || p.fuse == 4 ? 2 : 1) == (int64_t)p.cta_m * p.sub_m &&
                        d.block_n * (p.fuse >= 2 ? 2 : 1) == (int64_t)p.cta_n * p.sub_n;
  if (!d.deterministic && split_k == 1 && d.c_dtype == TB_F32 && d.beta && !exprs && exact_hw)
    tb_choose_tail_split(p.work_items, resident, ceil_div(d.k, p.kb), &p.dp_items, &p.tail_items,
                         &p.tail_segs);
  if (p.tail_items) {
    p.tail_slots = resident;
    p.tail_fills = ceil_div(d.k, p.kb);
  }
  p.positions = p.dp_items + p.tail_segs * p.tail_slots;
  p.grid = p.ctas_per_tile * std::max<int64_t>(1, std::min<int64_t>(p.positions, resident));
  // Small problems (every item's K range within 128 elements on a one-CTA
  // tile at most 128 wide) are launch- and latency-bound: they run on the
  // latency kernel, which skips the tensor maps and the warp-role pipeline.
  const int64_t k_item = std::min<int64_t>(d.k, ceil_div(tiles_k, split_k) * d.block_k);
  p.small = !big && p.ctas_per_tile == 1 && p.cta_n <= 128 && k_item <= 128 && !d.a_col_major &&
            !d.b_col_major && p.tail_items == 0 && p.positions <= 4 * (p.grid / p.ctas_per_tile);
  if (p.small) {
    p.stages = 1;
    p.kb = 128;
    p.smem_bytes = tb_small_smem_bytes(p.cta_n, d.c_dtype);
    p.tmem_cols = p.cta_n;
  }

  return TB_OK;
}

extern "C" tbStatus tb_matmul_plan_destroy(tb_matmul_plan* plan) {
  delete plan;
  return TB_OK;
}

extern "C" size_t tb_matmul_workspace_bytes(const tb_matmul_plan* plan) {
  return plan && !plan->dynamic ? plan->workspace_bytes : 0;
}

extern "C" tbStatus tb_matmul_program_work(const tb_matmul_plan* plan, int64_t pid,
                                           tb_program_work* w) {
  if (!plan || !w) return tb_fail(TB_ERR_INVALID_ARGUMENT, "plan and work must not be NULL");
  if (plan->dynamic)
    return tb_fail(TB_ERR_INVALID_ARGUMENT,
                   "program work of a dynamic plan: take tb_matmul_plan_for_shape first");
  if (pid < 0 || pid >= plan->map.total_programs)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "program id out of range");
  const tb::Work x = tb::program_work(plan->map, (int32_t)pid);
  w->tile_m = x.tile_m;
  w->tile_n = x.tile_n;
  w->split_part = x.part;
  w->k_tile_begin = x.kt_begin;
  w->k_tile_count = x.kt_count;
  return TB_OK;
}

extern "C" tbStatus tb_matmul_plan_describe(const tb_matmul_plan* plan, char* buf,
                                            size_t len, size_t* needed) {
  if (!plan) return tb_fail(TB_ERR_INVALID_ARGUMENT, "plan must not be NULL");
  if (plan->dynamic) {
    const std::string s = tb_describe_dynamic(plan);
    if (needed) *needed = s.size() + 1;
    if (!buf || len < s.size() + 1)
      return tb_fail(TB_ERR_INVALID_ARGUMENT, "describe buffer too small");
    std::memcpy(buf, s.c_str(), s.size() + 1);
    return TB_OK;
  }
  const tb_matmul_desc& d = plan->desc;
  const char* small_names[] = {"tb_gemm_sm100_small_128x64", "tb_gemm_sm100_small_128x128"};
  const char* kernel_names[] = {"tb_gemm_sm100_128x64", "tb_gemm_sm100_128x128",
                                "tb_gemm_sm100_128x256", "tb_gemm_sm100_pair_256x128",
                                "tb_gemm_sm100_pair_256x256", "tb_gemm_sm100_pair_256x512"};
  const char* epi_names[] = {"store", "workspace_partial", "atomic_add"};
  std::ostringstream o;
  o << "{";
  o << "\"problem\": [" << d.m << ", " << d.n << ", " << d.k << "], ";
  o << "\"tile\": [" << d.block_m << ", " << d.block_n << ", " << d.block_k << "], ";
  o << "\"dtypes\": \"" << dtype_name(d.a_dtype) << "x" << dtype_name(d.b_dtype)
    << "->" << dtype_name(d.c_dtype) << "\", ";
  o << "\"exact_tile\": " << (d.exact_tile ? "true" : "false") << ", ";
  o << "\"num_warps\": " << d.num_warps << ", ";
  o << "\"requested_stages\": " << d.num_stages << ", ";
  o << "\"warp_grid\": [" << plan->warp_grid_m << ", " << plan->warp_grid_n << "], ";
  o << "\"mapping_kind\": \"" << plan->mapping_kind << "\", ";
  o << "\"launch_order\": \"" << plan->launch_order << "\", ";
  o << "\"swizzle_kind\": \"" << plan->swizzle_kind << "\", ";
  o << "\"problem_tiles\": [" << plan->map.tiles_m << ", " << plan->map.tiles_n
    << ", " << plan->map.tiles_k << "], ";
  o << "\"group_m\": " << (plan->map.kind == tb::kMapGroupedTile ? plan->map.group_span_m : 1) << ", ";
  o << "\"group_tile_span_m\": " << plan->map.group_span_m << ", ";
  o << "\"group_tile_span_n\": " << plan->group_tile_span_n << ", ";
  o << "\"programs_per_launch_group\": " << plan->map.programs_per_group << ", ";
  o << "\"launch_group_count\": " << plan->launch_group_count << ", ";
  o << "\"total_programs\": " << plan->map.total_programs << ", ";
  o << "\"split_k\": " << plan->map.split_k << ", ";
  o << "\"programs_per_tile\": " << plan->programs_per_tile << ", ";
  o << "\"reduction_kind\": \"" << plan->reduction_kind << "\", ";
  o << "\"persistent\": " << (d.persistent ? "true" : "false") << ", ";
  o << "\"persistent_kind\": \"" << (d.persistent ? "tile_stride_loop" : "none") << "\", ";
  o << "\"num_ctas\": " << plan->num_ctas << ", ";
  o << "\"resident_programs\": " << plan->resident_programs << ", ";
  o << "\"selected_mainline_kind\": \"" << plan->mainline_kind << "\", ";
  o << "\"num_sms\": " << plan->num_sms << ", ";
  o << "\"kernel\": \""
    << (plan->small ? small_names[plan->kernel_tile == kTile128x64 ? 0 : 1] : kernel_names[plan->kernel_tile])
    << "\", ";
  o << "\"cta_tile\": [" << plan->cta_m << ", " << plan->cta_n << ", " << plan->kb << "], ";
  o << "\"ctas_per_tile\": " << plan->ctas_per_tile << ", ";
  o << "\"fused_program_pairs\": \""
    << (plan->fuse == 1 ? "vertical" : plan->fuse == 2 || plan->fuse == 3 ? "horizontal"
        : plan->fuse == 4 ? "2x2" : "none")
    << "\", ";
  o << "\"work_items\": " << plan->work_items << ", ";
  o << "\"program_subtiles\": [" << plan->sub_m << ", " << plan->sub_n << "], ";
  o << "\"tail_split\": ";
  if (plan->tail_items)
    o << "{\"whole_items\": " << plan->dp_items << ", \"stream_k_items\": " << plan->tail_items
      << ", \"slots\": " << plan->tail_slots << ", \"segments_per_slot\": " << plan->tail_segs
      << ", \"fills_per_item\": " << plan->tail_fills << "}, ";
  else
    o << "null, ";
  o << "\"walk_positions\": " << plan->positions << ", ";
  {
    const char* walks[] = {"program_order", "row_groups", "serpentine_groups"};
    o << "\"hardware_walk\": \"" << walks[tb::walk_mode(plan->map, plan->fuse)] << "\", ";
  }
  o << "\"stages\": " << plan->stages << ", ";
  o << "\"smem_bytes\": " << plan->smem_bytes << ", ";
  o << "\"tmem_cols\": " << plan->tmem_cols << ", ";
  o << "\"grid\": " << plan->grid << ", ";
  o << "\"block_threads\": 192, ";
  o << "\"epilogue\": \"" << epi_names[plan->epilogue] << "\", ";
  o << "\"beta\": " << d.beta << ", ";
  o << "\"a_layout\": \"" << (d.a_col_major ? "col_major" : "row_major") << "\", ";
  o << "\"b_layout\": \"" << (d.b_col_major ? "col_major" : "row_major") << "\", ";
  {
    // the reference's EpilogueExprKind spelling, in application order
    const char* acts[] = {"", "activation(relu)", "activation(silu)", "activation(gelu_tanh)"};
    o << "\"epilogue_exprs\": [";
    bool first = true;
    auto item = [&](const std::string& x) { o << (first ? "" : ", ") << "\"" << x << "\""; first = false; };
    if (d.beta) item("add(c_in)");
    if (d.bias) { item("load_bias"); item("add"); }
    if (d.activation) item(acts[d.activation]);
    if (d.clamp) item("clamp");
    if (d.c_dtype == TB_F16) item("convert(f16)");
    o << "], ";
  }
  o << "\"workspace_bytes\": " << plan->workspace_bytes;
  o << "}";
  const std::string s = o.str();
  if (needed) *needed = s.size() + 1;
  if (!buf || len < s.size() + 1)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "describe buffer too small");
  std::memcpy(buf, s.c_str(), s.size() + 1);
  return TB_OK;
}

extern "C" tbStatus tb_matmul_run(const tb_matmul_plan* plan, const void* A, int64_t lda,
                                  const void* B, int64_t ldb, void* C, int64_t ldc,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  tb_clear_error();
  if (!plan) return tb_fail(TB_ERR_INVALID_ARGUMENT, "plan must not be NULL");
  return tb_launch(plan, A, lda, B, ldb, C, ldc, workspace, workspace_bytes, stream);
}

extern "C" tbStatus tb_matmul_run_epilogue(const tb_matmul_plan* plan, const void* A, int64_t lda,
                                           const void* B, int64_t ldb, void* C, int64_t ldc,
                                           const float* bias, void* workspace,
                                           size_t workspace_bytes, void* stream) {
  tb_clear_error();
  if (!plan) return tb_fail(TB_ERR_INVALID_ARGUMENT, "plan must not be NULL");
  return tb_launch_ex(plan, A, lda, B, ldb, C, ldc, bias, workspace, workspace_bytes, stream);
}

extern "C" tbStatus tb_matmul(const tb_matmul_desc* desc, const void* A, int64_t lda,
                              const void* B, int64_t ldb, void* C, int64_t ldc,
                              void* workspace, size_t workspace_bytes, void* stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return tb_fail(TB_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  tb_matmul_plan* plan = nullptr;
  tbStatus st = tb_matmul_plan_create(desc, dev, &plan);
  if (st != TB_OK) return st;
  st = tb_matmul_run(plan, A, lda, B, ldb, C, ldc, workspace, workspace_bytes, stream);
  tb_matmul_plan_destroy(plan);
  return st;
}
