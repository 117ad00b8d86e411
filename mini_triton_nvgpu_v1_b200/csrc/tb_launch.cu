// tb_launch.cu — the sm_100a `tb.matmul` kernels and their launcher.
//
// One kernel family replaces the reference's generated
// `kernel_tb_kernel_0` (cp.async → ldmatrix → mma.sync, statically unrolled
// over K/16; LowerPipelineToNVGPU.cpp:2019-2607) with a warp-specialised,
// persistent tcgen05 pipeline:
//
//   warp 0 (one lane)  TMA producer: A box [128 × 64] (K-major) and B boxes
//                      [64 × 64] (N-major), both 128-byte swizzled, into an
//                      S-deep shared-memory ring guarded by full/empty
//                      mbarriers.
//   warp 1 (one lane)  MMA issuer: tcgen05.mma kind::f16, M=128, N=BN, K=16
//                      per instruction into one of two TMEM accumulators;
//                      tcgen05.commit frees ring stages and publishes tiles.
//   warps 2-5          epilogue: tcgen05.ld TMEM → registers, adds C_in
//                      (the reference's C-init, :2192-2278), masked stores
//                      (the boundary-aware epilogue, EpiloguePlan.cpp:864-979),
//                      or split-K partial / atomic output (:1862-1912).
//
// Each CTA walks program ids pid = blockIdx.x, blockIdx.x + gridDim.x, …
// and maps each with tb::program_work — the reference's mapping formulas —
// so tile, grouped, split-K and persistent mappings compute exactly the
// reference's (tile, split part) set. Double-buffered TMEM lets the
// epilogue of one program overlap the mainloop of the next.
//
// Every wait is bounded: when a wait runs past kWaitBudgetCycles the thread
// records TB_ERR_DEVICE_TIMEOUT in g_tb_status, raises a CTA-wide abort flag
// and every role leaves its loop; in-flight TMA loads and MMAs are drained
// (with bounded waits) before TMEM is released.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <type_traits>
#include <cstring>
#include <cstdio>
#include <mutex>
#include <string>

#include "tb_plan.h"
#include "tb_sm100.cuh"

using namespace tb::sm100;

__device__ uint32_t g_tb_status = 0;

namespace {

constexpr int kThreads = 192;
constexpr int kCtaM = 128;            // tcgen05 M per CTA
constexpr size_t kSmemLimit = 232448;  // 227 KB opt-in per CTA
constexpr long long kWaitBudgetCycles = 2000000000LL;  // ≈1 s at 1.9 GHz

constexpr uint32_t kSiteProducer = 1, kSiteMma = 2, kSiteEpilogue = 3, kSiteDrain = 4,
                   kSiteSelfTest = 5;

// G = CTAs per tile: 1 (cta_group::1, 128-row tile) or 2 (cta_group::2 pair,
// 256-row tile; each CTA holds 128 rows of A, BN/2 columns of B and 128
// rows of the accumulator).
// KB = K elements per ring stage: 64, or 128 when a CTA holds only 64 B
// columns (its short MMA stages would otherwise be paced by the per-stage
// barrier handshake; 8 MMAs per stage amortise it: measured −15 % time for
// 128×64 and −9 % for the 256×128 pair at 8192³; 128×128 is L2-feed bound
// and gains nothing).
// BN = 512 (CTA pair only, for 256 < block_n <= 512): two N = 256 MMAs per
// K step share each A tile (25 % less L2→SM operand traffic per FLOP than
// 256 × 256); its accumulator fills TMEM, so there is one accumulator and the
// epilogue does not overlap the next tile's MMAs.
template <int BN, int G>
struct Cfg {
  static constexpr int kBnCta = BN / G;                  // B columns per CTA
  static constexpr int kMmaN = BN > 256 ? 256 : BN;      // N of one tcgen05.mma
  static constexpr int kMmaPerK = BN / kMmaN;            // MMAs per K step (1 or 2)
  static constexpr int kAccs = 2 * BN <= 512 ? 2 : 1;    // TMEM accumulators
  // B bytes per CTA feeding one MMA of a K step (the second MMA's B starts
  // this far into the stage: MN-major box 2, or K-major row 128).
  static constexpr uint32_t kBHalf = (uint32_t)(kBnCta / kMmaPerK) * 64 * 2;
  static constexpr int kKB = kBnCta <= 64 ? 128 : 64;
  static constexpr uint32_t kABytes = kCtaM * kKB * 2;   // KB/64 K-major [128 × 64] sub-tiles
  static constexpr uint32_t kASub = kCtaM * 64 * 2;      // one K-major A sub-tile
  static constexpr uint32_t kBoxBytes = 64 * kKB * 2;    // one MN-major [KB k × 64 mn] box
  static constexpr uint32_t kBSub = kBnCta * 64 * 2;     // one K-major B sub-tile
  static constexpr uint32_t kBBytes = kBnCta * kKB * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  // f32 output staging for the TMA-store epilogue: 4 warps × 2 buffers of
  // [32 rows × 32 f32] (128-byte swizzled rows).
  static constexpr uint32_t kEpiBufBytes = 32 * 32 * 4;
  static constexpr uint32_t kEpiBytes = 4 * 2 * kEpiBufBytes;
  static constexpr int kRawStages = (int)((kSmemLimit - 1024 - 512 - kEpiBytes) / kStageBytes);
  static constexpr int kCap = 8;
  static constexpr int kStages = kRawStages > kCap ? kCap : kRawStages;
  static constexpr uint32_t kTmemCols = kAccs * BN;  // kAccs accumulators of BN f32 columns
  static constexpr size_t kSmem = 1024 + (size_t)kStages * kStageBytes + kEpiBytes + 512;
  static_assert(kBnCta % 64 == 0, "B columns per CTA must be whole 64-column boxes");
  static_assert(kMmaPerK == 1 || (G == 2 && kKB == 64), "BN = 512 is a CTA-pair tile");
  static_assert(kTmemCols == 128 || kTmemCols == 256 || kTmemCols == 512, "TMEM columns");
};

// How the epilogue hands a finished f32 [32 × 32] chunk to memory.
enum TmaOut : int32_t {
  kTmaNone = 0,      // direct per-thread stores
  kTmaStoreC = 1,    // TMA store into C        (kEpiStore)
  kTmaReduceC = 2,   // TMA reduce-add into C   (kEpiAtomic)
  kTmaStoreWs = 3,   // TMA 3-D store into the [S][M][N] workspace (kEpiWorkspace)
};

// Fused epilogue expressions (EpilogueExprKind: LoadBias/Add, Activation,
// Clamp), applied to the complete f32 sum before the output conversion.
struct EpiExprs {
  const float* bias;  // per column, or null
  int32_t act;        // tbActivation
  int32_t clamp;
  float lo, hi;
  int32_t any;
};

__device__ __forceinline__ float apply_exprs(const EpiExprs& x, float v, int64_t col) {
  if (x.bias) v += __ldg(x.bias + col);
  if (x.act == TB_ACT_RELU) {
    v = fmaxf(v, 0.f);
  } else if (x.act == TB_ACT_SILU) {
    v = v / (1.f + __expf(-v));
  } else if (x.act == TB_ACT_GELU_TANH) {
    // 0.5·v·(1 + tanh(sqrt(2/π)·(v + 0.044715·v³)))
    v = 0.5f * v * (1.f + tanhf(0.7978845608f * (v + 0.044715f * v * v * v)));
  }
  if (x.clamp) v = fminf(fmaxf(v, x.lo), x.hi);
  return v;
}

struct KParams {
  tb::MappingArgs map;
  int32_t M, N, K;
  int32_t block_m, block_n, block_k;
  int32_t epilogue;  // TbEpilogue
  int32_t beta;
  int32_t vec_c;     // C rows allow 16-byte vector access
  int32_t vec_ws;    // workspace rows allow 16-byte vector access
  int32_t tma_out;   // TmaOut: f32 tile output written by TMA from swizzled shared staging
  int32_t fuse;      // program pairing (plan.fuse): work item w runs programs 2w and 2w+1
  int32_t cin_smem;  // one work item per CTA: the epilogue stages C_in through the idle ring
  int32_t one_item;  // every CTA (pair) runs at most one work item: the ring is idle in its epilogue
  int32_t walk_grouped;  // tb::WalkMode: the order resident CTAs take work items in
  int32_t work_items;    // hardware work items (programs × sub-tiles, or fused programs)
  int32_t positions;     // walk positions: dp_items + tail_segs · tail_slots
  int32_t sub_m, sub_n;  // hardware tiles per program along M / N (programs larger than a tile)
  // Stream-K tail (tb_choose_tail_split): positions [0, dp_items) run whole
  // work items; the last tail_items items are one run of tail_items ·
  // tail_fills ring fills cut into tail_slots equal ranges, the slot of
  // position dp_items + s·tail_slots + q being q and s its segment.
  int32_t dp_items, tail_items, tail_slots, tail_segs, tail_fills;
  EpiExprs ex;       // applied in kEpiStore (split_k_serial: in the reduction)
  int32_t a_mn;      // A stored M-major (column-major m × k): MN-major UMMA operand
  int32_t b_kmaj;    // B stored K-major (column-major k × n): K-major UMMA operand
  void* C;
  int64_t ldc;
  float* ws;
};

__device__ __forceinline__ void record_error(uint32_t code, uint32_t site) {
  const uint32_t v = (code << 24) | (site << 16) | (blockIdx.x & 0xFFFFu);
  atomicCAS(&g_tb_status, 0u, v);
}

// Bounded wait: false when the abort flag is up or the budget ran out.
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity,
                                             volatile int* abort_flag, uint32_t site) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitBudgetCycles) {
      record_error(TB_ERR_DEVICE_TIMEOUT, site);
      *abort_flag = 1;
      return false;
    }
  }
}

// Lane 0 waits (bounded), the result is broadcast so the warp stays converged.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          uint32_t site, int lane) {
  // Every lane probes first with the non-blocking test_wait: in the common
  // case (phase already complete) that is one probe, while a blocking
  // try_wait costs hundreds of cycles even on a completed phase (measured:
  // 142 → 118 cycles per MMA for a 128×128 tile, 154 → 132 for 128×256).
  if (mbar_test_wait(bar, parity)) return true;
  int ok = 0;
  if (lane == 0) ok = wait_bounded(bar, parity, abort_flag, site);
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

struct Extent {
  int32_t m0, n0, rows, cols, k_begin, k_end, nkb, part;
  bool piece;  // part of a tail work item (stream-K): its partial sum is reduce-added into C
};

// Work of walk position `pos` on a HM × HN hardware tile: its rows and
// columns inside the problem (clipped to its program tile) and its K range;
// nkb counts ring fills of kb K elements.
__host__ __device__ __forceinline__ int32_t imin(int32_t a, int32_t b) { return a < b ? a : b; }

template <int HM, int HN>
__host__ __device__ __forceinline__ Extent program_extent(const KParams& p, int32_t pos, int32_t kb) {
  int32_t w = pos;
  int32_t f0 = 0, f1 = 0;   // the position's fills of its item (stream-K tail)
  const bool tail = pos >= p.dp_items;
  if (tail) {
    const int32_t t = pos - p.dp_items;
    const int32_t seg = t / p.tail_slots, q = t % p.tail_slots;
    const int64_t U = (int64_t)p.tail_items * p.tail_fills;
    const int64_t u0 = (int64_t)q * U / p.tail_slots, u1 = (int64_t)(q + 1) * U / p.tail_slots;
    const int32_t i = (int32_t)(u0 / p.tail_fills) + seg;
    const int64_t b = (int64_t)i * p.tail_fills;
    f0 = (int32_t)((u0 > b ? u0 : b) - b);
    f1 = (int32_t)((u1 < b + p.tail_fills ? u1 : b + p.tail_fills) - b);
    if (i >= p.tail_items) f1 = f0;  // past the run: an empty position
    w = p.dp_items + (i < p.tail_items ? i : p.tail_items - 1);
  }
  const int32_t nsub = p.sub_m * p.sub_n;
  const int32_t sub = w % nsub;
  const int32_t item = tb::walk_item(p.map, p.fuse, p.walk_grouped, w / nsub);
  const tb::Work wk = tb::program_work(p.map, tb::item_first_pid(p.map, p.fuse, item));
  Extent e;
  // A program larger than the hardware tile runs as sub_m × sub_n work
  // items, each [HM × HN] of the program tile (the last ones clipped to it).
  const int32_t sm = (sub / p.sub_n) * HM, sn = (sub % p.sub_n) * HN;
  e.m0 = wk.tile_m * p.block_m + sm;
  e.n0 = wk.tile_n * p.block_n + sn;
  e.rows = imin(p.block_m * (p.fuse == 1 || p.fuse == 4 ? 2 : 1) - sm, p.M - e.m0);
  e.cols = imin(p.block_n * (p.fuse >= 2 ? 2 : 1) - sn, p.N - e.n0);
  if (nsub > 1) {
    e.rows = imin(e.rows, HM);
    e.cols = imin(e.cols, HN);
  }
  e.k_begin = wk.kt_begin * p.block_k;
  e.k_end = imin(p.K, (wk.kt_begin + wk.kt_count) * p.block_k);
  e.nkb = e.k_end > e.k_begin && e.rows > 0 && e.cols > 0 ? (e.k_end - e.k_begin + kb - 1) / kb : 0;
  e.part = wk.part;
  e.piece = false;
  if (tail) {
    if (f1 <= f0) {  // empty (its range ends before this item): no loads, no MMA, no stores
      e.nkb = 0;
      e.cols = 0;
      return e;
    }
    // a partial segment adds its sum into C; a whole item stores as usual
    e.piece = f1 - f0 < e.nkb;
    e.k_end = imin(e.k_end, e.k_begin + f1 * kb);
    e.k_begin += f0 * kb;
    e.nkb = f1 - f0;
  }
  return e;
}

// K chunk the kb-th ring fill of a work item loads. Every other round of a
// resident CTA's walk runs K backwards: the rounds of all CTAs move in step,
// so a round that starts where the last one ended finds the A (or B) panel
// slices it shares with that round still in L2 (measured +1.5 % sustained
// at 8192³, fewer DRAM re-reads). The MMA sums in the same order it loads.
__device__ __forceinline__ int k_chunk(int32_t pid, int32_t first_pid, int32_t pid_stride, int kb,
                                       int nkb) {
  return (((pid - first_pid) / pid_stride) & 1) ? nkb - 1 - kb : kb;
}

template <typename OutT>
struct OutIO;

// C is touched once per tile: loads and stores use the streaming (evict-first)
// cache policy so they do not push reusable A/B lines out of L2.
template <>
struct OutIO<float> {
  static __device__ __forceinline__ float load(const float* p) { return __ldcs(p); }
  static __device__ __forceinline__ void store(float* p, float v) { __stcs(p, v); }
  // 32 consecutive values, 16-byte aligned.
  static __device__ __forceinline__ void load32(const float* p, float (&c)[32]) {
    const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 t = __ldcs(q + i);
      c[4 * i] = t.x; c[4 * i + 1] = t.y; c[4 * i + 2] = t.z; c[4 * i + 3] = t.w;
    }
  }
  static __device__ __forceinline__ void store32(float* p, const float (&v)[32]) {
    float4* q = reinterpret_cast<float4*>(p);
#pragma unroll
    for (int i = 0; i < 8; ++i) __stcs(q + i, make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
  }
};

template <>
struct OutIO<__half> {
  static __device__ __forceinline__ float load(const __half* p) {
    const unsigned short u = __ldcs(reinterpret_cast<const unsigned short*>(p));
    return __half2float(__ushort_as_half(u));
  }
  static __device__ __forceinline__ void store(__half* p, float v) {
    __stcs(reinterpret_cast<unsigned short*>(p), __half_as_ushort(__float2half_rn(v)));
  }
  static __device__ __forceinline__ void load32(const __half* p, float (&c)[32]) {
    const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 t = __ldcs(q + i);
      const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __half2 h = *reinterpret_cast<const __half2*>(&w[j]);
        const float2 f = __half22float2(h);
        c[8 * i + 2 * j] = f.x;
        c[8 * i + 2 * j + 1] = f.y;
      }
    }
  }
  static __device__ __forceinline__ void store32(__half* p, const float (&v)[32]) {
    uint4* q = reinterpret_cast<uint4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __half2 h = __floats2half2_rn(v[8 * i + 2 * j], v[8 * i + 2 * j + 1]);
        w[j] = *reinterpret_cast<const uint32_t*>(&h);
      }
      __stcs(q + i, make_uint4(w[0], w[1], w[2], w[3]));
    }
  }
};

template <int BN, int G, typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
    tb_gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmC, const KParams p) {
  using Cf = Cfg<BN, G>;
  constexpr int S = Cf::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + (size_t)S * Cf::kABytes;
  uint8_t* sEpi = sB + (size_t)S * Cf::kBBytes;  // 1024-aligned: stage sizes are multiples of 1 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sEpi + Cf::kEpiBytes);
  uint64_t* full = bars;            // leader: A/B of both CTAs landed
  uint64_t* empty = bars + S;       // every CTA: stage consumed by the MMAs
  uint64_t* tfull = bars + 2 * S;   // every CTA: accumulator ready
  uint64_t* tempty = bars + 2 * S + 2;  // leader: accumulator drained by all epilogues
  uint64_t* drain = bars + 2 * S + 4;
  uint64_t* cinbar = bars + 2 * S + 5;  // per epilogue warp: C_in chunks loaded by TMA
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * S + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = __shfl_sync(0xffffffffu, threadIdx.x / 32, 0);
  const int lane = threadIdx.x % 32;
  const uint32_t rank = (G == 2) ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int32_t first_pid = blockIdx.x / G;
  const int32_t pid_stride = gridDim.x / G;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_addr(&tfull[a]), 1);
      mbar_init(smem_addr(&tempty[a]), 4 * G);
    }
    mbar_init(smem_addr(drain), 1);
    for (int w = 0; w < 4; ++w) mbar_init(smem_addr(&cinbar[w]), 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (p.tma_out != kTmaNone) tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc_g<G>(smem_addr(tmem_holder), Cf::kTmemCols);
    tmem_relinquish_g<G>();
  }
  tc_fence_before();
  if constexpr (G == 2) cluster_sync(); else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // A dependent grid (the split-K reduction) may be scheduled now; it waits
  // for this grid's completion before reading anything.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // The whole warp runs the loop (warp-uniform values live in uniform
    // registers); one elected lane issues the TMA copies.
    int stage = 0;
    uint32_t phase = 0;
    long long issued = 0;
    for (int32_t pid = first_pid; pid < p.positions; pid += pid_stride) {
      const Extent e = program_extent<kCtaM * G, BN>(p, pid, Cf::kKB);
      bool ok = true;
      for (int kb = 0; kb < e.nkb; ++kb) {
        if (!warp_wait(smem_addr(&empty[stage]), phase ^ 1u, abort_flag, kSiteProducer, lane)) {
          ok = false;
          break;
        }
        const uint32_t fb_local = smem_addr(&full[stage]);
        const int kc = k_chunk(pid, first_pid, pid_stride, kb, e.nkb);
        const int32_t kx = e.k_begin + kc * Cf::kKB;
        const uint32_t dA = smem_addr(sA + (size_t)stage * Cf::kABytes);
        const uint32_t dB = smem_addr(sB + (size_t)stage * Cf::kBBytes);
        if (elect_one()) {
          if (leader) mbar_expect_tx(fb_local, G * Cf::kStageBytes);
          if constexpr (G == 2) {
            const uint32_t fb = map_to_cta(fb_local, 0);
            const int32_t am = e.m0 + (int32_t)rank * 128;
            const int32_t bn = e.n0 + (int32_t)rank * Cf::kBnCta;
            if (p.a_mn) {  // two [KB k × 64 m] boxes
              tma_load_2d_pair(dA, &tmA, fb, am, kx);
              tma_load_2d_pair(dA + Cf::kBoxBytes, &tmA, fb, am + 64, kx);
            } else {       // KB/64 [128 m × 64 k] sub-tiles
#pragma unroll
              for (int j = 0; j < Cf::kKB / 64; ++j)
                tma_load_2d_pair(dA + j * Cf::kASub, &tmA, fb, kx + 64 * j, am);
            }
            if constexpr (Cf::kMmaPerK == 2) {
              // Per MMA h, this CTA holds columns [256·h + 128·rank, +128):
              // TMEM column c of the pair's accumulator is tile column c.
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int32_t nh = e.n0 + 256 * h + (int32_t)rank * 128;
                if (p.b_kmaj) {  // one [128 n × 64 k] box
                  tma_load_2d_pair(dB + h * Cf::kBHalf, &tmB, fb, kx, nh);
                } else {         // two [64 k × 64 n] boxes
                  tma_load_2d_pair(dB + h * Cf::kBHalf, &tmB, fb, nh, kx);
                  tma_load_2d_pair(dB + h * Cf::kBHalf + Cf::kBoxBytes, &tmB, fb, nh + 64, kx);
                }
              }
            } else if (p.b_kmaj) {  // KB/64 [kBnCta n × 64 k] sub-tiles
#pragma unroll
              for (int j = 0; j < Cf::kKB / 64; ++j)
                tma_load_2d_pair(dB + j * Cf::kBSub, &tmB, fb, kx + 64 * j, bn);
            } else {         // kBnCta/64 [KB k × 64 n] boxes
#pragma unroll
              for (int j = 0; j < Cf::kBnCta / 64; ++j)
                tma_load_2d_pair(dB + j * Cf::kBoxBytes, &tmB, fb, bn + 64 * j, kx);
            }
          } else {
            if (p.a_mn) {
              tma_load_2d(dA, &tmA, fb_local, e.m0, kx);
              tma_load_2d(dA + Cf::kBoxBytes, &tmA, fb_local, e.m0 + 64, kx);
            } else {
#pragma unroll
              for (int j = 0; j < Cf::kKB / 64; ++j)
                tma_load_2d(dA + j * Cf::kASub, &tmA, fb_local, kx + 64 * j, e.m0);
            }
            if (p.b_kmaj) {
#pragma unroll
              for (int j = 0; j < Cf::kKB / 64; ++j)
                tma_load_2d(dB + j * Cf::kBSub, &tmB, fb_local, kx + 64 * j, e.n0);
            } else {
#pragma unroll
              for (int j = 0; j < Cf::kBnCta / 64; ++j)
                tma_load_2d(dB + j * Cf::kBoxBytes, &tmB, fb_local, e.n0 + 64 * j, kx);
            }
          }
        }
        __syncwarp();
        ++issued;
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
    }
    if (lane == 0) {
      // Drain: the newest fill of each stage must land before the CTA exits
      // (only the leader's full barriers count the bytes).
      if (leader) {
        const long long last = issued < S ? issued : S;
        for (long long i = 0; i < last; ++i) {
          const long long f = issued - 1 - i;
          const int s = (int)(f % S);
          const uint32_t par = (uint32_t)((f / S) & 1);
          const long long t0 = clock64();
          while (!mbar_try_wait(smem_addr(&full[s]), par)) {
            if (clock64() - t0 > kWaitBudgetCycles) {
              record_error(TB_ERR_DEVICE_TIMEOUT, kSiteDrain);
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    // Leader CTA only. Whole warp runs the loop; descriptors are computed
    // warp-uniformly and one elected lane issues tcgen05.mma / commit.
    if (leader) {
      const uint32_t idesc = idesc_f16_f32(kCtaM * G, Cf::kMmaN, p.a_mn ? 1 : 0, p.b_kmaj ? 0 : 1);
      // Per-operand layout in shared memory (all 128-byte swizzled):
      //   K-major: sub-tiles of rows of 64 k (128 B), 8-row groups 1024 B
      //            apart (SBO); a K step of 16 elements is 32 B inside the
      //            swizzle atom, every 4th step moves to the next sub-tile.
      //   MN-major: [KB k × 64 mn] boxes kBoxBytes apart (LBO), 8 k-rows
      //            1024 B apart (SBO); a K step of 16 rows is 2048 B.
      const uint32_t a_lbo = p.a_mn ? Cf::kBoxBytes : 16u;
      const uint32_t b_lbo = p.b_kmaj ? 16u : Cf::kBoxBytes;
      auto a_off = [&](int kk) -> uint32_t {
        return p.a_mn ? (uint32_t)kk * 2048u : (uint32_t)(kk >> 2) * Cf::kASub + (uint32_t)(kk & 3) * 32u;
      };
      auto b_off = [&](int kk) -> uint32_t {
        return p.b_kmaj ? (uint32_t)(kk >> 2) * Cf::kBSub + (uint32_t)(kk & 3) * 32u : (uint32_t)kk * 2048u;
      };
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool issued_any = false;
      bool ok = true;
      for (int32_t pid = first_pid; pid < p.positions && ok; pid += pid_stride) {
        const Extent e = program_extent<kCtaM * G, BN>(p, pid, Cf::kKB);
        if (!warp_wait(smem_addr(&tempty[acc]), acc_phase ^ 1u, abort_flag, kSiteMma, lane)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        if (e.nkb == 0) {
          if (elect_one()) {
            mbar_arrive(smem_addr(&tfull[acc]));
            if constexpr (G == 2) mbar_arrive_cluster(map_to_cta(smem_addr(&tfull[acc]), 1));
          }
          __syncwarp();
        } else {
          for (int kb = 0; kb < e.nkb; ++kb) {
            if (!warp_wait(smem_addr(&full[stage]), phase, abort_flag, kSiteMma, lane)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const int kc = k_chunk(pid, first_pid, pid_stride, kb, e.nkb);
            const int kvalid = min(Cf::kKB, e.k_end - (e.k_begin + kc * Cf::kKB));
            const uint32_t a0 = smem_addr(sA + (size_t)stage * Cf::kABytes);
            const uint32_t b0 = smem_addr(sB + (size_t)stage * Cf::kBBytes);
            const uint64_t da0 = smem_desc_sw128(a0, a_lbo, 1024);
            const uint64_t db0 = smem_desc_sw128(b0, b_lbo, 1024);
            if (elect_one()) {
              if (kvalid == Cf::kKB) {
#pragma unroll
                for (int kk = 0; kk < Cf::kKB / 16; ++kk) {
                  // start-address field is bits [0,14) in 16-byte units
                  const uint64_t da = da0 + (uint64_t)(a_off(kk) >> 4);
                  const uint64_t db = db0 + (uint64_t)(b_off(kk) >> 4);
#pragma unroll
                  for (int h = 0; h < Cf::kMmaPerK; ++h) {
                    const uint32_t dd = d_tmem + (uint32_t)(h * Cf::kMmaN);
                    const uint64_t dbh = db + (uint64_t)((h * Cf::kBHalf) >> 4);
                    if constexpr (G == 2)
                      umma_f16_pair(dd, da, dbh, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                    else
                      umma_f16(dd, da, dbh, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                  }
                }
              } else {
                const int nk16 = (kvalid + 15) / 16;
                for (int kk = 0; kk < nk16; ++kk) {
                  const uint64_t da = da0 + (uint64_t)(a_off(kk) >> 4);
                  const uint64_t db = db0 + (uint64_t)(b_off(kk) >> 4);
                  for (int h = 0; h < Cf::kMmaPerK; ++h) {
                    const uint32_t dd = d_tmem + (uint32_t)(h * Cf::kMmaN);
                    const uint64_t dbh = db + (uint64_t)((h * Cf::kBHalf) >> 4);
                    if constexpr (G == 2)
                      umma_f16_pair(dd, da, dbh, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                    else
                      umma_f16(dd, da, dbh, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                  }
                }
              }
              if constexpr (G == 2) umma_commit_pair(smem_addr(&empty[stage]), 0x3);
              else umma_commit(smem_addr(&empty[stage]));
            }
            __syncwarp();
            issued_any = true;
            if (++stage == S) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          if (elect_one()) {
            if constexpr (G == 2) umma_commit_pair(smem_addr(&tfull[acc]), 0x3);
            else umma_commit(smem_addr(&tfull[acc]));
          }
          __syncwarp();
        }
        if (++acc == Cf::kAccs) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && issued_any && lane == 0) {
        // Aborted with MMAs possibly in flight: wait for them before TMEM goes.
        if constexpr (G == 2) umma_commit_pair(smem_addr(drain), 0x1);
        else umma_commit(smem_addr(drain));
        const long long t0 = clock64();
        while (!mbar_try_wait(smem_addr(drain), 0)) {
          if (clock64() - t0 > kWaitBudgetCycles) {
            record_error(TB_ERR_DEVICE_TIMEOUT, kSiteDrain);
            break;
          }
        }
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = (int)rank * 128 + q * 32 + lane;
    uint8_t* epi_buf = sEpi + (size_t)(warp - 2) * 2 * Cf::kEpiBufBytes;
    uint32_t epi_slot = 0;
    // 128-byte staging rows: 32 f32 or 64 f16 columns per chunk
    constexpr int kChunkCols = 128 / (int)sizeof(OutT);
    constexpr uint32_t kRingWarp = (uint32_t)S * Cf::kStageBytes / 4;  // ring bytes per epilogue warp
    constexpr int kRingSlots = (int)(kRingWarp / Cf::kEpiBufBytes);
    uint32_t cin_phase = 0;
    if (p.one_item && p.beta && p.epilogue == kEpiStore && first_pid < p.positions) {
      // One item per CTA: its C_in rows are prefetched into L2 while the
      // mainloop runs, so the epilogue's C_in loads hit L2.
      const Extent e0 = program_extent<kCtaM * G, BN>(p, first_pid, Cf::kKB);
      const uint32_t bytes = (uint32_t)(e0.cols * (int)sizeof(OutT)) & ~15u;
      if (row_in_tile < e0.rows && bytes > 0 && p.vec_c) {
        const char* src = reinterpret_cast<const char*>(reinterpret_cast<const OutT*>(p.C) +
                                                        ((int64_t)e0.m0 + row_in_tile) * p.ldc + e0.n0);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
      }
    }
    const uint32_t tempty_leader0 = G == 2 ? map_to_cta(smem_addr(&tempty[0]), 0) : smem_addr(&tempty[0]);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int32_t pid = first_pid; pid < p.positions; pid += pid_stride) {
      const Extent e = program_extent<kCtaM * G, BN>(p, pid, Cf::kKB);
      int ok = 0;
      if (lane == 0) ok = wait_bounded(smem_addr(&tfull[acc]), acc_phase, abort_flag, kSiteEpilogue);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const bool row_ok = row_in_tile < e.rows;
      const int64_t grow = (int64_t)e.m0 + row_in_tile;
      // A K piece of a tail item adds its partial sum into C (which holds
      // C_in and the other pieces' sums) instead of storing C_in + sum.
      const int32_t tma_out = e.piece ? (int32_t)kTmaReduceC : p.tma_out;
      // When each CTA has a single work item, the mainloop's ring is idle
      // once tfull arrives (every MMA that read it has completed, and no
      // load follows). Each thread then copies its whole C_in row into it
      // with cp.async — all 16-byte pieces in flight at once — instead of one
      // DRAM round trip per 32-column chunk (a clock64 timeline of a
      // single-wave 2048³ launch showed ~1.3k of each chunk's ~1.7k cycles
      // waiting on that load). Rows are padded by 16 bytes: the warp's
      // per-row reads then spread over all banks.
      constexpr uint32_t kCinStride = (uint32_t)(BN * sizeof(OutT)) + 16u;
      constexpr bool kCinFits = 128u * kCinStride <= (uint32_t)S * Cf::kStageBytes;
      const bool cin_from_smem = kCinFits && p.cin_smem && p.beta && p.epilogue == kEpiStore && row_ok &&
                                 !(tma_out != kTmaNone && p.one_item &&
                                   (e.cols + kChunkCols - 1) / kChunkCols <= kRingSlots);
      const uint8_t* cin_row = smem + (size_t)((warp - 2) * 32 + lane) * kCinStride;
      if (cin_from_smem) {
        fence_proxy_async_smem();
        const char* src = reinterpret_cast<const char*>(reinterpret_cast<const OutT*>(p.C) +
                                                        grow * p.ldc + e.n0);
        const int bytes = e.cols * (int)sizeof(OutT);
        for (int off = 0; off < bytes; off += 16)
          cp_async_16(smem_addr(cin_row + off), src + off, (uint32_t)min(16, bytes - off));
        cp_async_wait_all();
      }
      // C_in of columns [c0, c0 + 32) of this row (zero past ncol).
      auto load_cin = [&](int c0, int ncol, float (&c)[32]) {
        if (cin_from_smem) {
          if constexpr (sizeof(OutT) == 4) {
            const float4* q4 = reinterpret_cast<const float4*>(cin_row + c0 * 4);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 t = q4[j];
              c[4 * j] = t.x; c[4 * j + 1] = t.y; c[4 * j + 2] = t.z; c[4 * j + 3] = t.w;
            }
          } else {
            const __half2* h2 = reinterpret_cast<const __half2*>(cin_row + c0 * 2);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float2 f = __half22float2(h2[j]);
              c[2 * j] = f.x; c[2 * j + 1] = f.y;
            }
          }
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i >= ncol) c[i] = 0.f;
          return;
        }
        const OutT* src = reinterpret_cast<const OutT*>(p.C) + grow * p.ldc + e.n0 + c0;
        if (ncol == 32 && (p.vec_c || tma_out == kTmaStoreC)) {
          OutIO<OutT>::load32(src, c);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) c[i] = i < ncol ? OutIO<OutT>::load(src + i) : 0.f;
        }
      };
      if (tma_out != kTmaNone) {
        // TMA path (program tile == hardware tile, or a whole sub-tile of
        // one). The warp's 32 rows go out in chunks of 32 × 128 bytes (32 f32
        // or 64 f16 columns) staged in 128-byte-swizzled shared memory (row
        // r's 16-byte piece j at piece j ^ (r % 8): the warp's 16-byte writes
        // are bank-conflict free), written, reduce-added or stored by TMA;
        // rows/columns past M/N are clipped by TMA, so rows past M carry zeros.
        // Two staging buffers per warp rotate; with one work item per CTA
        // (wide) the idle ring holds all of the warp's chunks at once, C_in
        // comes in by TMA into the same buffers, and no chunk waits for the
        // previous one's store.
        // chunk element: OutT for C stores; f32 for reduce-adds and the
        // split_k_serial workspace
        bool wide = false;
        auto chunks = [&](auto f16_tag) -> bool {
          constexpr bool kF16 = decltype(f16_tag)::value;
          constexpr int kCw = kF16 ? 64 : 32;
          const int nch = (e.cols + kCw - 1) / kCw;
          wide = p.one_item && nch <= kRingSlots;
          uint8_t* slots = wide ? smem + (size_t)(warp - 2) * kRingWarp : epi_buf;
          const bool cin_tma = wide && tma_out == kTmaStoreC && p.beta;
          const int32_t y0 = (int32_t)(grow - lane);
          if (cin_tma) {
            const uint32_t cb = smem_addr(&cinbar[q]);
            if (lane == 0) {
              fence_proxy_async_smem();
              mbar_expect_tx(cb, (uint32_t)nch * Cf::kEpiBufBytes);
              for (int j = 0; j < nch; ++j)
                tma_load_2d(smem_addr(slots + (size_t)j * Cf::kEpiBufBytes), &tmC, cb,
                            (int32_t)(e.n0 + j * kCw), y0);
            }
            int okc = 0;
            if (lane == 0) okc = wait_bounded(cb, cin_phase, abort_flag, kSiteEpilogue);
            okc = __shfl_sync(0xffffffffu, okc, 0);
            cin_phase ^= 1u;
            if (!okc) return false;
          }
          // C_in through the rotating buffers: the boxes of the later chunks
          // are prefetched into L2 now, and each 32-column half's loads are
          // issued one half ahead of its use (a DRAM round trip per chunk
          // otherwise serialises the epilogue).
          const bool pipe_cin = !cin_tma && tma_out == kTmaStoreC && p.beta && row_ok && !cin_from_smem;
          if (!cin_tma && tma_out == kTmaStoreC && p.beta && !cin_from_smem && lane == 0)
            for (int j = 1; j < nch; ++j) tma_prefetch_l2_2d(&tmC, (int32_t)(e.n0 + j * kCw), y0);
          auto fetch_cin = [&](int cc, float (&c)[32]) {
            const int nc = max(0, min(32, e.cols - cc));
            if (nc > 0) {
              load_cin(cc, nc, c);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) c[i] = 0.f;
            }
          };
          float cn[32];
          if (pipe_cin) fetch_cin(0, cn);
          for (int j = 0; j < nch; ++j) {
            const int c0 = j * kCw;
            const int64_t gcol = (int64_t)e.n0 + c0;
            uint8_t* buf = wide ? slots + (size_t)j * Cf::kEpiBufBytes
                                : epi_buf + (size_t)(epi_slot & 1) * Cf::kEpiBufBytes;
            if (!wide) {
              // The bulk op issued two chunks ago must have finished reading buf.
              if (lane == 0) bulk_wait_group_read<1>();
              __syncwarp();
            }
            uint8_t* row = buf + lane * 128;
#pragma unroll
            for (int h = 0; h < kCw / 32; ++h) {  // 32-column halves (f16: two per chunk)
              const int cc = c0 + 32 * h;
              float v[32];
              if (e.nkb > 0) {
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + cc), v);
              } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = 0.f;
              }
              if (!row_ok) {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = 0.f;
              }
              const int ncol = max(0, min(32, e.cols - cc));
              if (tma_out == kTmaStoreC && p.beta && row_ok) {
                float c[32];
                if (cin_tma) {
                  if constexpr (!kF16) {
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                      const float4 t = *reinterpret_cast<const float4*>(row + ((u ^ (lane & 7)) * 16));
                      c[4 * u] = t.x; c[4 * u + 1] = t.y; c[4 * u + 2] = t.z; c[4 * u + 3] = t.w;
                    }
                  } else {
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                      const uint4 t = *reinterpret_cast<const uint4*>(row + (((4 * h + u) ^ (lane & 7)) * 16));
                      const uint32_t w4[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
                      for (int w = 0; w < 4; ++w) {
                        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[w]));
                        c[8 * u + 2 * w] = f.x; c[8 * u + 2 * w + 1] = f.y;
                      }
                    }
                  }
                } else if (pipe_cin) {
#pragma unroll
                  for (int i = 0; i < 32; ++i) c[i] = cn[i];
                  if (cc + 32 < nch * kCw) fetch_cin(cc + 32, cn);
                } else if (ncol > 0) {
                  load_cin(cc, ncol, c);
                } else {
#pragma unroll
                  for (int i = 0; i < 32; ++i) c[i] = 0.f;
                }
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] += c[i];
              }
              if (tma_out == kTmaStoreC && p.ex.any) {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                  if (i < ncol) v[i] = apply_exprs(p.ex, v[i], (int64_t)e.n0 + cc + i);
              }
              if constexpr (!kF16) {
#pragma unroll
                for (int u = 0; u < 8; ++u)
                  *reinterpret_cast<float4*>(row + ((u ^ (lane & 7)) * 16)) =
                      make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
              } else {
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  uint32_t w4[4];
#pragma unroll
                  for (int w = 0; w < 4; ++w) {
                    const __half2 hv = __floats2half2_rn(v[8 * u + 2 * w], v[8 * u + 2 * w + 1]);
                    w4[w] = *reinterpret_cast<const uint32_t*>(&hv);
                  }
                  *reinterpret_cast<uint4*>(row + (((4 * h + u) ^ (lane & 7)) * 16)) =
                      make_uint4(w4[0], w4[1], w4[2], w4[3]);
                }
              }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              if (tma_out == kTmaStoreC) tma_store_2d(&tmC, smem_addr(buf), (int32_t)gcol, y0);
              else if (tma_out == kTmaReduceC) tma_reduce_add_2d(&tmC, smem_addr(buf), (int32_t)gcol, y0);
              else tma_store_3d(&tmC, smem_addr(buf), (int32_t)gcol, y0, e.part);
              bulk_commit_group();
            }
            ++epi_slot;
          }
          return true;
        };
        const bool chunks_ok = (sizeof(OutT) == 2 && tma_out == kTmaStoreC)
                                   ? chunks(std::integral_constant<bool, true>())
                                   : chunks(std::integral_constant<bool, false>());
        if (!chunks_ok) break;
        if (wide) {
          // the ring is refilled only by a next item, which a wide CTA has
          // not; still, the stores must read their buffers before the CTA ends
          if (lane == 0) bulk_wait_group_read<0>();
          __syncwarp();
        }
      } else
      for (int c0 = 0; c0 < e.cols; c0 += 32) {
        float v[32];
        if (e.nkb > 0) {
          tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + c0), v);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.f;
        }
        const int ncol = min(32, e.cols - c0);
        const int64_t gcol = (int64_t)e.n0 + c0;
        if (!row_ok) continue;
        if (p.epilogue == kEpiStore) {
          OutT* dst = reinterpret_cast<OutT*>(p.C) + grow * p.ldc + gcol;
          if (ncol == 32 && p.vec_c) {
            if (p.beta) {
              float c[32];
              load_cin(c0, ncol, c);
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] += c[i];
            }
            if (p.ex.any) {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = apply_exprs(p.ex, v[i], gcol + i);
            }
            OutIO<OutT>::store32(dst, v);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              if (i < ncol) {
                float r = v[i];
                if (p.beta) r += OutIO<OutT>::load(dst + i);
                if (p.ex.any) r = apply_exprs(p.ex, r, gcol + i);
                OutIO<OutT>::store(dst + i, r);
              }
            }
          }
        } else if (p.epilogue == kEpiWorkspace) {
          float* dst = p.ws + ((int64_t)e.part * p.M + grow) * p.N + gcol;
          if (ncol == 32 && p.vec_ws) {
            OutIO<float>::store32(dst, v);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < ncol) dst[i] = v[i];
          }
        } else {  // kEpiAtomic: f32 C only
          float* dst = reinterpret_cast<float*>(p.C) + grow * p.ldc + gcol;
          if (ncol == 32 && p.vec_c) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              atomicAdd(reinterpret_cast<float4*>(dst) + i,
                        make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < ncol) atomicAdd(dst + i, v[i]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (G == 2) mbar_arrive_cluster(tempty_leader0 + acc * 8);
        else mbar_arrive(smem_addr(&tempty[acc]));
      }
      if (++acc == Cf::kAccs) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // Outstanding TMA stores must finish before the CTA (and its shared
    // memory) goes away.
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  __syncthreads();
  if constexpr (G == 2) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_g<G>(tmem_base, Cf::kTmemCols);
  }
}

// ---------------------------------------------------------------- small
// Latency kernel for problems whose every work item has at most kSmallK K
// elements on a one-CTA 128 × BN tile (the BASELINE's 64×64×32, 96×80×32,
// 192×128×32 and split 64×64×64 programs). No warp roles and no pipeline:
// one thread brings the item's A and B boxes (and the C_in tile, when C is
// TMA-addressable) in with TMA on one mbarrier while warp 0 allocates TMEM,
// then issues the K/16 tcgen05.mma steps, and every thread takes its
// accumulator row from TMEM and stores it. A CTA walks several items in turn
// when there are more items than CTAs (persistent plans).
constexpr int kSmallK = 128;
// Work of the first kSmallTab walk positions, derived on the host (the same
// program_extent): a single thread's chain of mapping arithmetic and
// parameter reads took ~0.6 µs of a ~4 µs kernel.
constexpr int kSmallTab = 64;
struct SmallTab {
  int32_t n;  // positions described (0: derive on the device)
  int32_t m0[kSmallTab], n0[kSmallTab], k_begin[kSmallTab];
  int16_t rows[kSmallTab], cols[kSmallTab], kvalid[kSmallTab], part[kSmallTab];
};
constexpr uint32_t kSmallASub = 128 * 64 * 2;         // one [128 m × 64 k] K-major sub-tile
constexpr uint32_t kSmallABytes = kSmallK / 64 * kSmallASub;
constexpr uint32_t kSmallBox = kSmallK * 64 * 2;      // one [kSmallK k × 64 n] MN-major box

template <int BN, typename OutT>
struct SmallCfg {
  static constexpr uint32_t kBBytes = BN / 64 * kSmallBox;
  static constexpr uint32_t kCinStride = BN * sizeof(OutT) + 16;  // padded row: conflict-free reads
  static constexpr size_t kSmem = 1024 + kSmallABytes + kBBytes + 128 * kCinStride + 64 + 16;
};

template <int BN, typename OutT>
__global__ void __launch_bounds__(128, 1)
    tb_gemm_small_kernel(const __grid_constant__ KParams pk, const __grid_constant__ SmallTab tab,
                         const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmC) {
  using Sc = SmallCfg<BN, OutT>;
  // The parameters come through the constant bank, which each launch
  // refills: reading them field by field inside the dependent mapping
  // arithmetic costs a miss per cache line in series (~0.6 µs measured).
  // One word per thread brings every line in at once; the kernel then reads
  // its shared-memory copy.
  static_assert(sizeof(KParams) % 4 == 0 && sizeof(KParams) <= 4 * 128, "KParams copy");
  __shared__ __align__(16) KParams p_s;
  if (threadIdx.x < sizeof(KParams) / 4)
    reinterpret_cast<uint32_t*>(&p_s)[threadIdx.x] = reinterpret_cast<const uint32_t*>(&pk)[threadIdx.x];
  __syncthreads();
  const KParams& p = p_s;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kSmallABytes;
  uint8_t* sCin = sB + Sc::kBBytes;
  uint64_t* done = reinterpret_cast<uint64_t*>(sCin + 128 * Sc::kCinStride);
  uint64_t* ld_bar = done + 1;  // the item's TMA loads (A, B and, when C is TMA-addressable, C_in)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(done + 2);
  // C_in by TMA: [32 rows × 128 bytes] boxes, 128-byte swizzled, box (w, j)
  // (row group w, 128-byte column chunk j) at sCin + (w · kCinChunks + j) · 4 KB
  constexpr int kCinChunks = BN * (int)sizeof(OutT) / 128;
  constexpr int kCinCols = 128 / (int)sizeof(OutT);  // columns per chunk
  const int t = threadIdx.x;
  const int warp = t / 32;
  if (t == 0) {
    mbar_init(smem_addr(done), 1);
    mbar_init(smem_addr(ld_bar), 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  __syncthreads();
  uint32_t ld_phase = 0;
  const bool cin_tma = p.tma_out == kTmaStoreC && p.beta && p.epilogue == kEpiStore;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const uint32_t idesc = idesc_f16_f32(128, BN, 0, 1);
  uint32_t phase = 0;
  uint32_t tmem_base = 0;
  bool have_tmem = false;
  for (int32_t pos = blockIdx.x; pos < p.positions; pos += gridDim.x) {
    Extent e;
    int kvalid;
    if (pos < tab.n) {
      e.m0 = tab.m0[pos];
      e.n0 = tab.n0[pos];
      e.k_begin = tab.k_begin[pos];
      e.rows = tab.rows[pos];
      e.cols = tab.cols[pos];
      e.part = tab.part[pos];
      kvalid = tab.kvalid[pos];
    } else {
      e = program_extent<128, BN>(p, pos, kSmallK);
      kvalid = e.nkb > 0 ? e.k_end - e.k_begin : 0;  // <= kSmallK (plan rule)
    }
    const int k16 = (kvalid + 15) / 16 * 16;                 // K covered by the MMA steps
    // ---- one thread brings the item in with TMA on one mbarrier: A as
    //      [128 m × 64 k] K-major boxes, B as [128 k × 64 n] MN-major boxes
    //      (both 128-byte swizzled, the layouts the UMMA descriptors read;
    //      zero past M/N/K), and, when C is TMA-addressable, the C_in tile as
    //      [32 rows × 128 bytes] boxes. Only the K steps below the item's
    //      range are issued: its end is a multiple of 16 (block_k) or the end
    //      of K, where the boxes read zeros.
    if (t == 0) {
      const int na = (k16 + 63) / 64;
      const int nrg = cin_tma ? min(4, (e.rows + 31) / 32) : 0;
      const int nch = cin_tma ? (e.cols + kCinCols - 1) / kCinCols : 0;
      const uint32_t bytes =
          k16 > 0 ? (uint32_t)(na * kSmallASub + (BN / 64) * kSmallBox + nrg * nch * 4096) : (uint32_t)(nrg * nch * 4096);
      mbar_expect_tx(smem_addr(ld_bar), bytes);
      if (k16 > 0) {
        for (int j = 0; j < na; ++j)
          tma_load_2d(smem_addr(sA + (size_t)j * kSmallASub), &tmA, smem_addr(ld_bar), e.k_begin + 64 * j, e.m0);
        for (int j = 0; j < BN / 64; ++j)
          tma_load_2d(smem_addr(sB + (size_t)j * kSmallBox), &tmB, smem_addr(ld_bar), e.n0 + 64 * j, e.k_begin);
      }
      for (int w = 0; w < nrg; ++w)
        for (int j = 0; j < nch; ++j)
          tma_load_2d(smem_addr(sCin + (size_t)(w * kCinChunks + j) * 4096), &tmC, smem_addr(ld_bar),
                      e.n0 + j * kCinCols, e.m0 + 32 * w);
    }
    // ---- this thread's C_in row, fetched alongside the operands
    const bool row_ok = t < e.rows;
    const int64_t grow = (int64_t)e.m0 + t;
    const bool cin_smem = p.cin_smem && p.beta && p.epilogue == kEpiStore && row_ok;
    uint8_t* cin_row = sCin + (size_t)t * Sc::kCinStride;
    if (cin_smem) {
      const char* src = reinterpret_cast<const char*>(reinterpret_cast<const OutT*>(p.C) + grow * p.ldc + e.n0);
      const int bytes = e.cols * (int)sizeof(OutT);
      for (int off = 0; off < bytes; off += 16)
        cp_async_16(smem_addr(cin_row + off), src + off, (uint32_t)min(16, bytes - off));
    }
    if (!have_tmem && warp == 0) {
      // first item: the TMEM allocation (~0.35 µs) overlaps the copies in flight
      tmem_alloc(smem_addr(tmem_holder), BN);
      tmem_relinquish();
    }
    cp_async_wait_all();  // the per-row C_in copies, when C is not TMA-addressable
    {
      const long long t0 = clock64();
      while (!mbar_try_wait(smem_addr(ld_bar), ld_phase)) {
        if (clock64() - t0 > kWaitBudgetCycles) {
          record_error(TB_ERR_DEVICE_TIMEOUT, kSiteEpilogue);
          break;
        }
      }
      ld_phase ^= 1u;
    }
    fence_proxy_async_smem();  // cp.async wrote through the generic proxy; the MMA reads via async
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (!have_tmem) {
      tmem_base = *tmem_holder;
      have_tmem = true;
    }
    if (t == 0 && k16 > 0) {
      tc_fence_after();
      const uint64_t da0 = smem_desc_sw128(smem_addr(sA), 16, 1024);
      const uint64_t db0 = smem_desc_sw128(smem_addr(sB), kSmallBox, 1024);
      for (int kk = 0; kk < k16 / 16; ++kk) {
        const uint64_t da = da0 + (uint64_t)((((kk >> 2) * kSmallASub) + (kk & 3) * 32) >> 4);
        const uint64_t db = db0 + (uint64_t)((kk * 2048) >> 4);
        umma_f16(tmem_base, da, db, idesc, kk > 0 ? 1u : 0u);
      }
      umma_commit(smem_addr(done));
    }
    if (k16 > 0) {
      // every thread waits (bounded) for the MMAs
      const long long t0 = clock64();
      while (!mbar_try_wait(smem_addr(done), phase)) {
        if (clock64() - t0 > kWaitBudgetCycles) {
          record_error(TB_ERR_DEVICE_TIMEOUT, kSiteEpilogue);
          break;
        }
      }
      phase ^= 1u;
      tc_fence_after();
    }
    // ---- epilogue: thread t owns row t of the tile (TMEM lane t)
    for (int c0 = 0; c0 < e.cols; c0 += 32) {
      float v[32];
      if (k16 > 0) {
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.f;
      }
      if (!row_ok) continue;
      const int ncol = min(32, e.cols - c0);
      const int64_t gcol = (int64_t)e.n0 + c0;
      if (p.epilogue == kEpiStore) {
        OutT* dst = reinterpret_cast<OutT*>(p.C) + grow * p.ldc + gcol;
        if (p.beta) {
          if (cin_tma) {
            // row t of box (warp, chunk): 16-byte piece u at piece u ^ (t % 8)
            const int lane = t % 32;
            const int byte0 = c0 * (int)sizeof(OutT);
            const uint8_t* crow = sCin + (size_t)(warp * kCinChunks + byte0 / 128) * 4096 + lane * 128;
            const int u0 = (byte0 % 128) / 16;
            float c[32];
            if constexpr (sizeof(OutT) == 4) {
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                const float4 q4 = *reinterpret_cast<const float4*>(crow + ((u ^ (lane & 7)) * 16));
                c[4 * u] = q4.x; c[4 * u + 1] = q4.y; c[4 * u + 2] = q4.z; c[4 * u + 3] = q4.w;
              }
            } else {
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const uint4 q4 = *reinterpret_cast<const uint4*>(crow + (((u0 + u) ^ (lane & 7)) * 16));
                const uint32_t w4[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[w]));
                  c[8 * u + 2 * w] = f.x; c[8 * u + 2 * w + 1] = f.y;
                }
              }
            }
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < ncol) v[i] += c[i];
          } else if (cin_smem) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              float c = 0.f;
              if constexpr (sizeof(OutT) == 4) c = reinterpret_cast<const float*>(cin_row)[c0 + i];
              else c = __half2float(reinterpret_cast<const __half*>(cin_row)[c0 + i]);
              if (i < ncol) v[i] += c;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < ncol) v[i] += OutIO<OutT>::load(dst + i);
          }
        }
        if (p.ex.any) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < ncol) v[i] = apply_exprs(p.ex, v[i], gcol + i);
        }
        if (ncol == 32 && p.vec_c) {
          OutIO<OutT>::store32(dst, v);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < ncol) OutIO<OutT>::store(dst + i, v[i]);
        }
      } else if (p.epilogue == kEpiWorkspace) {
        float* dst = p.ws + ((int64_t)e.part * p.M + grow) * p.N + gcol;
        if (ncol == 32 && p.vec_ws) {
          OutIO<float>::store32(dst, v);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < ncol) dst[i] = v[i];
        }
      } else {  // kEpiAtomic: f32 C only
        float* dst = reinterpret_cast<float*>(p.C) + grow * p.ldc + gcol;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < ncol) atomicAdd(dst + i, v[i]);
      }
    }
    // the next item overwrites shared memory and TMEM
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  if (have_tmem && warp == 0) tmem_dealloc(tmem_base, BN);
}

// C = beta·C_in + Σ_s ws[s] in a fixed order (split_k_serial): deterministic.
// HBM bound; every thread keeps up to 8 partial loads in flight. Launched
// with programmatic dependent launch: the grid may start while the GEMM
// drains and waits (griddepcontrol.wait) until the GEMM's writes are visible.
template <typename OutT>
__global__ void __launch_bounds__(256)
    tb_splitk_reduce_kernel(const float* __restrict__ ws, int32_t S, int32_t M, int32_t N,
                            void* Cv, int64_t ldc, int32_t beta, int32_t vec, EpiExprs ex) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  OutT* C = reinterpret_cast<OutT*>(Cv);
  const int64_t plane = (int64_t)M * N;
  if (vec) {  // N % 4 == 0 and C rows aligned for 4-element access
    const int64_t nvec = plane / 4;
    const float4* w4 = reinterpret_cast<const float4*>(ws);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nvec;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t e = i * 4;
      const int64_t r = e / N, c = e % N;
      float4 acc = __ldcs(w4 + i);
      for (int s0 = 1; s0 < S; s0 += 8) {
        float4 t[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (s0 + u < S) t[u] = __ldcs(w4 + (int64_t)(s0 + u) * (plane / 4) + i);
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (s0 + u < S) {
            acc.x += t[u].x; acc.y += t[u].y; acc.z += t[u].z; acc.w += t[u].w;
          }
      }
      OutT* dst = C + r * ldc + c;
      if (beta) {
        acc.x += OutIO<OutT>::load(dst);
        acc.y += OutIO<OutT>::load(dst + 1);
        acc.z += OutIO<OutT>::load(dst + 2);
        acc.w += OutIO<OutT>::load(dst + 3);
      }
      if (ex.any) {
        acc.x = apply_exprs(ex, acc.x, c);
        acc.y = apply_exprs(ex, acc.y, c + 1);
        acc.z = apply_exprs(ex, acc.z, c + 2);
        acc.w = apply_exprs(ex, acc.w, c + 3);
      }
      OutIO<OutT>::store(dst, acc.x);
      OutIO<OutT>::store(dst + 1, acc.y);
      OutIO<OutT>::store(dst + 2, acc.z);
      OutIO<OutT>::store(dst + 3, acc.w);
    }
  } else {
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < plane;
         e += (int64_t)gridDim.x * blockDim.x) {
      const int64_t r = e / N, c = e % N;
      float acc = ws[e];
      for (int s = 1; s < S; ++s) acc += ws[s * plane + e];
      OutT* dst = C + r * ldc + c;
      if (beta) acc += OutIO<OutT>::load(dst);
      if (ex.any) acc = apply_exprs(ex, acc, c);
      OutIO<OutT>::store(dst, acc);
    }
  }
}

// dst[r][c] = src[r][c] for c < cols, 0 for cols <= c < ld_dst (f16 rows).
__global__ void __launch_bounds__(256)
    tb_pack_rows_kernel(const uint16_t* __restrict__ src, int64_t ld_src, uint16_t* __restrict__ dst,
                        int64_t ld_dst, int64_t rows, int64_t cols) {
  const int64_t total = rows * ld_dst;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / ld_dst, c = i % ld_dst;
    dst[i] = c < cols ? src[r * ld_src + c] : (uint16_t)0;
  }
}

// ------------------------------------------------------------------ host
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_err = cudaSuccess;

tbStatus get_encoder() {
  std::call_once(g_encode_once, [] {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    g_encode_err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (g_encode_err == cudaSuccess && q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode)
    return tb_fail(TB_ERR_CUDA, std::string("cuTensorMapEncodeTiled unavailable: ") +
                                    cudaGetErrorString(g_encode_err));
  return TB_OK;
}

// Encoding a tensor map costs ~1 µs of host time per operand; repeated calls
// on the same buffers reuse it. The cache is per host thread (no locking) and
// keyed by every encode argument, so a hit always equals a fresh encode.
struct MapKey {
  int dtype, rank, swizzle;
  const void* base;
  cuuint64_t dims[3], strides[2];
  cuuint32_t box[3];
};
struct MapEntry {
  MapKey key;
  CUtensorMap map;
  bool used;
};
constexpr int kMapCacheSize = 8;
thread_local MapEntry t_map_cache[kMapCacheSize];
thread_local int t_map_next = 0;

CUresult encode_cached(CUtensorMap* out, CUtensorMapDataType dtype, int rank, void* base,
                       const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                       CUtensorMapSwizzle swizzle, CUtensorMapL2promotion l2) {
  MapKey k;
  std::memset(&k, 0, sizeof(k));
  k.dtype = (int)dtype;
  k.rank = rank;
  k.swizzle = (int)swizzle | ((int)l2 << 8);
  k.base = base;
  for (int i = 0; i < rank; ++i) {
    k.dims[i] = dims[i];
    k.box[i] = box[i];
  }
  for (int i = 0; i + 1 < rank; ++i) k.strides[i] = strides[i];
  for (int i = 0; i < kMapCacheSize; ++i) {
    if (t_map_cache[i].used && std::memcmp(&t_map_cache[i].key, &k, sizeof(k)) == 0) {
      *out = t_map_cache[i].map;
      return CUDA_SUCCESS;
    }
  }
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(out, dtype, (cuuint32_t)rank, base, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, l2, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_SUCCESS) {
    MapEntry& e = t_map_cache[t_map_next];
    t_map_next = (t_map_next + 1) % kMapCacheSize;
    e.key = k;
    e.map = *out;
    e.used = true;
  }
  return r;
}

// Row-major f16 matrix rows × cols with row stride ld (elements), boxed
// [box_rows × 64] with 128-byte swizzle; out-of-range elements read as 0.
tbStatus encode_f16_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld,
                       uint32_t box_rows, const char* what) {
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, box_rows};
  CUresult r = encode_cached(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                             strides, box, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (r != CUDA_SUCCESS)
    return tb_fail(TB_ERR_CUDA, std::string("cuTensorMapEncodeTiled(") + what +
                                    ") failed with CUresult " + std::to_string((int)r));
  return TB_OK;
}

constexpr int kMaxDevices = 64;
constexpr int kNumTiles = 6;
std::atomic<bool> g_attr_set[kNumTiles][2][kMaxDevices];

template <int BN, int G, typename OutT>
tbStatus launch_gemm(const tb_matmul_plan* plan, const CUtensorMap& ta, const CUtensorMap& tb_,
                     const CUtensorMap& tc, const KParams& kp, cudaStream_t stream, int kt, int ot) {
  auto kern = tb_gemm_sm100_kernel<BN, G, OutT>;
  constexpr size_t smem = Cfg<BN, G>::kSmem;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices || !g_attr_set[kt][ot][dev].load()) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess)
      return tb_fail(TB_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    if (dev >= 0 && dev < kMaxDevices) g_attr_set[kt][ot][dev].store(true);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)plan->grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = G;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb_, tc, kp);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess)
    return tb_fail(TB_ERR_CUDA, std::string("tb_gemm_sm100 launch: ") + cudaGetErrorString(e));
  return TB_OK;
}

template <typename OutT>
tbStatus dispatch_tile(const tb_matmul_plan* plan, const CUtensorMap& ta, const CUtensorMap& tb_,
                       const CUtensorMap& tc, const KParams& kp, cudaStream_t stream, int ot) {
  switch (plan->kernel_tile) {
    case kTile128x64: return launch_gemm<64, 1, OutT>(plan, ta, tb_, tc, kp, stream, 0, ot);
    case kTile128x128: return launch_gemm<128, 1, OutT>(plan, ta, tb_, tc, kp, stream, 1, ot);
    case kTile128x256: return launch_gemm<256, 1, OutT>(plan, ta, tb_, tc, kp, stream, 2, ot);
    case kTile256x128: return launch_gemm<128, 2, OutT>(plan, ta, tb_, tc, kp, stream, 3, ot);
    case kTile256x256: return launch_gemm<256, 2, OutT>(plan, ta, tb_, tc, kp, stream, 4, ot);
    case kTile256x512: return launch_gemm<512, 2, OutT>(plan, ta, tb_, tc, kp, stream, 5, ot);
  }
  return tb_fail(TB_ERR_UNSUPPORTED, "unknown kernel tile");
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

std::atomic<bool> g_small_attr_set[2][2][kMaxDevices];

template <int BN, typename OutT>
tbStatus launch_small_bn(const tb_matmul_plan* plan, const KParams& kp, const CUtensorMap& ta,
                         const CUtensorMap& tb_, const CUtensorMap& tcm, const void* A, int64_t lda,
                         const void* B, int64_t ldb, cudaStream_t stream, int ot) {
  auto kern = tb_gemm_small_kernel<BN, OutT>;
  constexpr size_t smem = SmallCfg<BN, OutT>::kSmem;
  const int bi = BN == 64 ? 0 : 1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices || !g_small_attr_set[bi][ot][dev].load()) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess)
      return tb_fail(TB_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    if (dev >= 0 && dev < kMaxDevices) g_small_attr_set[bi][ot][dev].store(true);
  }
  SmallTab tab;
  std::memset(&tab, 0, sizeof(tab));
  tab.n = kp.positions <= kSmallTab ? kp.positions : 0;
  for (int32_t pos = 0; pos < tab.n; ++pos) {
    const Extent e = program_extent<128, BN>(kp, pos, kSmallK);
    tab.m0[pos] = e.m0;
    tab.n0[pos] = e.n0;
    tab.k_begin[pos] = e.k_begin;
    tab.rows[pos] = (int16_t)std::max(-1, std::min(e.rows, 32767));
    tab.cols[pos] = (int16_t)std::max(-1, std::min(e.cols, 32767));
    tab.kvalid[pos] = (int16_t)(e.nkb > 0 ? e.k_end - e.k_begin : 0);
    tab.part[pos] = (int16_t)e.part;
  }
  (void)A; (void)lda; (void)B; (void)ldb;
  kern<<<(unsigned)plan->grid, 128, smem, stream>>>(kp, tab, ta, tb_, tcm);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return tb_fail(TB_ERR_CUDA, std::string("tb_gemm_small launch: ") + cudaGetErrorString(e));
  return TB_OK;
}

template <typename OutT>
tbStatus launch_small(const tb_matmul_plan* plan, const KParams& kp, const CUtensorMap& ta,
                      const CUtensorMap& tb_, const CUtensorMap& tcm, const void* A, int64_t lda,
                      const void* B, int64_t ldb, cudaStream_t stream, int ot) {
  return plan->cta_n == 64 ? launch_small_bn<64, OutT>(plan, kp, ta, tb_, tcm, A, lda, B, ldb, stream, ot)
                           : launch_small_bn<128, OutT>(plan, kp, ta, tb_, tcm, A, lda, B, ldb, stream, ot);
}

tbStatus pack_rows_f16(const void* src, int64_t ld_src, void* dst, int64_t ld_dst, int64_t rows,
                       int64_t cols, int num_sms, cudaStream_t stream) {
  const int64_t total = rows * ld_dst;
  int64_t blocks = (total + 255) / 256;
  if (blocks > (int64_t)num_sms * 16) blocks = (int64_t)num_sms * 16;
  if (blocks < 1) blocks = 1;
  tb_pack_rows_kernel<<<(unsigned)blocks, 256, 0, stream>>>(static_cast<const uint16_t*>(src), ld_src,
                                                            static_cast<uint16_t*>(dst), ld_dst, rows,
                                                            cols);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TB_OK
                          : tb_fail(TB_ERR_CUDA, std::string("tb_pack_rows launch: ") + cudaGetErrorString(e));
}

}  // namespace

size_t tb_kernel_smem_bytes(int32_t kernel_tile, int32_t /*stages*/) {
  switch (kernel_tile) {
    case kTile128x64: return Cfg<64, 1>::kSmem;
    case kTile128x128: return Cfg<128, 1>::kSmem;
    case kTile128x256: return Cfg<256, 1>::kSmem;
    case kTile256x128: return Cfg<128, 2>::kSmem;
    case kTile256x256: return Cfg<256, 2>::kSmem;
    case kTile256x512: return Cfg<512, 2>::kSmem;
  }
  return 0;
}

size_t tb_small_smem_bytes(int32_t cta_n, int32_t c_dtype) {
  if (cta_n == 64) return c_dtype == TB_F16 ? SmallCfg<64, __half>::kSmem : SmallCfg<64, float>::kSmem;
  return c_dtype == TB_F16 ? SmallCfg<128, __half>::kSmem : SmallCfg<128, float>::kSmem;
}

int32_t tb_kernel_kb(int32_t kernel_tile) {
  switch (kernel_tile) {
    case kTile128x64: return Cfg<64, 1>::kKB;
    case kTile128x128: return Cfg<128, 1>::kKB;
    case kTile128x256: return Cfg<256, 1>::kKB;
    case kTile256x128: return Cfg<128, 2>::kKB;
    case kTile256x256: return Cfg<256, 2>::kKB;
    case kTile256x512: return Cfg<512, 2>::kKB;
  }
  return 0;
}

int32_t tb_kernel_max_stages(int32_t kernel_tile) {
  switch (kernel_tile) {
    case kTile128x64: return Cfg<64, 1>::kStages;
    case kTile128x128: return Cfg<128, 1>::kStages;
    case kTile128x256: return Cfg<256, 1>::kStages;
    case kTile256x128: return Cfg<128, 2>::kStages;
    case kTile256x256: return Cfg<256, 2>::kStages;
    case kTile256x512: return Cfg<512, 2>::kStages;
  }
  return 0;
}

tbStatus tb_launch(const tb_matmul_plan* plan, const void* A, int64_t lda, const void* B,
                   int64_t ldb, void* Cp, int64_t ldc, void* workspace, size_t workspace_bytes,
                   void* stream_v) {
  return tb_launch_ex(plan, A, lda, B, ldb, Cp, ldc, nullptr, workspace, workspace_bytes, stream_v);
}

tbStatus tb_launch_ex(const tb_matmul_plan* plan, const void* A, int64_t lda, const void* B,
                      int64_t ldb, void* Cp, int64_t ldc, const float* bias, void* workspace,
                      size_t workspace_bytes, void* stream_v) {
  if (plan->dynamic)
    return tb_fail(TB_ERR_INVALID_ARGUMENT,
                   "this plan has dynamic dims: run it with tb_matmul_run_dynamic");
  const tb_matmul_desc& d = plan->desc;
  if (d.bias && !bias)
    return tb_fail(TB_ERR_INVALID_ARGUMENT,
                   "this plan applies a bias: pass it with tb_matmul_run_epilogue");
  if (!d.bias && bias)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "bias given to a plan made without desc.bias");
  if (!A || !B || !Cp) return tb_fail(TB_ERR_INVALID_ARGUMENT, "A, B and C must not be NULL");
  // Row-major A (m × k, row stride lda) is the reference layout; a_col_major
  // means A is stored column-major (lda = stride between columns, >= m).
  // Likewise B (k × n): row-major ldb >= n, column-major ldb >= k.
  if (lda < (d.a_col_major ? d.m : d.k) || ldb < (d.b_col_major ? d.k : d.n) || ldc < d.n)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "leading dimensions must be >= the row length");
  // TMA reads rows whose stride is a multiple of 16 bytes from a 16-byte
  // aligned base; other operands are first copied, zero-padded, into the
  // plan's packing space in the workspace.
  const bool pack_a = lda % 8 != 0 || !aligned16(A);
  const bool pack_b = ldb % 8 != 0 || !aligned16(B);
  if ((pack_a && !plan->pack_a_bytes) || (pack_b && !plan->pack_b_bytes))
    return tb_fail(TB_ERR_UNSUPPORTED,
                   "lda and ldb must be multiples of 8 elements and A, B 16-byte aligned "
                   "(16-byte TMA strides); only plans whose row length is not a multiple of 8 "
                   "reserve workspace to repack an operand");
  const bool need_ws = plan->partial_bytes > 0 || pack_a || pack_b;
  if (need_ws && (!workspace || workspace_bytes < plan->workspace_bytes))
    return tb_fail(TB_ERR_WORKSPACE, "this run needs a workspace of " +
                                         std::to_string(plan->workspace_bytes) + " bytes");
  if (d.m > INT32_MAX || d.n > INT32_MAX || d.k > INT32_MAX)
    return tb_fail(TB_ERR_UNSUPPORTED, "problem dimensions must fit in 32 bits");
  tbStatus st = get_encoder();
  if (st != TB_OK) return st;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_v);

  if (pack_a || pack_b) {
    uint8_t* wsb = static_cast<uint8_t*>(workspace);
    if (pack_a) {
      const int64_t rows = d.a_col_major ? d.k : d.m, cols = d.a_col_major ? d.m : d.k;
      const int64_t ld = (cols + 7) / 8 * 8;
      st = pack_rows_f16(A, lda, wsb + plan->pack_a_offset, ld, rows, cols, plan->num_sms, stream);
      if (st != TB_OK) return st;
      A = wsb + plan->pack_a_offset;
      lda = ld;
    }
    if (pack_b) {
      const int64_t rows = d.b_col_major ? d.n : d.k, cols = d.b_col_major ? d.k : d.n;
      const int64_t ld = (cols + 7) / 8 * 8;
      st = pack_rows_f16(B, ldb, wsb + plan->pack_b_offset, ld, rows, cols, plan->num_sms, stream);
      if (st != TB_OK) return st;
      B = wsb + plan->pack_b_offset;
      ldb = ld;
    }
  }

  CUtensorMap ta, tbm;
  memset(&ta, 0, sizeof(ta));
  memset(&tbm, 0, sizeof(tbm));
  if (plan->small)  // the latency kernel: [128 m × 64 k] A boxes (row-major only)
    st = encode_f16_2d(&ta, A, d.m, d.k, lda, kCtaM, "A");
  else if (d.a_col_major)  // storage k × m (m contiguous): [64 k × 64 m] boxes
    st = encode_f16_2d(&ta, A, d.k, d.m, lda, (uint32_t)plan->kb, "A");
  else                // storage m × k: [128 m × 64 k] boxes
    st = encode_f16_2d(&ta, A, d.m, d.k, lda, kCtaM, "A");
  if (st != TB_OK) return st;
  if (plan->small)  // [kSmallK k × 64 n] B boxes
    st = encode_f16_2d(&tbm, B, d.k, d.n, ldb, (uint32_t)kSmallK, "B");
  else if (d.b_col_major)  // storage n × k (k contiguous): [BN/G n × 64 k] boxes; the 256 × 512
                      // pair tile loads its 256 columns per CTA as two 128-row boxes
    st = encode_f16_2d(&tbm, B, d.n, d.k, ldb,
                       (uint32_t)(plan->cta_n > 256 ? 128 : plan->cta_n / plan->ctas_per_tile), "B");
  else                // storage k × n: [64 k × 64 n] boxes
    st = encode_f16_2d(&tbm, B, d.k, d.n, ldb, (uint32_t)plan->kb, "B");
  if (st != TB_OK) return st;

  const size_t out_bytes = d.c_dtype == TB_F16 ? 2 : 4;
  KParams kp;
  kp.map = plan->map;
  kp.M = (int32_t)d.m;
  kp.N = (int32_t)d.n;
  kp.K = (int32_t)d.k;
  kp.block_m = (int32_t)d.block_m;
  kp.block_n = (int32_t)d.block_n;
  kp.block_k = (int32_t)d.block_k;
  kp.epilogue = plan->epilogue;
  kp.beta = d.beta ? 1 : 0;
  kp.fuse = plan->fuse;
  kp.walk_grouped = tb::walk_mode(kp.map, plan->fuse);
  kp.work_items = (int32_t)plan->work_items;
  kp.sub_m = plan->sub_m;
  kp.sub_n = plan->sub_n;
  kp.dp_items = (int32_t)plan->dp_items;
  kp.tail_items = (int32_t)plan->tail_items;
  kp.tail_slots = (int32_t)std::max<int64_t>(1, plan->tail_slots);
  kp.tail_segs = (int32_t)plan->tail_segs;
  kp.tail_fills = (int32_t)std::max<int64_t>(1, plan->tail_fills);
  kp.positions = (int32_t)plan->positions;
  kp.a_mn = d.a_col_major ? 1 : 0;
  kp.b_kmaj = d.b_col_major ? 1 : 0;
  kp.ex.bias = d.bias ? bias : nullptr;
  kp.ex.act = d.activation;
  kp.ex.clamp = d.clamp;
  kp.ex.lo = d.clamp_lo;
  kp.ex.hi = d.clamp_hi;
  kp.ex.any = (d.bias || d.activation != TB_ACT_NONE || d.clamp) ? 1 : 0;
  kp.vec_c = aligned16(Cp) && ((ldc * (int64_t)out_bytes) % 16 == 0) &&
             ((d.block_n * (int64_t)out_bytes) % 16 == 0);
  kp.vec_ws = (d.n % 4 == 0) && (d.block_n % 4 == 0) && aligned16(workspace);
  kp.one_item = plan->positions <= plan->grid / plan->ctas_per_tile ? 1 : 0;
  kp.cin_smem = kp.one_item && kp.vec_c;
  kp.C = Cp;
  kp.ldc = ldc;
  kp.ws = reinterpret_cast<float*>(workspace);

  if (plan->epilogue == kEpiAtomic && !d.beta) {
    // C = A·B through atomics: start from zero.
    cudaError_t e = cudaMemset2DAsync(Cp, (size_t)ldc * 4, 0, (size_t)d.n * 4, (size_t)d.m, stream);
    if (e != cudaSuccess)
      return tb_fail(TB_ERR_CUDA, std::string("cudaMemset2DAsync: ") + cudaGetErrorString(e));
  }

  // TMA epilogue: f32 output, program tile == hardware tile (so a box never
  // covers a neighbour program's rows or columns), 16-byte aligned rows.
  CUtensorMap tcm;
  memset(&tcm, 0, sizeof(tcm));
  kp.tma_out = kTmaNone;
  if (plan->small) {
    // every item stages its C_in tile: by TMA boxes when C is TMA-addressable
    // (the kernel reads kp.tma_out == kTmaStoreC as "C map valid"), else by
    // per-row cp.async
    const bool cmap = d.beta && plan->epilogue == kEpiStore && aligned16(Cp) &&
                      ldc % (d.c_dtype == TB_F16 ? 8 : 4) == 0;
    kp.cin_smem = cmap ? 0 : kp.vec_c;
    if (cmap) kp.tma_out = kTmaStoreC;
  }
  const bool exact_hw_tile = !plan->small &&
      d.block_m * (plan->fuse == 1 || plan->fuse == 4 ? 2 : 1) == (int64_t)plan->cta_m * plan->sub_m &&
      d.block_n * (plan->fuse >= 2 ? 2 : 1) == (int64_t)plan->cta_n * plan->sub_n;
  if (exact_hw_tile && d.c_dtype == TB_F32 && aligned16(Cp) && ldc % 4 == 0) {
    if (plan->epilogue == kEpiStore) kp.tma_out = kTmaStoreC;
    if (plan->epilogue == kEpiAtomic) kp.tma_out = kTmaReduceC;
  }
  if (exact_hw_tile && d.c_dtype == TB_F16 && aligned16(Cp) && ldc % 8 == 0 && plan->epilogue == kEpiStore)
    kp.tma_out = kTmaStoreC;  // f16 C: [32 rows × 64 columns] boxes
  if (exact_hw_tile && plan->epilogue == kEpiWorkspace && aligned16(workspace) && d.n % 4 == 0)
    kp.tma_out = kTmaStoreWs;
  // The tail's K pieces reduce-add f32 partial tiles through the same C
  // tensor map; without it (C not TMA-addressable) every item runs whole.
  if (plan->tail_items && kp.tma_out != kTmaStoreC) {
    kp.dp_items = kp.work_items;
    kp.tail_items = 0;
    kp.tail_segs = 0;
    kp.positions = kp.work_items;
  }
  if (kp.tma_out != kTmaNone) {
    cuuint32_t box[3] = {32, 32, 1};
    CUresult r;
    if (kp.tma_out == kTmaStoreWs) {
      cuuint64_t dims[3] = {(cuuint64_t)d.n, (cuuint64_t)d.m, (cuuint64_t)kp.map.split_k};
      cuuint64_t strides[2] = {(cuuint64_t)d.n * 4, (cuuint64_t)d.m * (cuuint64_t)d.n * 4};
      r = encode_cached(&tcm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, workspace, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE);
    } else if (d.c_dtype == TB_F16) {
      cuuint64_t dims[2] = {(cuuint64_t)d.n, (cuuint64_t)d.m};
      cuuint64_t strides[1] = {(cuuint64_t)ldc * 2};
      cuuint32_t box16[2] = {64, 32};
      r = encode_cached(&tcm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Cp, dims, strides, box16,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE);
    } else {
      cuuint64_t dims[2] = {(cuuint64_t)d.n, (cuuint64_t)d.m};
      cuuint64_t strides[1] = {(cuuint64_t)ldc * 4};
      r = encode_cached(&tcm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, Cp, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE);
    }
    if (r != CUDA_SUCCESS)
      return tb_fail(TB_ERR_CUDA, "cuTensorMapEncodeTiled(C) failed with CUresult " +
                                      std::to_string((int)r));
  }

  if (plan->small)
    st = d.c_dtype == TB_F16 ? launch_small<__half>(plan, kp, ta, tbm, tcm, A, lda, B, ldb, stream, 1)
                             : launch_small<float>(plan, kp, ta, tbm, tcm, A, lda, B, ldb, stream, 0);
  else
    st = d.c_dtype == TB_F16 ? dispatch_tile<__half>(plan, ta, tbm, tcm, kp, stream, 1)
                             : dispatch_tile<float>(plan, ta, tbm, tcm, kp, stream, 0);
  if (st != TB_OK) return st;

  if (plan->epilogue == kEpiWorkspace) {
    const int64_t plane = d.m * d.n;
    const int vec = (d.n % 4 == 0) && aligned16(workspace) &&
                    (reinterpret_cast<uintptr_t>(Cp) % (4 * out_bytes) == 0) &&
                    ((ldc * (int64_t)out_bytes) % (4 * out_bytes) == 0);
    const int64_t items = vec ? plane / 4 : plane;
    int64_t blocks = (items + 255) / 256;
    const int64_t cap = (int64_t)plan->num_sms * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    cudaLaunchConfig_t rc = {};
    rc.gridDim = dim3((unsigned)blocks, 1, 1);
    rc.blockDim = dim3(256, 1, 1);
    rc.dynamicSmemBytes = 0;
    rc.stream = stream;
    cudaLaunchAttribute rattr[1];
    rattr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    rattr[0].val.programmaticStreamSerializationAllowed = 1;
    rc.attrs = rattr;
    rc.numAttrs = 1;
    cudaError_t le;
    if (d.c_dtype == TB_F16)
      le = cudaLaunchKernelEx(&rc, tb_splitk_reduce_kernel<__half>, (const float*)kp.ws,
                              (int32_t)kp.map.split_k, kp.M, kp.N, Cp, (int64_t)ldc, kp.beta,
                              (int32_t)vec, kp.ex);
    else
      le = cudaLaunchKernelEx(&rc, tb_splitk_reduce_kernel<float>, (const float*)kp.ws,
                              (int32_t)kp.map.split_k, kp.M, kp.N, Cp, (int64_t)ldc, kp.beta,
                              (int32_t)vec, kp.ex);
    if (le != cudaSuccess)
      return tb_fail(TB_ERR_CUDA, std::string("tb_splitk_reduce launch: ") + cudaGetErrorString(le));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
      return tb_fail(TB_ERR_CUDA, std::string("tb_splitk_reduce launch: ") + cudaGetErrorString(e));
  }
  return TB_OK;
}

// ------------------------------------------------ allocation-free entry point
//
// Scratch for tb_matmul_run_no_alloc: a fixed device array that lives in the
// module image, so a call never allocates. 16 MiB holds the split_k_serial
// partials of, e.g., 512 x 512 with split_k = 16. Every device that loads this
// library keeps the array until the process exits.
constexpr size_t kNoAllocScratchBytes = 16u << 20;
static __device__ __align__(256) unsigned char g_tb_no_alloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_no_alloc_mu;
void* g_no_alloc_addr[kMaxDevices] = {};

// The host-side name of g_tb_no_alloc_scratch is only a stand-in; its device
// address is looked up once per device, with that device current.
tbStatus no_alloc_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return tb_fail(TB_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return tb_fail(TB_ERR_UNSUPPORTED, "device ordinal beyond the library's table");
  std::lock_guard<std::mutex> lock(g_no_alloc_mu);
  if (!g_no_alloc_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_tb_no_alloc_scratch);
    if (e != cudaSuccess || !p)
      return tb_fail(TB_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") +
                                      cudaGetErrorString(e));
    g_no_alloc_addr[dev] = p;
  }
  *out = g_no_alloc_addr[dev];
  return TB_OK;
}
}  // namespace

extern "C" tbStatus tb_matmul_run_no_alloc(const tb_matmul_plan* plan, const void* A, int64_t lda,
                                           const void* B, int64_t ldb, void* C, int64_t ldc,
                                           void* stream) {
  tb_clear_error();
  if (!plan) return tb_fail(TB_ERR_INVALID_ARGUMENT, "plan must not be NULL");
  if (plan->dynamic)
    return tb_fail(TB_ERR_INVALID_ARGUMENT,
                   "this plan has dynamic dims: run it with tb_matmul_run_dynamic");
  const size_t need = plan->workspace_bytes;
  if (need > kNoAllocScratchBytes)
    return tb_fail(TB_ERR_WORKSPACE,
                   "tb_matmul_run_no_alloc: this plan needs " + std::to_string(need) +
                       " bytes of scratch; the built-in scratch holds at most " +
                       std::to_string(kNoAllocScratchBytes) +
                       " bytes (use tb_matmul_run with a caller-owned workspace)");
  void* scratch = nullptr;
  if (need > 0) {
    tbStatus st = no_alloc_scratch_address(&scratch);
    if (st != TB_OK) return st;
  }
  // Every split part writes all of its m x n partial plane before the
  // reduction reads it, so the scratch needs no clearing between calls.
  return tb_launch(plan, A, lda, B, ldb, C, ldc, scratch, need > 0 ? kNoAllocScratchBytes : 0, stream);
}

// Self-test of the failure-detection path: one warp waits, bounded by
// `budget` cycles, on an mbarrier nothing ever arrives on — the same probe,
// budget check and status recording the GEMM's waits use — then returns.
__global__ void tb_selftest_wait_kernel(long long budget) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(smem_addr(&bar), 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const long long t0 = clock64();
    while (!mbar_try_wait(smem_addr(&bar), 0)) {
      if (clock64() - t0 > budget) {
        record_error(TB_ERR_DEVICE_TIMEOUT, kSiteSelfTest);
        break;
      }
    }
  }
}

extern "C" tbStatus tb_selftest_bounded_wait(void* stream, uint64_t budget_cycles) {
  tb_clear_error();
  if (budget_cycles == 0 || budget_cycles > (uint64_t)kWaitBudgetCycles)
    return tb_fail(TB_ERR_INVALID_ARGUMENT, "budget_cycles must be in (0, 2e9]");
  tb_selftest_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>((long long)budget_cycles);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TB_OK
                          : tb_fail(TB_ERR_CUDA, std::string("tb_selftest launch: ") + cudaGetErrorString(e));
}

extern "C" tbStatus tb_device_status(void* stream, uint32_t* raw) {
  cudaError_t e = cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess)
    return tb_fail(TB_ERR_CUDA, std::string("cudaStreamSynchronize: ") + cudaGetErrorString(e));
  uint32_t v = 0;
  e = cudaMemcpyFromSymbol(&v, g_tb_status, sizeof(v));
  if (e != cudaSuccess)
    return tb_fail(TB_ERR_CUDA, std::string("cudaMemcpyFromSymbol: ") + cudaGetErrorString(e));
  if (raw) *raw = v;
  if (v != 0) {
    const uint32_t zero = 0;
    cudaMemcpyToSymbol(g_tb_status, &zero, sizeof(zero));
    char hex[16];
    std::snprintf(hex, sizeof hex, "%08x", v);
    return tb_fail(TB_ERR_DEVICE_TIMEOUT, std::string("a device-side wait timed out (status 0x") + hex +
                                              ": code << 24 | site << 16 | block)");
  }
  return TB_OK;
}
