/*
 * tb_oracle.c — CPU restatement of the reference `tb.matmul` semantics.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker the parity tests compare
 * the sm_100a kernels against, and the CPU baseline bench.py times; it is
 * never linked into or called by the product library.
 *
 * Semantics restated (C_out = C_in + A·B with f16 A/B widened to f32 and f32
 * accumulation):
 *   - op contract: include/tb/IR/TBOps.td:32-58
 *   - accumulator initialised from C when there is no split-K:
 *       lib/Transforms/LowerPipelineToNVGPU.cpp:994-999, :2192-2278
 *   - K loop of f16·f16→f32 products: :2454-2503 (mma.sync m16n8k16)
 *   - masked ragged edges (out-of-range A/B read as 0, C stores masked):
 *       :1983-2000, EpiloguePlan.cpp:915-919
 *   - the same contract stated in Triton:
 *       tools/build_triton_stage1_kernel.py:50-74
 * Parity status: pinned against golden vectors produced by running the
 * reference's own Triton statement of the op (tests/golden/make_golden.py).
 *
 * Build: gcc -O3 -pthread -march=x86-64-v3 -shared -fPIC (oracle/Makefile).
 * Threads: POSIX threads, tiles dealt round-robin (no OpenMP runtime needed).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <unistd.h>

/* IEEE-754 binary16 → binary32, exact (every f16 value is an f32 value). */
static inline float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1Fu;
  const uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: value = man · 2^-24 */
      float v = (float)man * (1.0f / 16777216.0f);
      memcpy(&bits, &v, 4);
      bits |= sign;
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float out;
  memcpy(&out, &bits, 4);
  return out;
}

void tb_oracle_f16_to_f32(const uint16_t* src, float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = f16_to_f32(src[i]);
}

int tb_oracle_max_threads(void) {
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

enum { MB = 32, NB = 256, KB = 256 };

typedef struct {
  const uint16_t* A;
  int64_t lda;
  const float* Bf; /* K×N widened B, row stride N */
  float* C;
  int64_t ldc, M, N, K;
  int beta, nthreads, tid;
  int64_t b_ldb;
  const uint16_t* B;
} job_t;

static void* widen_b(void* arg) {
  job_t* j = (job_t*)arg;
  float* Bf = (float*)j->Bf;
  for (int64_t k = j->tid; k < j->K; k += j->nthreads)
    for (int64_t c = 0; c < j->N; ++c) Bf[k * j->N + c] = f16_to_f32(j->B[k * j->b_ldb + c]);
  return NULL;
}

static void* gemm_tiles(void* arg) {
  job_t* jb = (job_t*)arg;
  const int64_t M = jb->M, N = jb->N, K = jb->K;
  const int64_t tiles_m = (M + MB - 1) / MB, tiles_n = (N + NB - 1) / NB;
  float acc[MB][NB];
  float arow[KB];
  for (int64_t t = jb->tid; t < tiles_m * tiles_n; t += jb->nthreads) {
    const int64_t i0 = (t / tiles_n) * MB, j0 = (t % tiles_n) * NB;
    const int64_t mi = (M - i0) < MB ? (M - i0) : MB;
    const int64_t nj = (N - j0) < NB ? (N - j0) : NB;
    for (int64_t i = 0; i < mi; ++i)
      for (int64_t j = 0; j < nj; ++j) acc[i][j] = jb->beta ? jb->C[(i0 + i) * jb->ldc + j0 + j] : 0.0f;
    for (int64_t k0 = 0; k0 < K; k0 += KB) {
      const int64_t kk = (K - k0) < KB ? (K - k0) : KB;
      for (int64_t i = 0; i < mi; ++i) {
        const uint16_t* ar = jb->A + (i0 + i) * jb->lda + k0;
        for (int64_t k = 0; k < kk; ++k) arow[k] = f16_to_f32(ar[k]);
        float* ci = acc[i];
        for (int64_t k = 0; k < kk; ++k) {
          const float a = arow[k];
          const float* br = jb->Bf + (k0 + k) * N + j0;
          for (int64_t j = 0; j < nj; ++j) ci[j] += a * br[j];
        }
      }
    }
    for (int64_t i = 0; i < mi; ++i)
      for (int64_t j = 0; j < nj; ++j) jb->C[(i0 + i) * jb->ldc + j0 + j] = acc[i][j];
  }
  return NULL;
}

/*
 * C[M×N] (row stride ldc) = (beta ? C : 0) + A[M×K] · B[K×N], f32 accumulate,
 * k ascending for every element, C_in added first. A and B hold raw f16
 * bits. `threads` <= 0 uses every online CPU.
 */
void tb_oracle_matmul(const uint16_t* A, int64_t lda, const uint16_t* B, int64_t ldb, float* C,
                      int64_t ldc, int64_t M, int64_t N, int64_t K, int beta, int threads) {
  if (M <= 0 || N <= 0) return;
  int nt = threads > 0 ? threads : tb_oracle_max_threads();
  if (nt > 256) nt = 256;
  float* Bf = (float*)malloc(sizeof(float) * (size_t)(K > 0 ? K : 1) * (size_t)N);
  if (!Bf) return;
  pthread_t th[256];
  job_t jobs[256];
  for (int pass = 0; pass < 2; ++pass) {
    for (int t = 0; t < nt; ++t) {
      job_t j = {A, lda, Bf, C, ldc, M, N, K, beta, nt, t, ldb, B};
      jobs[t] = j;
    }
    for (int t = 1; t < nt; ++t)
      pthread_create(&th[t], NULL, pass == 0 ? widen_b : gemm_tiles, &jobs[t]);
    if (pass == 0) widen_b(&jobs[0]); else gemm_tiles(&jobs[0]);
    for (int t = 1; t < nt; ++t) pthread_join(th[t], NULL);
  }
  free(Bf);
}
