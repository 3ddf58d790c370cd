/*
 * tg_oracle.c -- CPU restatement of the reference's tropical GEMM semantics.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA engine
 * (tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs use it);
 * the product path never links or calls it.
 *
 * What it restates (reference = TensorBFS/tropical-gemm v0.2.0):
 *  - float semirings: crates/tropical-gemm/src/types/max_plus.rs:29-74,
 *    min_plus.rs:29-72, max_mul.rs:29-72 (zero -inf/+inf/0, mul +/+/*, the
 *    strict argmax update that keeps the earlier k on ties, :67-73);
 *  - the argmax GEMM loop: crates/tropical-gemm/src/core/kernel.rs:119-167
 *    (accumulator starts at zero with index 0, k ascending, global k =
 *    k_offset + p) driven by the BLIS blocking of core/gemm.rs:167-244 with
 *    TilingParams::PORTABLE (mc=nc=64, kc=256, mr=nr=4; core/tiling.rs:39-45);
 *  - integer semirings with the GPU sentinels and saturating adds of
 *    crates/tropical-gemm-cuda/kernels/tropical_gemm.cu:15-60 (the integer
 *    contract of the GPU path);
 *  - value-only float reduction = CUDA fmaxf/fminf as used by the reference
 *    plain kernels (tropical_gemm.cu:1043-1050): NaN operands are ignored and
 *    max(+0,-0) = +0, min(+0,-0) = -0 (behaviour measured on sm_100).
 *
 *  - the reference CPU SIMD path without argmax for MaxPlus f32
 *    (crates/tropical-gemm/src/simd/dispatch.rs:44-84 picking
 *    Avx2MaxPlusF32Kernel, simd/kernels/avx2.rs:12-74, with
 *    TilingParams::F32_AVX2 mc=nc=256, kc=512, mr=nr=8; core/tiling.rs:21-27;
 *    5-loop driver core/gemm.rs:56-140).
 *
 * Build: see oracle/Makefile (gcc -O3 -mavx2 -mfma -fopenmp -ffp-contract=off,
 * no fast-math).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif
#if defined(__AVX2__)
#include <immintrin.h>
#endif

enum { MAXPLUS = 0, MINPLUS = 1, MAXMUL = 2 };
enum { F32 = 0, F64 = 1, I32 = 2, I64 = 3 };

#define INF_I32 46340
#define INF_I64 3037000499LL

/* ---------------------------------------------------------------- floats */
#define FLOAT_OPS(T, SFX, INF)                                                        \
  static inline T zero_##SFX(int s) { return s == MAXPLUS ? -INF : s == MINPLUS ? INF : (T)0; } \
  static inline T mul_##SFX(int s, T a, T b) { return s == MAXMUL ? a * b : a + b; }           \
  static inline int better_##SFX(int s, T p, T acc) { return s == MINPLUS ? p < acc : p > acc; } \
  static inline T reduce_##SFX(int s, T acc, T p) {                                  \
    if (isnan(p)) return acc;                                                        \
    if (isnan(acc)) return p;                                                        \
    if (s == MINPLUS) {                                                              \
      if (p < acc) return p;                                                         \
      if (p == acc && p == 0 && signbit(p)) return p;                                \
      return acc;                                                                    \
    }                                                                                \
    if (p > acc) return p;                                                           \
    if (p == acc && p == 0 && !signbit(p)) return p;                                 \
    return acc;                                                                      \
  }

FLOAT_OPS(float, f32, INFINITY)
FLOAT_OPS(double, f64, (double)INFINITY)

/* ---------------------------------------------------------------- integers */
static inline int32_t zero_i32(int s) { return s == MAXPLUS ? -INF_I32 : s == MINPLUS ? INF_I32 : 0; }
static inline int64_t zero_i64(int s) { return s == MAXPLUS ? -INF_I64 : s == MINPLUS ? INF_I64 : 0; }
static inline int32_t mul_i32(int s, int32_t a, int32_t b) {
  if (s == MAXPLUS) return (a == -INF_I32 || b == -INF_I32) ? -INF_I32 : (int32_t)((uint32_t)a + (uint32_t)b);
  if (s == MINPLUS) return (a == INF_I32 || b == INF_I32) ? INF_I32 : (int32_t)((uint32_t)a + (uint32_t)b);
  return (int32_t)((uint32_t)a * (uint32_t)b);
}
static inline int64_t mul_i64(int s, int64_t a, int64_t b) {
  if (s == MAXPLUS) return (a == -INF_I64 || b == -INF_I64) ? -INF_I64 : (int64_t)((uint64_t)a + (uint64_t)b);
  if (s == MINPLUS) return (a == INF_I64 || b == INF_I64) ? INF_I64 : (int64_t)((uint64_t)a + (uint64_t)b);
  return (int64_t)((uint64_t)a * (uint64_t)b);
}
#define INT_CMP(T, SFX)                                                                \
  static inline int better_##SFX(int s, T p, T acc) { return s == MINPLUS ? p < acc : p > acc; } \
  static inline T reduce_##SFX(int s, T acc, T p) { return better_##SFX(s, p, acc) ? p : acc; }
INT_CMP(int32_t, i32)
INT_CMP(int64_t, i64)

/* Straight triple loop over row-major A[m,k], B[k,n] -> C[m,n] (+argmax). */
#define SIMPLE_GEMM(T, SFX)                                                           \
  static void gemm_##SFX(int s, int64_t m, int64_t n, int64_t k, const T* a, const T* b, \
                         T* c, int32_t* am, int nthreads) {                           \
    _Pragma("omp parallel for schedule(dynamic, 4) num_threads(nthreads)")             \
    for (int64_t i = 0; i < m; ++i) {                                                 \
      for (int64_t j = 0; j < n; ++j) {                                               \
        T acc = zero_##SFX(s);                                                        \
        int32_t idx = 0;                                                              \
        for (int64_t p = 0; p < k; ++p) {                                             \
          T prod = mul_##SFX(s, a[i * k + p], b[p * n + j]);                          \
          if (am) {                                                                   \
            if (better_##SFX(s, prod, acc)) { acc = prod; idx = (int32_t)p; }         \
          } else {                                                                    \
            acc = reduce_##SFX(s, acc, prod);                                         \
          }                                                                           \
        }                                                                             \
        c[i * n + j] = acc;                                                           \
        if (am) am[i * n + j] = idx;                                                  \
      }                                                                               \
    }                                                                                 \
  }
SIMPLE_GEMM(float, f32)
SIMPLE_GEMM(double, f64)
SIMPLE_GEMM(int32_t, i32)
SIMPLE_GEMM(int64_t, i64)

int tg_oracle_gemm(int semiring, int dtype, int64_t m, int64_t n, int64_t k, const void* a, const void* b,
                   void* c, int32_t* argmax, int nthreads) {
  if (nthreads < 1) nthreads = 1;
  switch (dtype) {
    case F32: gemm_f32(semiring, m, n, k, (const float*)a, (const float*)b, (float*)c, argmax, nthreads); return 0;
    case F64: gemm_f64(semiring, m, n, k, (const double*)a, (const double*)b, (double*)c, argmax, nthreads); return 0;
    case I32: gemm_i32(semiring, m, n, k, (const int32_t*)a, (const int32_t*)b, (int32_t*)c, argmax, nthreads); return 0;
    case I64: gemm_i64(semiring, m, n, k, (const int64_t*)a, (const int64_t*)b, (int64_t*)c, argmax, nthreads); return 0;
  }
  return 1;
}

/*
 * The reference CPU argmax path for f32, as it runs: BLIS 5-loop blocking
 * (jc over nc=64, pc over kc=256, ic over mc=64) with packed panels and a
 * 4x4 scalar microkernel that carries (value, index) across kc blocks
 * (core/gemm.rs:196-243, core/kernel.rs:119-167).  The reference runs it on
 * one thread; nthreads > 1 splits the jc loop across threads, each with its
 * own packing buffers (the same arithmetic per output, so identical results).
 */
#define MC 64
#define NC 64
#define KC 256
#define MR 4
#define NR 4

static void micro_argmax_f32(int s, int mr, int nr, int kc, int koff, const float* pa, const float* pb,
                             float* c, int32_t* am, int64_t ldc) {
  float acc[MR][NR];
  int32_t idx[MR][NR];
  for (int i = 0; i < mr; ++i)
    for (int j = 0; j < nr; ++j) { acc[i][j] = c[i * ldc + j]; idx[i][j] = am[i * ldc + j]; }
  for (int p = 0; p < kc; ++p) {
    const int32_t kk = koff + p;
    for (int i = 0; i < mr; ++i) {
      const float av = pa[p * MR + i];
      for (int j = 0; j < nr; ++j) {
        const float prod = mul_f32(s, av, pb[p * NR + j]);
        if (better_f32(s, prod, acc[i][j])) { acc[i][j] = prod; idx[i][j] = kk; }
      }
    }
  }
  for (int i = 0; i < mr; ++i)
    for (int j = 0; j < nr; ++j) { c[i * ldc + j] = acc[i][j]; am[i * ldc + j] = idx[i][j]; }
}

int tg_oracle_blis_argmax_f32(int semiring, int64_t m, int64_t n, int64_t k, const float* a, const float* b,
                              float* c, int32_t* argmax, int nthreads) {
  if (nthreads < 1) nthreads = 1;
  const float z = zero_f32(semiring);
  for (int64_t e = 0; e < m * n; ++e) { c[e] = z; argmax[e] = 0; }
  if (m == 0 || n == 0 || k == 0) return 0;
  const int64_t njc = (n + NC - 1) / NC;
  _Pragma("omp parallel num_threads(nthreads)")
  {
    float* pa = (float*)malloc(sizeof(float) * MC * KC);
    float* pb = (float*)malloc(sizeof(float) * KC * NC);
    _Pragma("omp for schedule(dynamic, 1)")
    for (int64_t jb = 0; jb < njc; ++jb) {
      const int64_t jc = jb * NC, nc = (n - jc) < NC ? (n - jc) : NC;
      for (int64_t pc = 0; pc < k; pc += KC) {
        const int64_t kc = (k - pc) < KC ? (k - pc) : KC;
        /* pack B panel kc x nc into NR-wide slivers, zero padded */
        for (int64_t jr = 0; jr < nc; jr += NR)
          for (int64_t p = 0; p < kc; ++p)
            for (int j = 0; j < NR; ++j)
              pb[jr * kc + p * NR + j] = (jr + j < nc) ? b[(pc + p) * n + jc + jr + j] : 0.0f;
        for (int64_t ic = 0; ic < m; ic += MC) {
          const int64_t mc = (m - ic) < MC ? (m - ic) : MC;
          for (int64_t ir = 0; ir < mc; ir += MR)
            for (int64_t p = 0; p < kc; ++p)
              for (int i = 0; i < MR; ++i)
                pa[ir * kc + p * MR + i] = (ir + i < mc) ? a[(ic + ir + i) * k + pc + p] : 0.0f;
          for (int64_t jr = 0; jr < nc; jr += NR) {
            const int nr = (nc - jr) < NR ? (int)(nc - jr) : NR;
            for (int64_t ir = 0; ir < mc; ir += MR) {
              const int mr = (mc - ir) < MR ? (int)(mc - ir) : MR;
              micro_argmax_f32(semiring, mr, nr, (int)kc, (int)pc, pa + ir * kc, pb + jr * kc,
                               c + (ic + ir) * n + jc + jr, argmax + (ic + ir) * n + jc + jr, n);
            }
          }
        }
      }
    }
    free(pa);
    free(pb);
  }
  return 0;
}

/*
 * The reference CPU SIMD value-only path for MaxPlus f32: BLIS 5-loop
 * blocking (jc over nc=256, pc over kc=512, ic over mc=256), A packed into
 * 8-row slivers and B into 8-column slivers, and an 8x8 microkernel that
 * keeps one 8-lane vector per row of C: acc[i] = max(acc[i], a[i] + b[0..8)).
 * The vector max is the AVX `max_ps(acc, product)` that the reference's
 * f32x8::max compiles to, so NaN behaviour follows that instruction (not
 * pinned by any reference test).  C is read and written per kc block, as in
 * the reference, starting from the semiring zero.  nthreads > 1 splits the
 * jc loop (per-thread packing buffers; identical arithmetic per output).
 * Returns 1 when the build has no AVX2.
 */
#define SMC 256
#define SNC 256
#define SKC 512
#define SMR 8
#define SNR 8

int tg_oracle_simd_maxplus_f32(int64_t m, int64_t n, int64_t k, const float* a, const float* b, float* c,
                               int nthreads) {
#if defined(__AVX2__)
  if (nthreads < 1) nthreads = 1;
  for (int64_t e = 0; e < m * n; ++e) c[e] = -INFINITY;
  if (m == 0 || n == 0 || k == 0) return 0;
  const int64_t njc = (n + SNC - 1) / SNC;
  _Pragma("omp parallel num_threads(nthreads)")
  {
    float* pa = (float*)aligned_alloc(32, sizeof(float) * SMC * SKC);
    float* pb = (float*)aligned_alloc(32, sizeof(float) * SKC * SNC);
    _Pragma("omp for schedule(dynamic, 1)")
    for (int64_t jb = 0; jb < njc; ++jb) {
      const int64_t jc = jb * SNC, nc = (n - jc) < SNC ? (n - jc) : SNC;
      for (int64_t pc = 0; pc < k; pc += SKC) {
        const int64_t kc = (k - pc) < SKC ? (k - pc) : SKC;
        for (int64_t jr = 0; jr < nc; jr += SNR)
          for (int64_t p = 0; p < kc; ++p)
            for (int j = 0; j < SNR; ++j)
              pb[jr * kc + p * SNR + j] = (jr + j < nc) ? b[(pc + p) * n + jc + jr + j] : 0.0f;
        for (int64_t ic = 0; ic < m; ic += SMC) {
          const int64_t mc = (m - ic) < SMC ? (m - ic) : SMC;
          for (int64_t ir = 0; ir < mc; ir += SMR)
            for (int64_t p = 0; p < kc; ++p)
              for (int i = 0; i < SMR; ++i)
                pa[ir * kc + p * SMR + i] = (ir + i < mc) ? a[(ic + ir + i) * k + pc + p] : 0.0f;
          for (int64_t jr = 0; jr < nc; jr += SNR) {
            const int nr = (nc - jr) < SNR ? (int)(nc - jr) : SNR;
            for (int64_t ir = 0; ir < mc; ir += SMR) {
              const int mr = (mc - ir) < SMR ? (int)(mc - ir) : SMR;
              float* cp = c + (ic + ir) * n + jc + jr;
              const float* ap = pa + ir * kc;
              const float* bp = pb + jr * kc;
              __m256 acc[SMR];
              for (int i = 0; i < SMR; ++i) {
                float row[SNR];
                for (int j = 0; j < SNR; ++j) row[j] = (i < mr && j < nr) ? cp[i * n + j] : -INFINITY;
                acc[i] = _mm256_loadu_ps(row);
              }
              for (int64_t p = 0; p < kc; ++p) {
                const __m256 bv = _mm256_loadu_ps(bp + p * SNR);
                for (int i = 0; i < SMR; ++i)
                  acc[i] = _mm256_max_ps(acc[i], _mm256_add_ps(_mm256_set1_ps(ap[p * SMR + i]), bv));
              }
              for (int i = 0; i < mr; ++i) {
                float row[SNR];
                _mm256_storeu_ps(row, acc[i]);
                for (int j = 0; j < nr; ++j) cp[i * n + j] = row[j];
              }
            }
          }
        }
      }
    }
    free(pa);
    free(pb);
  }
  return 0;
#else
  (void)m; (void)n; (void)k; (void)a; (void)b; (void)c; (void)nthreads;
  return 1;
#endif
}

/*
 * SIMD argmax path for f32, all three semirings (the "AVX-512/AVX2 CPU path
 * for argmax" the reference lacks: its argmax microkernel,
 * crates/tropical-gemm/src/core/kernel.rs:119-167, is scalar).  Same BLIS
 * blocking as the AVX2 value-only path above (mc=nc=256, kc=512, 8x8 tiles),
 * one 8-lane accumulator and one 8-lane index vector per row of C.  Per k
 * (ascending, global k = pc + p) the product vector is compared strictly
 * against the accumulator (ordered compare: NaN never wins) and both the
 * value and the index are blended under that mask -- lane for lane the
 * scalar rule of types/max_plus.rs:67-73 (keep the earlier k on ties), so
 * values and indices equal tg_oracle_blis_argmax_f32 bit for bit.
 * Returns 1 when the build has no AVX2.
 */
int tg_oracle_simd_argmax_f32(int semiring, int64_t m, int64_t n, int64_t k, const float* a, const float* b,
                              float* c, int32_t* argmax, int nthreads) {
#if defined(__AVX2__)
  if (nthreads < 1) nthreads = 1;
  const float z = zero_f32(semiring);
  for (int64_t e = 0; e < m * n; ++e) { c[e] = z; argmax[e] = 0; }
  if (m == 0 || n == 0 || k == 0) return 0;
  const int64_t njc = (n + SNC - 1) / SNC;
  const int minplus = semiring == MINPLUS, maxmul = semiring == MAXMUL;
  _Pragma("omp parallel num_threads(nthreads)")
  {
    float* pa = (float*)aligned_alloc(32, sizeof(float) * SMC * SKC);
    float* pb = (float*)aligned_alloc(32, sizeof(float) * SKC * SNC);
    _Pragma("omp for schedule(dynamic, 1)")
    for (int64_t jb = 0; jb < njc; ++jb) {
      const int64_t jc = jb * SNC, nc = (n - jc) < SNC ? (n - jc) : SNC;
      for (int64_t pc = 0; pc < k; pc += SKC) {
        const int64_t kc = (k - pc) < SKC ? (k - pc) : SKC;
        for (int64_t jr = 0; jr < nc; jr += SNR)
          for (int64_t p = 0; p < kc; ++p)
            for (int j = 0; j < SNR; ++j)
              pb[jr * kc + p * SNR + j] = (jr + j < nc) ? b[(pc + p) * n + jc + jr + j] : 0.0f;
        for (int64_t ic = 0; ic < m; ic += SMC) {
          const int64_t mc = (m - ic) < SMC ? (m - ic) : SMC;
          for (int64_t ir = 0; ir < mc; ir += SMR)
            for (int64_t p = 0; p < kc; ++p)
              for (int i = 0; i < SMR; ++i)
                pa[ir * kc + p * SMR + i] = (ir + i < mc) ? a[(ic + ir + i) * k + pc + p] : 0.0f;
          for (int64_t jr = 0; jr < nc; jr += SNR) {
            const int nr = (nc - jr) < SNR ? (int)(nc - jr) : SNR;
            for (int64_t ir = 0; ir < mc; ir += SMR) {
              const int mr = (mc - ir) < SMR ? (int)(mc - ir) : SMR;
              float* cp = c + (ic + ir) * n + jc + jr;
              int32_t* ip = argmax + (ic + ir) * n + jc + jr;
              const float* ap = pa + ir * kc;
              const float* bp = pb + jr * kc;
              __m256 acc[SMR];
              __m256i idx[SMR];
              for (int i = 0; i < SMR; ++i) {
                float row[SNR];
                int32_t irow[SNR];
                for (int j = 0; j < SNR; ++j) {
                  const int in = i < mr && j < nr;
                  row[j] = in ? cp[i * n + j] : z;
                  irow[j] = in ? ip[i * n + j] : 0;
                }
                acc[i] = _mm256_loadu_ps(row);
                idx[i] = _mm256_loadu_si256((const __m256i*)irow);
              }
              for (int64_t p = 0; p < kc; ++p) {
                const __m256 bv = _mm256_loadu_ps(bp + p * SNR);
                const __m256i kv = _mm256_set1_epi32((int32_t)(pc + p));
                for (int i = 0; i < SMR; ++i) {
                  const __m256 av = _mm256_set1_ps(ap[p * SMR + i]);
                  const __m256 prod = maxmul ? _mm256_mul_ps(av, bv) : _mm256_add_ps(av, bv);
                  const __m256 win = minplus ? _mm256_cmp_ps(prod, acc[i], _CMP_LT_OQ)
                                             : _mm256_cmp_ps(prod, acc[i], _CMP_GT_OQ);
                  acc[i] = _mm256_blendv_ps(acc[i], prod, win);
                  idx[i] = _mm256_castps_si256(
                      _mm256_blendv_ps(_mm256_castsi256_ps(idx[i]), _mm256_castsi256_ps(kv), win));
                }
              }
              for (int i = 0; i < mr; ++i) {
                float row[SNR];
                int32_t irow[SNR];
                _mm256_storeu_ps(row, acc[i]);
                _mm256_storeu_si256((__m256i*)irow, idx[i]);
                for (int j = 0; j < nr; ++j) { cp[i * n + j] = row[j]; ip[i * n + j] = irow[j]; }
              }
            }
          }
        }
      }
    }
    free(pa);
    free(pb);
  }
  return 0;
#else
  (void)semiring; (void)m; (void)n; (void)k; (void)a; (void)b; (void)c; (void)argmax; (void)nthreads;
  return 1;
#endif
}

/*
 * Backward reference: ordered sums (row-major, contiguous).
 * want_a: grad_a[i, am[i,j]] += g[i,j] * (maxmul ? b[am, j] : 1)
 * else:   grad_b[am[i,j], j] += g[i,j] * (maxmul ? a[i, am] : 1)
 * Follows crates/tropical-gemm-python/src/lib.rs:212-300 (skips k >= K)
 * and the multiplicative rule of python/tropical_gemm/pytorch.py:521-548.
 */
#define BACKWARD(T, SFX)                                                              \
  static void backward_##SFX(int s, int want_a, int64_t m, int64_t n, int64_t k, const T* g, \
                             const int32_t* am, const T* partner, T* out) {           \
    if (want_a) memset(out, 0, sizeof(T) * m * k); else memset(out, 0, sizeof(T) * k * n); \
    for (int64_t i = 0; i < m; ++i)                                                   \
      for (int64_t j = 0; j < n; ++j) {                                               \
        const int32_t kk = am[i * n + j];                                             \
        if (kk < 0 || kk >= k) continue;                                              \
        T v = g[i * n + j];                                                           \
        if (want_a) {                                                                 \
          if (s == MAXMUL) v = v * partner[(int64_t)kk * n + j];                      \
          out[i * k + kk] += v;                                                       \
        } else {                                                                      \
          if (s == MAXMUL) v = v * partner[i * k + kk];                               \
          out[(int64_t)kk * n + j] += v;                                              \
        }                                                                             \
      }                                                                               \
  }
BACKWARD(float, f32)
BACKWARD(double, f64)

int tg_oracle_backward(int semiring, int dtype, int want_a, int64_t m, int64_t n, int64_t k, const void* grad_c,
                       const int32_t* argmax, const void* partner, void* out) {
  if (dtype == F32) { backward_f32(semiring, want_a, m, n, k, (const float*)grad_c, argmax, (const float*)partner, (float*)out); return 0; }
  if (dtype == F64) { backward_f64(semiring, want_a, m, n, k, (const double*)grad_c, argmax, (const double*)partner, (double*)out); return 0; }
  return 1;
}
