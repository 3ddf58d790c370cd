// Kernel dispatch of the engine (host templates), instantiated per semiring
// by tg_gemm_{maxplus,minplus,maxmul}.cu:
//  * f32: the fast kernels (values only, or argmax by k-pair tracking for
//    short K and by chunk detection for long K);
//  * f64: the wide kernel; i32 / i64: exact conversion to f32 / f64 behind a
//    device-side range gate, the exact integer kernel otherwise;
//  * anything else: the generic exact kernel.
#pragma once
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include "tg_internal.h"
#include "tg_semiring.cuh"
#include "tg_generic.cuh"
#include "tg_fast_f32.cuh"
#include "tg_argmax_fused.cuh"
#include "tg_wide.cuh"

namespace tgi {

template <int S, typename T>
__global__ void fill_zero_kernel(T* c, int32_t* idx, int64_t m, int64_t n, int64_t ldc, int64_t sc) {
  using R = tg::Ring<S, T>;
  T* cb = c + int64_t(blockIdx.y) * sc;
  int32_t* ib = idx ? idx + int64_t(blockIdx.y) * sc : nullptr;
  const int64_t total = m * n;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t o = (e / n) * ldc + e % n;
    cb[o] = R::zero();
    if (ib) ib[o] = 0;
  }
}

constexpr int64_t kPairMaxK = 1024;

// Long-K f32 argmax through the persistent fused-resolution kernel.  Needs
// 16-byte aligned A and B rows (TMA / 16-byte copies), a fresh C (no
// accumulate), K <= 2 x 1024 x 32 and stream-ordered scratch for two copies
// of B; returns TG_ERR_UNSUPPORTED (nothing launched) when any of that is
// missing, and the caller uses the chunk re-stream kernel instead.
// By default it runs where it measured faster than the chunk kernel -- K >=
// 8192 and at least 16 tiles per SM (8192^3: 41.9 vs 42.9 ms; 8192 x 16384
// x 8192: 78.1 vs 82.0; but 16384 x 4096 x 16384: 93.3 vs 92.7 and 4096^3:
// 6.13 vs 5.89) -- TROPICAL_GEMM_ARGMAX_FUSED=1 selects it wherever it is
// supported and =0 never.
template <int S>
tg_status launch_argmax_fused(const Problem& P, cudaStream_t st, float acc_init) {
  static const int mode = [] {
    const char* e = std::getenv("TROPICAL_GEMM_ARGMAX_FUSED");
    return e && e[0] == '0' ? 0 : (e && e[0] == '1' ? 1 : -1);
  }();
  const tg::GemmArgs& g = P.g;
  if (mode == 0 || g.accumulate || g.gate) return TG_ERR_UNSUPPORTED;
  const int64_t ntiles = P.batch * ((g.m + tg::kFBM - 1) / tg::kFBM) * ((g.n + tg::kFBN - 1) / tg::kFBN);
  if (mode < 0 && (g.k < 8192 || ntiles < 16 * int64_t(sm_count()))) return TG_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(g.a) & 15) || (reinterpret_cast<uintptr_t>(g.b) & 15) || g.lda % 4 || g.ldb % 4 ||
      (P.batch > 1 && (g.sa % 4 || g.sb % 4)))
    return TG_ERR_UNSUPPORTED;
  // chunks of two k-tiles, at most kFMaxChunks of them
  if (P.batch > 65535 || g.n > (int64_t(1) << 30) || g.k > int64_t(2) * tg::kFMaxChunks * tg::kFBK)
    return TG_ERR_UNSUPPORTED;
  auto kern = tg::fast_f32_argmax_fused_kernel<S>;
  if (ensure_smem(reinterpret_cast<const void*>(kern), tg::kFSmemFused) != TG_OK) {
    clear_error();
    return TG_ERR_UNSUPPORTED;
  }
  // scratch: B k-pair interleaved ([K2][np][2]) then B transposed ([N][kp])
  const int64_t np = (g.n + 3) & ~int64_t(3), k2 = (g.k + 1) / 2, kp = (g.k + 3) & ~int64_t(3);
  const size_t il_bytes = (size_t(P.batch) * size_t(k2) * size_t(np) * 8 + 1023) & ~size_t(1023);
  const size_t bytes = il_bytes + size_t(P.batch) * size_t(g.n) * size_t(kp) * 4;
  void* ws = nullptr;
  if (scratch_alloc(&ws, bytes, st) != cudaSuccess) {
    cudaGetLastError();
    return TG_ERR_UNSUPPORTED;
  }
  float* bil = static_cast<float*>(ws);
  float* bt = reinterpret_cast<float*>(static_cast<char*>(ws) + il_bytes);
  CUtensorMap tm_bil, tm_bt;
  std::memset(&tm_bil, 0, sizeof(tm_bil));
  std::memset(&tm_bt, 0, sizeof(tm_bt));
  if (!encode_tma_f32(bil, 2 * np, k2, 2 * np, P.batch, 2 * np * k2, 2 * tg::kFBN, tg::kFBK / 2, &tm_bil, false) ||
      !encode_tma_f32(bt, g.k, g.n, kp, P.batch, g.n * kp, tg::kFBK, tg::kFBN, &tm_bt, true)) {
    scratch_free(ws, st);
    return TG_ERR_UNSUPPORTED;
  }
  {
    // one pass over B writes both copies (32 x 32 blocks over n < np, k < kp)
    const int64_t bx = (np + 31) / 32, by = std::min<int64_t>((kp + 31) / 32, 65535);
    tg_status s = TG_OK;
    if (bx > 0x7fffffff) s = fail(TG_ERR_UNSUPPORTED, "problem too large for one launch");
    else {
      tg::copy_b_kernel<<<dim3(unsigned(bx), unsigned(by), unsigned(P.batch)), 256, 0, st>>>(
          static_cast<const float*>(g.b), g.k, g.n, g.ldb, g.sb, bil, np, bt, kp);
      s = check_launch("copy_b_kernel launch");
    }
    if (s != TG_OK) {
      scratch_free(ws, st);
      return s;
    }
  }
  tg::FusedArgs w;
  w.p = g;
  w.nbatch = P.batch;
  w.acc_init = acc_init;
  const unsigned grid = unsigned(std::min<int64_t>(ntiles, sm_count()));
  kern<<<grid, tg::kFThreads, tg::kFSmemFused, st>>>(w, tm_bil, tm_bt);
  tg_status s = check_launch("fast_f32_argmax_fused_kernel launch");
  scratch_free(ws, st);
  return s;
}

template <int S, bool ARGMAX, bool OUTI = false>
tg_status launch_fast_f32(const Problem& P, cudaStream_t st, float acc_init) {
  // variant: argmax by chunk re-stream or by k-pair tracking (short K; with
  // B's panel resident in shared memory up to K = 256);
  // A staged by 16-byte copies when every batch's A rows are 16-byte aligned
  const bool pair = ARGMAX && P.g.k <= kPairMaxK;
  const bool panel = !OUTI && pair && P.g.k <= tg::kPanelMaxK;
  const size_t smem = panel ? tg::kFSmemPanel : (ARGMAX && !pair ? tg::kFSmemArgmax : tg::kFSmemValues);
  const bool avec = (reinterpret_cast<uintptr_t>(P.g.a) & 15) == 0 && P.g.lda % 4 == 0 &&
                    (P.batch == 1 || P.g.sa % 4 == 0);
  using KernT = void (*)(tg::GemmArgs, int, int, float, const CUtensorMap, const CUtensorMap, int);
  KernT kern;
  if constexpr (OUTI) {   // the i32 path stages padded, aligned copies
    kern = pair ? tg::fast_f32_kernel<S, ARGMAX, OUTI, true> : tg::fast_f32_kernel<S, ARGMAX, OUTI, false>;
  } else {
    if (panel) kern = avec ? tg::fast_f32_kernel<S, ARGMAX, false, true, true, true>
                           : tg::fast_f32_kernel<S, ARGMAX, false, true, false, true>;
    else if (pair) kern = avec ? tg::fast_f32_kernel<S, ARGMAX, false, true, true> : tg::fast_f32_kernel<S, ARGMAX, false, true, false>;
    else kern = avec ? tg::fast_f32_kernel<S, ARGMAX, false, false, true> : tg::fast_f32_kernel<S, ARGMAX, false, false, false>;
  }
  {
    tg_status s = ensure_smem(reinterpret_cast<const void*>(kern), smem);
    if (s != TG_OK) return s;
  }
  const int64_t ktiles = (P.g.k + tg::kFBK - 1) / tg::kFBK;
  int tpc = 2;
  const int b_vec = ((reinterpret_cast<uintptr_t>(P.g.b) & 15) == 0 && P.g.ldb % 4 == 0 &&
                     (P.batch == 1 || P.g.sb % 4 == 0)) ? 1 : 0;
  while ((ktiles + tpc - 1) / tpc > tg::kFMaxChunks) tpc *= 2;
  if constexpr (ARGMAX && !OUTI) {
    if (!pair) {
      const tg_status s = launch_argmax_fused<S>(P, st, acc_init);
      if (s != TG_ERR_UNSUPPORTED) return s;
    }
  }
  // (Short K: the re-stream costs as much per output as at long K, so the
  // argmax is tracked per k-pair in registers instead; measured crossover K ~ 1024-1536.)
  const int64_t gx = (P.g.m + tg::kFBM - 1) / tg::kFBM;
  const int64_t gy = (P.g.n + tg::kFBN - 1) / tg::kFBN;
  if (gx > 0x7fffffff || gy > 65535) return fail(TG_ERR_UNSUPPORTED, "problem too large for one launch");
  for (int64_t b0 = 0; b0 < P.batch; b0 += 65535) {
    const int64_t nb = std::min<int64_t>(65535, P.batch - b0);
    tg::GemmArgs g = P.g;
    g.a = static_cast<const float*>(g.a) + b0 * g.sa;
    g.b = static_cast<const float*>(g.b) + b0 * g.sb;
    g.c = static_cast<float*>(g.c) + b0 * g.sc;
    if (ARGMAX) g.argmax = g.argmax + b0 * g.sc;
    // the chunk re-stream by TMA when A and B rows and batch strides are 16-byte aligned
    CUtensorMap ta, tb;
    std::memset(&ta, 0, sizeof(ta));
    std::memset(&tb, 0, sizeof(tb));
    int use_tma = 0;
    if (ARGMAX && !pair && avec && b_vec && (reinterpret_cast<uintptr_t>(g.a) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(g.b) & 15) == 0 && (nb == 1 || (g.sa % 4 == 0 && g.sb % 4 == 0)))
      use_tma = encode_tma_f32(g.a, g.k, g.m, g.lda, nb, g.sa, tg::kFBK, tg::kFBM, &ta) &&
                encode_tma_f32(g.b, g.n, g.k, g.ldb, nb, g.sb, 32, tg::kFBK, &tb);
    kern<<<dim3(unsigned(gx), unsigned(gy), unsigned(nb)), tg::kFThreads, smem, st>>>(g, tpc, b_vec, acc_init, ta, tb,
                                                                                       use_tma);
    tg_status s = check_launch("fast_f32_kernel launch");
    if (s != TG_OK) return s;
  }
  return TG_OK;
}

template <int S, bool ARGMAX, bool OUTI = false>
tg_status launch_wide_f64(const Problem& P, cudaStream_t st, double acc_init) {
  auto kern = tg::wide_f64_kernel<S, ARGMAX, OUTI>;
  {
    tg_status s = ensure_smem(reinterpret_cast<const void*>(kern), tg::kWSmem);
    if (s != TG_OK) return s;
  }
  const int64_t gx = (P.g.m + tg::kWBM - 1) / tg::kWBM;
  const int64_t gy = (P.g.n + tg::kWBN - 1) / tg::kWBN;
  if (gx > 0x7fffffff || gy > 65535) return fail(TG_ERR_UNSUPPORTED, "problem too large for one launch");
  for (int64_t b0 = 0; b0 < P.batch; b0 += 65535) {
    const int64_t nb = std::min<int64_t>(65535, P.batch - b0);
    tg::GemmArgs g = P.g;
    g.a = static_cast<const double*>(g.a) + b0 * g.sa;
    g.b = static_cast<const double*>(g.b) + b0 * g.sb;
    g.c = static_cast<double*>(g.c) + b0 * g.sc;
    if (ARGMAX) g.argmax = g.argmax + b0 * g.sc;
    kern<<<dim3(unsigned(gx), unsigned(gy), unsigned(nb)), tg::kWThreads, tg::kWSmem, st>>>(g, acc_init);
    tg_status s = check_launch("wide_f64_kernel launch");
    if (s != TG_OK) return s;
  }
  return TG_OK;
}

template <int S, typename T, bool ARGMAX>
tg_status launch_generic(const Problem& P, cudaStream_t st) {
  const int64_t gx = (P.g.m + tg::kGenBM - 1) / tg::kGenBM;
  const int64_t gy = (P.g.n + tg::kGenBN - 1) / tg::kGenBN;
  if (gx > 0x7fffffff || gy > 65535) return fail(TG_ERR_UNSUPPORTED, "problem too large for one launch");
  for (int64_t b0 = 0; b0 < P.batch; b0 += 65535) {
    const int64_t nb = std::min<int64_t>(65535, P.batch - b0);
    tg::GemmArgs g = P.g;
    g.a = static_cast<const T*>(g.a) + b0 * g.sa;
    g.b = static_cast<const T*>(g.b) + b0 * g.sb;
    g.c = static_cast<T*>(g.c) + b0 * g.sc;
    if (ARGMAX) g.argmax = g.argmax + b0 * g.sc;
    tg::generic_gemm_kernel<S, T, ARGMAX><<<dim3(unsigned(gx), unsigned(gy), unsigned(nb)), tg::kGenThreads, 0, st>>>(g);
    tg_status s = check_launch("generic_gemm_kernel launch");
    if (s != TG_OK) return s;
  }
  return TG_OK;
}

// ---------------------------------------------------------------- i32 path
// Integer MaxPlus / MinPlus / MaxMul are computed exactly in f32 when every
// operand is small enough: |x| <= 2^23 for the additive semirings (sums stay
// below 2^24, so every f32 sum is the exact integer sum and never wraps) and
// |x| <= 4096 for MaxMul (products below 2^24).  The reference's sentinel
// (+46340 for MinPlus, -46340 for MaxPlus; tropical_gemm.cu:15-50) becomes
// +-inf, whose products never win, and the accumulator starts at the sentinel
// itself, so a finite product equal to or beyond it never wins either --
// exactly the saturating-add semantics.  Operands are converted into stream-
// ordered scratch (the library's own memory pool) together with an out-of-range flag; the
// fast f32 kernel and the exact integer kernel are both enqueued behind that
// flag, and whichever does not apply exits at once.  No host synchronisation.
constexpr int64_t kI32FastMinOutputs = 128 * 128;

template <int S>
__global__ void i32_to_f32_kernel(const int32_t* __restrict__ src, float* __restrict__ dst, int64_t rows,
                                  int64_t cols, int64_t ld, int64_t stride, int64_t dld, int* flag) {
  const int32_t* s = src + int64_t(blockIdx.y) * stride;
  float* d = dst + int64_t(blockIdx.y) * rows * dld;
  const int64_t total = rows * cols;
  const int32_t lim = S == tg::kMaxMul ? 4096 : (1 << 23);
  bool bad = false;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int32_t x = s[(e / cols) * ld + e % cols];
    float v;
    if (S == tg::kMinPlus && x == tg::kInfI32) v = INFINITY;
    else if (S == tg::kMaxPlus && x == -tg::kInfI32) v = -INFINITY;
    else {
      v = float(x);
      if (x > lim || x < -lim) bad = true;
    }
    d[(e / cols) * dld + e % cols] = v;
  }
  if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(flag, 1);
}

template <int S>
tg_status launch_i32_via_f32(const Problem& P, cudaStream_t st) {
  // scratch rows padded to 16 bytes (the fast kernel's vector loads)
  const int64_t lda_f = (P.g.k + 3) & ~int64_t(3), ldb_f = (P.g.n + 3) & ~int64_t(3);
  const int64_t asz = P.g.m * lda_f, bsz = P.g.k * ldb_f;
  const size_t bytes = size_t(P.batch) * size_t(asz + bsz) * 4 + 256;
  void* ws = nullptr;
  cudaError_t e = scratch_alloc(&ws, bytes, st);
  if (e != cudaSuccess) {  // no scratch: exact integer kernel only
    cudaGetLastError();
    return P.g.argmax ? launch_generic<S, int32_t, true>(P, st) : launch_generic<S, int32_t, false>(P, st);
  }
  int* flag = static_cast<int*>(ws);
  float* af = reinterpret_cast<float*>(static_cast<char*>(ws) + 256);
  float* bf = af + size_t(P.batch) * asz;
  tg_status s = TG_OK;
  if (cudaMemsetAsync(flag, 0, sizeof(int), st) != cudaSuccess) s = fail(TG_ERR_CUDA, "cudaMemsetAsync failed");
  for (int64_t b0 = 0; s == TG_OK && b0 < P.batch; b0 += 65535) {
    const int64_t nb = std::min<int64_t>(65535, P.batch - b0);
    i32_to_f32_kernel<S><<<dim3(1024, unsigned(nb)), 256, 0, st>>>(
        static_cast<const int32_t*>(P.g.a) + b0 * P.g.sa, af + b0 * asz, P.g.m, P.g.k, P.g.lda, P.g.sa, lda_f, flag);
    i32_to_f32_kernel<S><<<dim3(1024, unsigned(nb)), 256, 0, st>>>(
        static_cast<const int32_t*>(P.g.b) + b0 * P.g.sb, bf + b0 * bsz, P.g.k, P.g.n, P.g.ldb, P.g.sb, ldb_f, flag);
    s = check_launch("i32_to_f32_kernel launch");
  }
  if (s == TG_OK) {
    Problem F = P;
    F.g.a = af; F.g.lda = lda_f; F.g.sa = asz;
    F.g.b = bf; F.g.ldb = ldb_f; F.g.sb = bsz;
    F.g.gate = flag; F.g.gate_run_if_set = 0;
    const float init = S == tg::kMaxPlus ? -float(tg::kInfI32) : (S == tg::kMinPlus ? float(tg::kInfI32) : 0.0f);
    s = P.g.argmax ? launch_fast_f32<S, true, true>(F, st, init) : launch_fast_f32<S, false, true>(F, st, init);
  }
  if (s == TG_OK) {
    Problem X = P;
    X.g.gate = flag; X.g.gate_run_if_set = 1;
    s = P.g.argmax ? launch_generic<S, int32_t, true>(X, st) : launch_generic<S, int32_t, false>(X, st);
  }
  scratch_free(ws, st);
  return s;
}

// ---------------------------------------------------------------- i64 path
// Same idea as the i32 path, in f64: exact while |x| <= 2^51 (additive; sums
// below 2^52) or |x| <= 2^26 (MaxMul; products below 2^52); the sentinel
// +-3037000499 becomes +-inf and the accumulator starts at the sentinel.
template <int S>
__global__ void i64_to_f64_kernel(const int64_t* __restrict__ src, double* __restrict__ dst, int64_t rows,
                                  int64_t cols, int64_t ld, int64_t stride, int64_t dld, int* flag) {
  const int64_t* s = src + int64_t(blockIdx.y) * stride;
  double* d = dst + int64_t(blockIdx.y) * rows * dld;
  const int64_t total = rows * cols;
  const int64_t lim = S == tg::kMaxMul ? (int64_t(1) << 26) : (int64_t(1) << 51);
  bool bad = false;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t x = s[(e / cols) * ld + e % cols];
    double v;
    if (S == tg::kMinPlus && x == tg::kInfI64) v = INFINITY;
    else if (S == tg::kMaxPlus && x == -tg::kInfI64) v = -INFINITY;
    else {
      v = double(x);
      if (x > lim || x < -lim) bad = true;
    }
    d[(e / cols) * dld + e % cols] = v;
  }
  if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(flag, 1);
}

template <int S>
tg_status launch_i64_via_f64(const Problem& P, cudaStream_t st) {
  const int64_t lda_f = (P.g.k + 1) & ~int64_t(1), ldb_f = (P.g.n + 1) & ~int64_t(1);
  const int64_t asz = P.g.m * lda_f, bsz = P.g.k * ldb_f;
  const size_t bytes = size_t(P.batch) * size_t(asz + bsz) * 8 + 256;
  void* ws = nullptr;
  if (scratch_alloc(&ws, bytes, st) != cudaSuccess) {
    cudaGetLastError();
    return P.g.argmax ? launch_generic<S, int64_t, true>(P, st) : launch_generic<S, int64_t, false>(P, st);
  }
  int* flag = static_cast<int*>(ws);
  double* af = reinterpret_cast<double*>(static_cast<char*>(ws) + 256);
  double* bf = af + size_t(P.batch) * asz;
  tg_status s = TG_OK;
  if (cudaMemsetAsync(flag, 0, sizeof(int), st) != cudaSuccess) s = fail(TG_ERR_CUDA, "cudaMemsetAsync failed");
  for (int64_t b0 = 0; s == TG_OK && b0 < P.batch; b0 += 65535) {
    const int64_t nb = std::min<int64_t>(65535, P.batch - b0);
    i64_to_f64_kernel<S><<<dim3(1024, unsigned(nb)), 256, 0, st>>>(
        static_cast<const int64_t*>(P.g.a) + b0 * P.g.sa, af + b0 * asz, P.g.m, P.g.k, P.g.lda, P.g.sa, lda_f, flag);
    i64_to_f64_kernel<S><<<dim3(1024, unsigned(nb)), 256, 0, st>>>(
        static_cast<const int64_t*>(P.g.b) + b0 * P.g.sb, bf + b0 * bsz, P.g.k, P.g.n, P.g.ldb, P.g.sb, ldb_f, flag);
    s = check_launch("i64_to_f64_kernel launch");
  }
  if (s == TG_OK) {
    Problem F = P;
    F.g.a = af; F.g.lda = lda_f; F.g.sa = asz;
    F.g.b = bf; F.g.ldb = ldb_f; F.g.sb = bsz;
    F.g.gate = flag; F.g.gate_run_if_set = 0;
    const double init = S == tg::kMaxPlus ? -double(tg::kInfI64) : (S == tg::kMinPlus ? double(tg::kInfI64) : 0.0);
    s = P.g.argmax ? launch_wide_f64<S, true, true>(F, st, init) : launch_wide_f64<S, false, true>(F, st, init);
  }
  if (s == TG_OK) {
    Problem X = P;
    X.g.gate = flag; X.g.gate_run_if_set = 1;
    s = P.g.argmax ? launch_generic<S, int64_t, true>(X, st) : launch_generic<S, int64_t, false>(X, st);
  }
  scratch_free(ws, st);
  return s;
}

template <int S, typename T>
tg_status dispatch_typed(const Problem& P, cudaStream_t st) {
  const bool am = P.g.argmax != nullptr;
  if (P.g.k == 0) {
    for (int64_t b0 = 0; b0 < P.batch; b0 += 65535) {
      const int64_t nb = std::min<int64_t>(65535, P.batch - b0);
      fill_zero_kernel<S, T><<<dim3(256, unsigned(nb)), 256, 0, st>>>(
          static_cast<T*>(P.g.c) + b0 * P.g.sc, am ? P.g.argmax + b0 * P.g.sc : nullptr,
          P.g.m, P.g.n, P.g.ldc, P.g.sc);
      tg_status s = check_launch("fill_zero_kernel launch");
      if (s != TG_OK) return s;
    }
    return TG_OK;
  }
  if constexpr (std::is_same<T, float>::value) {
    const float z = S == tg::kMaxPlus ? -INFINITY : (S == tg::kMinPlus ? INFINITY : 0.0f);
    if (fast_f32_ok(P)) return am ? launch_fast_f32<S, true>(P, st, z) : launch_fast_f32<S, false>(P, st, z);
  }
  if constexpr (std::is_same<T, int32_t>::value) {
    if (P.g.m * P.g.n >= kI32FastMinOutputs && fast_f32_ok(P)) return launch_i32_via_f32<S>(P, st);
  }
  if constexpr (std::is_same<T, double>::value) {
    const double z = S == tg::kMaxPlus ? -double(INFINITY) : (S == tg::kMinPlus ? double(INFINITY) : 0.0);
    // the wide kernel: strict update for argmax; value-only a strict select
    // with a zero-sign re-run (equal to the fmax/fmin fold, about twice its rate)
    return am ? launch_wide_f64<S, true>(P, st, z) : launch_wide_f64<S, false>(P, st, z);
  }
  if constexpr (std::is_same<T, int64_t>::value) {
    if (P.g.m * P.g.n >= kI32FastMinOutputs) return launch_i64_via_f64<S>(P, st);
  }
  return am ? launch_generic<S, T, true>(P, st) : launch_generic<S, T, false>(P, st);
}

template <int S>
tg_status dispatch(tg_dtype dtype, const Problem& P, cudaStream_t st) {
  switch (dtype) {
    case TG_F32: return dispatch_typed<S, float>(P, st);
    case TG_F64: return dispatch_typed<S, double>(P, st);
    case TG_I32: return dispatch_typed<S, int32_t>(P, st);
    case TG_I64: return dispatch_typed<S, int64_t>(P, st);
  }
  return fail(TG_ERR_INVALID_ARGUMENT, "unknown dtype %d", int(dtype));
}

template <int S>
tg_status noalloc_i32(const Problem& P, cudaStream_t st, unsigned char* ws) {
  const int64_t lda_f = (P.g.k + 3) & ~int64_t(3), ldb_f = (P.g.n + 3) & ~int64_t(3);
  const int64_t asz = P.g.m * lda_f, bsz = P.g.k * ldb_f;
  int* flag = reinterpret_cast<int*>(ws);
  float* af = reinterpret_cast<float*>(ws + 256);
  float* bf = af + asz;
  // the array keeps the previous call's contents: the flag must start at zero
  if (cudaMemsetAsync(flag, 0, sizeof(int), st) != cudaSuccess) return fail(TG_ERR_CUDA, "cudaMemsetAsync failed");
  i32_to_f32_kernel<S><<<dim3(1024, 1), 256, 0, st>>>(static_cast<const int32_t*>(P.g.a), af, P.g.m, P.g.k,
                                                      P.g.lda, 0, lda_f, flag);
  i32_to_f32_kernel<S><<<dim3(1024, 1), 256, 0, st>>>(static_cast<const int32_t*>(P.g.b), bf, P.g.k, P.g.n,
                                                      P.g.ldb, 0, ldb_f, flag);
  tg_status s = check_launch("i32_to_f32_kernel launch");
  if (s != TG_OK) return s;
  Problem F = P;
  F.g.a = af; F.g.lda = lda_f; F.g.sa = asz;
  F.g.b = bf; F.g.ldb = ldb_f; F.g.sb = bsz;
  F.g.gate = flag; F.g.gate_run_if_set = 0;
  const float init = S == tg::kMaxPlus ? -float(tg::kInfI32) : (S == tg::kMinPlus ? float(tg::kInfI32) : 0.0f);
  s = P.g.argmax ? launch_fast_f32<S, true, true>(F, st, init) : launch_fast_f32<S, false, true>(F, st, init);
  if (s != TG_OK) return s;
  Problem X = P;
  X.g.gate = flag; X.g.gate_run_if_set = 1;
  return P.g.argmax ? launch_generic<S, int32_t, true>(X, st) : launch_generic<S, int32_t, false>(X, st);
}

#define TG_INSTANTIATE_SEMIRING(S)                                                        \
  template tg_status dispatch<S>(tg_dtype, const Problem&, cudaStream_t);                 \
  template tg_status noalloc_i32<S>(const Problem&, cudaStream_t, unsigned char*);

}  // namespace tgi
