// C ABI of the engine: validation, layout mapping and kernel dispatch.
// Declarations and per-function contracts live in include/tropical_gemm_b200.h.
//
// Host-side responsibilities (the reference's cu/src/{kernels,lib}.rs):
//  * shape / leading-dimension / pointer checks with error codes instead
//    of Rust `Result`s (crates/tropical-gemm-cuda/src/error.rs:8-29);
//  * column-major callers become the canonical row-major problem
//    C^T = B^T (x) A^T by swapping operands and M <-> N -- the same trick
//    the reference applies for row-major DLPack tensors (kernels.rs:416-430),
//    here in the opposite direction;
//  * kernel choice: the f32 fast path when alignment allows, else the
//    generic exact kernel;
//  * stream-ordered launches only: no allocation, no synchronisation.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <algorithm>
#include <mutex>
#include <cuda_runtime.h>
#include "../../include/tropical_gemm_b200.h"
#include "tg_semiring.cuh"
#include "tg_generic.cuh"
#include "tg_fast_f32.cuh"
#include "tg_backward.cuh"
#include "tg_wide.cuh"

namespace {

thread_local std::string g_last_error;

tg_status fail(tg_status s, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
tg_status fail(tg_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return s;
}

tg_status check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(TG_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return TG_OK;
}

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

struct Problem {
  tg::GemmArgs g;
  int64_t batch;
};

bool fast_f32_ok(const Problem& P) {
  const auto& g = P.g;
  // any A alignment: the kernel switches to 4-byte copies for unaligned rows
  if (g.k >= (int64_t(1) << 31)) return false;
  // argmax: the re-stream ring holds whole chunks of <= 4 k-tiles (1024 chunks)
  if (g.argmax && (g.k + tg::kFBK - 1) / tg::kFBK > int64_t(4) * tg::kFMaxChunks) return false;
  return true;
}

constexpr int64_t kPairMaxK = 1024;

template <int S, bool ARGMAX, bool OUTI = false>
tg_status launch_fast_f32(const Problem& P, cudaStream_t st, float acc_init) {
  const size_t smem = ARGMAX ? tg::kFSmemArgmax : tg::kFSmemValues;
  // variant: argmax by chunk re-stream or by k-pair tracking (short K);
  // A staged by 16-byte copies when every batch's A rows are 16-byte aligned
  const bool pair = ARGMAX && P.g.k <= kPairMaxK;
  const bool avec = (reinterpret_cast<uintptr_t>(P.g.a) & 15) == 0 && P.g.lda % 4 == 0 &&
                    (P.batch == 1 || P.g.sa % 4 == 0);
  using KernT = void (*)(tg::GemmArgs, int, int, float);
  KernT kern;
  int variant;
  if constexpr (OUTI) {   // the i32 path stages padded, aligned copies
    kern = pair ? tg::fast_f32_kernel<S, ARGMAX, OUTI, true> : tg::fast_f32_kernel<S, ARGMAX, OUTI, false>;
    variant = pair ? 1 : 0;
  } else {
    if (pair) kern = avec ? tg::fast_f32_kernel<S, ARGMAX, false, true, true> : tg::fast_f32_kernel<S, ARGMAX, false, true, false>;
    else kern = avec ? tg::fast_f32_kernel<S, ARGMAX, false, false, true> : tg::fast_f32_kernel<S, ARGMAX, false, false, false>;
    variant = (pair ? 1 : 0) + (avec ? 0 : 2);
  }
  static bool configured[64][4] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev][variant]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return fail(TG_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    configured[dev][variant] = true;
  }
  const int64_t ktiles = (P.g.k + tg::kFBK - 1) / tg::kFBK;
  int tpc = 2;
  const int b_vec = ((reinterpret_cast<uintptr_t>(P.g.b) & 15) == 0 && P.g.ldb % 4 == 0 &&
                     (P.batch == 1 || P.g.sb % 4 == 0)) ? 1 : 0;
  while ((ktiles + tpc - 1) / tpc > tg::kFMaxChunks) tpc *= 2;
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
    kern<<<dim3(unsigned(gx), unsigned(gy), unsigned(nb)), tg::kFThreads, smem, st>>>(g, tpc, b_vec, acc_init);
    tg_status s = check_launch("fast_f32_kernel launch");
    if (s != TG_OK) return s;
  }
  return TG_OK;
}

template <int S, bool ARGMAX, bool OUTI = false>
tg_status launch_wide_f64(const Problem& P, cudaStream_t st, double acc_init) {
  auto kern = tg::wide_f64_kernel<S, ARGMAX, OUTI>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(tg::kWSmem));
    if (e != cudaSuccess) return fail(TG_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    configured[dev] = true;
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
// ordered scratch (cudaMallocAsync) together with an out-of-range flag; the
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

// Stream-ordered scratch from the device's default memory pool.  A pool
// whose release threshold is 0 (the CUDA default) hands freed memory back to
// the OS at every synchronisation, so a caller that synchronises between
// calls would pay a fresh mapping each time; the first allocation on a device
// therefore raises the threshold to 1 GiB if it is still 0 (process-local:
// the pool keeps at most that much freed memory for reuse).
cudaError_t scratch_alloc(void** p, size_t bytes, cudaStream_t st) {
  static std::mutex mu;
  static bool tuned[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64) {
    std::lock_guard<std::mutex> lock(mu);
    if (!tuned[dev]) {
      tuned[dev] = true;
      cudaMemPool_t pool;
      if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
        uint64_t thr = 0;
        if (cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr) == cudaSuccess && thr == 0) {
          thr = uint64_t(1) << 30;
          cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
        }
      }
      cudaGetLastError();
    }
  }
  return cudaMallocAsync(p, bytes, st);
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
  cudaFreeAsync(ws, st);
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
  cudaFreeAsync(ws, st);
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

template <typename T>
tg_status dispatch_semiring(tg_semiring s, const Problem& P, cudaStream_t st) {
  switch (s) {
    case TG_MAXPLUS: return dispatch_typed<tg::kMaxPlus, T>(P, st);
    case TG_MINPLUS: return dispatch_typed<tg::kMinPlus, T>(P, st);
    case TG_MAXMUL: return dispatch_typed<tg::kMaxMul, T>(P, st);
  }
  return fail(TG_ERR_INVALID_ARGUMENT, "unknown semiring %d", int(s));
}

size_t dtype_size(tg_dtype t) {
  switch (t) {
    case TG_F32: case TG_I32: return 4;
    case TG_F64: case TG_I64: return 8;
  }
  return 0;
}

tg_status gemm_impl(tg_semiring semiring, tg_dtype dtype, tg_layout layout, int64_t batch,
                    int64_t m, int64_t n, int64_t k, const void* a, int64_t lda, int64_t sa,
                    const void* b, int64_t ldb, int64_t sb, void* c, int64_t ldc, int64_t sc,
                    int32_t* argmax, void* stream) {
  g_last_error.clear();
  if (semiring < TG_MAXPLUS || semiring > TG_MAXMUL) return fail(TG_ERR_INVALID_ARGUMENT, "unknown semiring %d", int(semiring));
  if (dtype_size(dtype) == 0) return fail(TG_ERR_INVALID_ARGUMENT, "unknown dtype %d", int(dtype));
  if (layout != TG_ROW_MAJOR && layout != TG_COL_MAJOR) return fail(TG_ERR_INVALID_ARGUMENT, "unknown layout %d", int(layout));
  if (batch < 0 || m < 0 || n < 0 || k < 0) return fail(TG_ERR_INVALID_ARGUMENT, "negative size (batch=%lld m=%lld n=%lld k=%lld)", (long long)batch, (long long)m, (long long)n, (long long)k);
  if (batch == 0 || m == 0 || n == 0) return TG_OK;
  if (!c) return fail(TG_ERR_INVALID_ARGUMENT, "C is null");
  if (k > 0 && (!a || !b)) return fail(TG_ERR_INVALID_ARGUMENT, "A or B is null");
  if (k >= (int64_t(1) << 31)) return fail(TG_ERR_UNSUPPORTED, "K=%lld exceeds the int32 argmax range", (long long)k);
  // Leading-dimension checks in the caller's layout.
  const bool row = layout == TG_ROW_MAJOR;
  const int64_t need_lda = row ? k : m, need_ldb = row ? n : k, need_ldc = row ? n : m;
  if (k > 0 && lda < std::max<int64_t>(1, need_lda)) return fail(TG_ERR_DIMENSION_MISMATCH, "lda=%lld < %lld", (long long)lda, (long long)need_lda);
  if (k > 0 && ldb < std::max<int64_t>(1, need_ldb)) return fail(TG_ERR_DIMENSION_MISMATCH, "ldb=%lld < %lld", (long long)ldb, (long long)need_ldb);
  if (ldc < std::max<int64_t>(1, need_ldc)) return fail(TG_ERR_DIMENSION_MISMATCH, "ldc=%lld < %lld", (long long)ldc, (long long)need_ldc);
  if (batch > 1 && (sa < 0 || sb < 0 || sc < 0)) return fail(TG_ERR_INVALID_ARGUMENT, "negative batch stride");

  Problem P;
  P.batch = batch;
  if (row) {
    P.g = tg::GemmArgs{m, n, k, a, lda, sa, b, ldb, sb, c, ldc, sc, argmax};
  } else {  // C^T (N x M, row-major, ldc) = B^T (N x K, ldb) (x) A^T (K x M, lda)
    P.g = tg::GemmArgs{n, m, k, b, ldb, sb, a, lda, sa, c, ldc, sc, argmax};
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case TG_F32: return dispatch_semiring<float>(semiring, P, st);
    case TG_F64: return dispatch_semiring<double>(semiring, P, st);
    case TG_I32: return dispatch_semiring<int32_t>(semiring, P, st);
    case TG_I64: return dispatch_semiring<int64_t>(semiring, P, st);
  }
  return fail(TG_ERR_INVALID_ARGUMENT, "unknown dtype");
}

// ------------------------------------------------------------- backward
template <typename T>
tg_status hist_launch(bool rows_kind, const tg::HistArgs& h, int64_t batch, cudaStream_t st) {
  int dev = 0;
  cudaGetDevice(&dev);
  int max_optin = 0;
  cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const size_t bins = rows_kind ? size_t(h.k) * sizeof(T) : size_t(h.k) * 32 * sizeof(T);
  for (int64_t b0 = 0; b0 < batch; b0 += 65535) {
    const int64_t nb = std::min<int64_t>(65535, batch - b0);
    tg::HistArgs g = h;
    g.gc = static_cast<const T*>(h.gc) + b0 * h.sc;
    g.arg = h.arg + b0 * h.sc;
    if (h.w) g.w = static_cast<const T*>(h.w) + b0 * h.sw;
    g.out = static_cast<T*>(h.out) + b0 * h.so;
    const size_t wbins = size_t(h.k) * sizeof(T) * 8;   // one warp per row, 8 rows per CTA
    if (rows_kind && wbins <= size_t(max_optin) && (h.rows + 7) / 8 <= 0x7fffffff) {
      constexpr int64_t epv = 16 / sizeof(T);
      // 16-byte grad_C loads (and 4 * epv-byte argmax loads) on every row
      const bool vec = (reinterpret_cast<uintptr_t>(g.gc) & 15) == 0 &&
                       (reinterpret_cast<uintptr_t>(g.arg) & (4 * epv - 1)) == 0 && h.cols % epv == 0 &&
                       h.ldc % epv == 0 && (nb == 1 || h.sc % epv == 0);
      auto kern = vec ? tg::hist_rows_warp_kernel<T, true> : tg::hist_rows_warp_kernel<T, false>;
      if (wbins > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(wbins));
      kern<<<dim3(unsigned((h.rows + 7) / 8), unsigned(nb)), 256, wbins, st>>>(g);
    } else if (bins <= size_t(max_optin) && (rows_kind ? h.rows <= 0x7fffffff : (h.cols + 31) / 32 <= 0x7fffffff)) {
      if (rows_kind) {
        auto kern = tg::hist_rows_kernel<T>;
        if (bins > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bins));
        kern<<<dim3(unsigned(h.rows), unsigned(nb)), 256, bins, st>>>(g);
      } else {
        auto kern = tg::hist_cols_kernel<T>;
        if (bins > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bins));
        kern<<<dim3(unsigned((h.cols + 31) / 32), unsigned(nb)), 256, bins, st>>>(g);
      }
    } else {
      const int64_t out_rows = rows_kind ? h.rows : h.k, out_cols = rows_kind ? h.k : h.cols;
      if (!h.accumulate)
        tg::zero_matrix_kernel<T><<<dim3(1024, unsigned(nb)), 256, 0, st>>>(static_cast<T*>(g.out), out_rows, out_cols, h.ldo, h.so);
      if (rows_kind) tg::hist_atomic_kernel<T, true><<<dim3(2048, unsigned(nb)), 256, 0, st>>>(g);
      else tg::hist_atomic_kernel<T, false><<<dim3(2048, unsigned(nb)), 256, 0, st>>>(g);
    }
    tg_status s = check_launch("backward launch");
    if (s != TG_OK) return s;
  }
  return TG_OK;
}

tg_status backward_impl(bool want_a, tg_semiring semiring, tg_dtype dtype, tg_layout layout,
                        int64_t batch, int64_t m, int64_t n, int64_t k,
                        const void* grad_c, int64_t ldc, int64_t sc, const int32_t* argmax,
                        const void* w, int64_t ldw, int64_t sw,
                        void* grad, int64_t ldg, int64_t sg, int accumulate, void* stream) {
  g_last_error.clear();
  if (semiring < TG_MAXPLUS || semiring > TG_MAXMUL) return fail(TG_ERR_INVALID_ARGUMENT, "unknown semiring %d", int(semiring));
  if (dtype != TG_F32 && dtype != TG_F64) return fail(TG_ERR_UNSUPPORTED, "backward is defined for f32/f64 only");
  if (layout != TG_ROW_MAJOR && layout != TG_COL_MAJOR) return fail(TG_ERR_INVALID_ARGUMENT, "unknown layout %d", int(layout));
  if (batch < 0 || m < 0 || n < 0 || k < 0) return fail(TG_ERR_INVALID_ARGUMENT, "negative size");
  if (batch == 0 || k == 0) return TG_OK;
  const bool row = layout == TG_ROW_MAJOR;
  // Output dims in caller layout: grad_A is M x K, grad_B is K x N.
  const int64_t g_rows = want_a ? m : k, g_cols = want_a ? k : n;
  if (g_rows == 0 || g_cols == 0) return TG_OK;
  if (!grad) return fail(TG_ERR_INVALID_ARGUMENT, "gradient output is null");
  const bool empty_c = (m == 0 || n == 0);
  if (!empty_c && (!grad_c || !argmax)) return fail(TG_ERR_INVALID_ARGUMENT, "grad_c or argmax is null");
  if (semiring == TG_MAXMUL && !empty_c && !w) return fail(TG_ERR_INVALID_ARGUMENT, "MaxMul backward needs the partner matrix (%s)", want_a ? "B" : "A");
  const int64_t need_ldc = row ? n : m;
  const int64_t need_ldg = row ? g_cols : g_rows;
  if (!empty_c && ldc < std::max<int64_t>(1, need_ldc)) return fail(TG_ERR_DIMENSION_MISMATCH, "ldc=%lld < %lld", (long long)ldc, (long long)need_ldc);
  if (ldg < std::max<int64_t>(1, need_ldg)) return fail(TG_ERR_DIMENSION_MISMATCH, "gradient ld=%lld < %lld", (long long)ldg, (long long)need_ldg);
  if (semiring == TG_MAXMUL && !empty_c) {
    // partner: B (K x N) for grad_A, A (M x K) for grad_B, in caller layout
    const int64_t need_ldw = want_a ? (row ? n : k) : (row ? k : m);
    if (ldw < std::max<int64_t>(1, need_ldw)) return fail(TG_ERR_DIMENSION_MISMATCH, "partner ld=%lld < %lld", (long long)ldw, (long long)need_ldw);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  tg::HistArgs h;
  // Canonical (row-major) view: row-major grad_A = row histogram, grad_B =
  // column histogram; column-major swaps the two roles (C^T = B^T (x) A^T).
  const bool rows_kind = (want_a == row);
  h.rows = row ? m : n;
  h.cols = row ? n : m;
  h.k = k;
  h.gc = grad_c; h.ldc = ldc; h.sc = sc; h.arg = argmax;
  h.w = semiring == TG_MAXMUL ? w : nullptr; h.ldw = ldw; h.sw = sw;
  h.out = grad; h.ldo = ldg; h.so = sg;
  h.accumulate = accumulate;
  if (empty_c) {  // nothing scatters; overwrite means zero
    if (accumulate) return TG_OK;
    const int64_t orow = rows_kind ? h.rows : k, ocol = rows_kind ? k : h.cols;
    (void)orow; (void)ocol;
    if (dtype == TG_F32) tg::zero_matrix_kernel<float><<<dim3(256, unsigned(std::min<int64_t>(batch, 65535))), 256, 0, st>>>(static_cast<float*>(grad), rows_kind ? h.rows : k, rows_kind ? k : h.cols, ldg, sg);
    else tg::zero_matrix_kernel<double><<<dim3(256, unsigned(std::min<int64_t>(batch, 65535))), 256, 0, st>>>(static_cast<double*>(grad), rows_kind ? h.rows : k, rows_kind ? k : h.cols, ldg, sg);
    return check_launch("zero_matrix_kernel launch");
  }
  return dtype == TG_F32 ? hist_launch<float>(rows_kind, h, batch, st) : hist_launch<double>(rows_kind, h, batch, st);
}

}  // namespace

extern "C" {

const char* tg_version(void) { return "0.2.0-b200"; }
const char* tg_last_error(void) { return g_last_error.c_str(); }

int tg_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) { cudaGetLastError(); return 0; }
  return n;
}

tg_status tg_gemm(tg_semiring semiring, tg_dtype dtype, tg_layout layout, int64_t m, int64_t n, int64_t k,
                  const void* a, int64_t lda, const void* b, int64_t ldb, void* c, int64_t ldc,
                  int32_t* argmax, void* stream) {
  return gemm_impl(semiring, dtype, layout, 1, m, n, k, a, lda, 0, b, ldb, 0, c, ldc, 0, argmax, stream);
}

tg_status tg_gemm_strided_batched(tg_semiring semiring, tg_dtype dtype, tg_layout layout, int64_t batch,
                                  int64_t m, int64_t n, int64_t k, const void* a, int64_t lda, int64_t stride_a,
                                  const void* b, int64_t ldb, int64_t stride_b, void* c, int64_t ldc,
                                  int64_t stride_c, int32_t* argmax, void* stream) {
  return gemm_impl(semiring, dtype, layout, batch, m, n, k, a, lda, stride_a, b, ldb, stride_b, c, ldc, stride_c,
                   argmax, stream);
}

tg_status tg_backward_a(tg_semiring semiring, tg_dtype dtype, tg_layout layout, int64_t batch, int64_t m, int64_t n,
                        int64_t k, const void* grad_c, int64_t ldc, int64_t stride_c, const int32_t* argmax,
                        const void* b, int64_t ldb, int64_t stride_b, void* grad_a, int64_t lda, int64_t stride_a,
                        int accumulate, void* stream) {
  return backward_impl(true, semiring, dtype, layout, batch, m, n, k, grad_c, ldc, stride_c, argmax, b, ldb, stride_b,
                       grad_a, lda, stride_a, accumulate, stream);
}

tg_status tg_backward_b(tg_semiring semiring, tg_dtype dtype, tg_layout layout, int64_t batch, int64_t m, int64_t n,
                        int64_t k, const void* grad_c, int64_t ldc, int64_t stride_c, const int32_t* argmax,
                        const void* a, int64_t lda, int64_t stride_a, void* grad_b, int64_t ldb, int64_t stride_b,
                        int accumulate, void* stream) {
  return backward_impl(false, semiring, dtype, layout, batch, m, n, k, grad_c, ldc, stride_c, argmax, a, lda, stride_a,
                       grad_b, ldb, stride_b, accumulate, stream);
}

tg_status tg_sharded_gemm(tg_semiring semiring, tg_dtype dtype, int64_t m_local, int64_t n, int64_t k,
                          const void* a_local, int64_t lda, void* b, int64_t ldb, void* c_local, int64_t ldc,
                          int32_t* argmax_local, int root, tg_broadcast_fn bcast, void* bcast_ctx, void* stream) {
  g_last_error.clear();
  if (semiring < TG_MAXPLUS || semiring > TG_MAXMUL) return fail(TG_ERR_INVALID_ARGUMENT, "unknown semiring %d", int(semiring));
  if (dtype < TG_F32 || dtype > TG_I64) return fail(TG_ERR_INVALID_ARGUMENT, "unknown dtype %d", int(dtype));
  if (m_local < 0 || n < 0 || k < 0)
    return fail(TG_ERR_INVALID_ARGUMENT, "negative size (m_local=%lld n=%lld k=%lld)", (long long)m_local, (long long)n,
                (long long)k);
  if (!bcast) return fail(TG_ERR_INVALID_ARGUMENT, "broadcast callback is null");
  if (root < 0) return fail(TG_ERR_INVALID_ARGUMENT, "negative root rank %d", root);
  // B must reach every rank even when this rank owns no rows
  if (k > 0 && n > 0) {
    if (!b) return fail(TG_ERR_INVALID_ARGUMENT, "B is null");
    if (ldb < n) return fail(TG_ERR_DIMENSION_MISMATCH, "ldb=%lld < n=%lld", (long long)ldb, (long long)n);
    const size_t elem = (dtype == TG_F64 || dtype == TG_I64) ? 8 : 4;
    const size_t bytes = (size_t(k - 1) * size_t(ldb) + size_t(n)) * elem;
    const int rc = bcast(b, bytes, root, stream, bcast_ctx);
    if (rc != 0) return fail(TG_ERR_CUDA, "broadcast callback failed (code %d)", rc);
  }
  return tg_gemm(semiring, dtype, TG_ROW_MAJOR, m_local, n, k, a_local, lda, b, ldb, c_local, ldc, argmax_local,
                 stream);
}

}  // extern "C"

#ifdef TG_PHASE_TIMING
extern "C" int tg_debug_phase_ts(long long* host, int n) {
  return (int)cudaMemcpyFromSymbol(host, tg::tg_phase_ts, sizeof(long long) * n);
}
#endif

// --------------------------------------------------------------------------
// Allocation-free variant of the i32 GEMM.
//
// Some callers cannot allocate device memory at call time: a host framework
// that has already reserved the GPU's memory for its own pool, or a serving
// or real-time loop that forbids cudaMalloc/cudaMallocAsync after start-up
// (an allocation can block, fail under memory pressure, or synchronise).
// tg_gemm_i32_noalloc gives them the i32 GEMM without any allocation: its
// scratch (the f32 copies of A and B plus the range flag) lives in the
// fixed array below, which every GPU that loads this library keeps for the
// life of the process.
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;   // 64 MiB per device
static __device__ __align__(256) unsigned char tg_noalloc_scratch[kNoAllocScratchBytes];

// Device address of tg_noalloc_scratch, looked up once per device (the
// symbol's host-side name is not a device address).
void* noalloc_scratch_address(int dev, tg_status* st) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  if (dev < 0 || dev >= 64) { *st = fail(TG_ERR_UNSUPPORTED, "device ordinal %d out of range", dev); return nullptr; }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, tg_noalloc_scratch);
    if (e != cudaSuccess) {
      *st = fail(TG_ERR_CUDA, "cudaGetSymbolAddress(tg_noalloc_scratch): %s", cudaGetErrorString(e));
      return nullptr;
    }
    addr[dev] = p;
  }
  *st = TG_OK;
  return addr[dev];
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

}  // namespace

extern "C" tg_status tg_gemm_i32_noalloc(tg_semiring semiring, tg_layout layout, int64_t m, int64_t n, int64_t k,
                                         const void* a, int64_t lda, const void* b, int64_t ldb, void* c,
                                         int64_t ldc, int32_t* argmax, void* stream) {
  g_last_error.clear();
  if (semiring < TG_MAXPLUS || semiring > TG_MAXMUL) return fail(TG_ERR_INVALID_ARGUMENT, "unknown semiring %d", int(semiring));
  if (layout != TG_ROW_MAJOR && layout != TG_COL_MAJOR) return fail(TG_ERR_INVALID_ARGUMENT, "unknown layout %d", int(layout));
  if (m < 0 || n < 0 || k < 0) return fail(TG_ERR_INVALID_ARGUMENT, "negative size (m=%lld n=%lld k=%lld)", (long long)m, (long long)n, (long long)k);
  if (m == 0 || n == 0) return TG_OK;
  if (!c) return fail(TG_ERR_INVALID_ARGUMENT, "C is null");
  if (k > 0 && (!a || !b)) return fail(TG_ERR_INVALID_ARGUMENT, "A or B is null");
  const bool row = layout == TG_ROW_MAJOR;
  const int64_t need_lda = row ? k : m, need_ldb = row ? n : k, need_ldc = row ? n : m;
  if (k > 0 && lda < std::max<int64_t>(1, need_lda)) return fail(TG_ERR_DIMENSION_MISMATCH, "lda=%lld < %lld", (long long)lda, (long long)need_lda);
  if (k > 0 && ldb < std::max<int64_t>(1, need_ldb)) return fail(TG_ERR_DIMENSION_MISMATCH, "ldb=%lld < %lld", (long long)ldb, (long long)need_ldb);
  if (ldc < std::max<int64_t>(1, need_ldc)) return fail(TG_ERR_DIMENSION_MISMATCH, "ldc=%lld < %lld", (long long)ldc, (long long)need_ldc);
  Problem P;
  P.batch = 1;
  P.g = row ? tg::GemmArgs{m, n, k, a, lda, 0, b, ldb, 0, c, ldc, 0, argmax}
            : tg::GemmArgs{n, m, k, b, ldb, 0, a, lda, 0, c, ldc, 0, argmax};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (k == 0 || !fast_f32_ok(P)) {   // no scratch needed: semiring zero and index 0, or the exact kernel
    switch (semiring) {
      case TG_MAXPLUS: return dispatch_typed<tg::kMaxPlus, int32_t>(P, st);
      case TG_MINPLUS: return dispatch_typed<tg::kMinPlus, int32_t>(P, st);
      default: return dispatch_typed<tg::kMaxMul, int32_t>(P, st);
    }
  }
  const int64_t lda_f = (P.g.k + 3) & ~int64_t(3), ldb_f = (P.g.n + 3) & ~int64_t(3);
  const double need = 256.0 + 4.0 * (double(P.g.m) * double(lda_f) + double(P.g.k) * double(ldb_f));
  if (need > double(kNoAllocScratchBytes))
    return fail(TG_ERR_UNSUPPORTED,
                "tg_gemm_i32_noalloc: A and B need %.0f bytes of scratch as f32 (rows padded to 4 elements), "
                "more than the fixed %zu-byte scratch; use tg_gemm instead",
                need, kNoAllocScratchBytes);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(TG_ERR_NO_DEVICE, "no current CUDA device");
  tg_status s;
  unsigned char* ws = static_cast<unsigned char*>(noalloc_scratch_address(dev, &s));
  if (!ws) return s;
  switch (semiring) {
    case TG_MAXPLUS: return noalloc_i32<tg::kMaxPlus>(P, st, ws);
    case TG_MINPLUS: return noalloc_i32<tg::kMinPlus>(P, st, ws);
    default: return noalloc_i32<tg::kMaxMul>(P, st, ws);
  }
}
