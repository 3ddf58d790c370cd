// Argmax-scatter backward pass (gradients of C = A (x) B through argmax).
//
// Reference: CUDA kernels TROPICAL_BACKWARD_A/B (one thread per C element,
// global atomicAdd: crates/tropical-gemm-cuda/kernels/tropical_gemm.cu:1002-1036)
// and the torch path (zeros + scatter_add_:
// crates/tropical-gemm-python/python/tropical_gemm/pytorch.py:386-403,
// multiplicative MaxMul rule :521-548).
//
// B200 design: both gradients are histograms of grad_C keyed by argmax.
//  * grad_A (row histogram): one warp per C row accumulates K bins in shared
//    memory (16-byte loads of grad_C and argmax) and writes the whole grad_A
//    row once, coalesced -- no global atomics and no separate zero-fill
//    pass.  K too large for 8 warps' bins: one CTA per row shares them.
//  * grad_B (column histogram): one CTA per 32-column strip walks every
//    row of the strip with coalesced loads, accumulates K x 32 bins in
//    shared memory, then writes its grad_B strip once.
//  * When K is too large for the shared-memory bins the scatter falls back
//    to global atomics (red.global.add) on a zero-filled output.
// Indices outside [0, K) are skipped like the reference kernels do.
// Summation order inside a bin is not fixed (shared-memory atomics), so
// float results agree with an ordered sum to rounding, as the reference's
// atomicAdd ones do.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace tg {

struct HistArgs {
  int64_t rows, cols, k;           // C' is rows x cols (canonical row-major)
  const void* gc; int64_t ldc, sc; // grad_C
  const int32_t* arg;              // same ld/stride as grad_C
  const void* w;  int64_t ldw, sw; // MaxMul partner matrix or nullptr
  void* out;      int64_t ldo, so; // gradient output
  int accumulate;
};

// grad_out[r, k] (+)= sum_c [arg[r,c] == k] * gc[r,c] * (w ? w[k*ldw + c] : 1)
template <typename T>
__global__ void __launch_bounds__(256) hist_rows_kernel(HistArgs p) {
  extern __shared__ __align__(16) unsigned char hsm[];
  T* bins = reinterpret_cast<T*>(hsm);
  const int64_t r = blockIdx.x, batch = blockIdx.y;
  const T* gc = static_cast<const T*>(p.gc) + batch * p.sc + r * p.ldc;
  const int32_t* arg = p.arg + batch * p.sc + r * p.ldc;
  const T* w = p.w ? static_cast<const T*>(p.w) + batch * p.sw : nullptr;
  T* out = static_cast<T*>(p.out) + batch * p.so + r * p.ldo;
  for (int64_t i = threadIdx.x; i < p.k; i += blockDim.x) bins[i] = T(0);
  __syncthreads();
  for (int64_t c = threadIdx.x; c < p.cols; c += blockDim.x) {
    const int32_t kk = arg[c];
    if (kk < 0 || kk >= p.k) continue;
    T g = gc[c];
    if (w) g = g * w[int64_t(kk) * p.ldw + c];
    atomicAdd(&bins[kk], g);
  }
  __syncthreads();
  for (int64_t i = threadIdx.x; i < p.k; i += blockDim.x)
    out[i] = p.accumulate ? out[i] + bins[i] : bins[i];
}

// Same histogram with one warp per C row: 8 rows per CTA, K bins per warp
// (no CTA barrier), and VEC = 16-byte loads of grad_C and argmax (EPV
// elements per lane per step) when every row is 16-byte aligned.
template <typename T, bool VEC>
__global__ void __launch_bounds__(256) hist_rows_warp_kernel(HistArgs p) {
  extern __shared__ __align__(16) unsigned char hsm[];
  constexpr int EPV = 16 / sizeof(T);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = int64_t(blockIdx.x) * 8 + warp, batch = blockIdx.y;
  if (r >= p.rows) return;   // warp-level work only below
  T* bins = reinterpret_cast<T*>(hsm) + int64_t(warp) * p.k;
  const T* gc = static_cast<const T*>(p.gc) + batch * p.sc + r * p.ldc;
  const int32_t* arg = p.arg + batch * p.sc + r * p.ldc;
  const T* w = p.w ? static_cast<const T*>(p.w) + batch * p.sw : nullptr;
  T* out = static_cast<T*>(p.out) + batch * p.so + r * p.ldo;
  for (int64_t i = lane; i < p.k; i += 32) bins[i] = T(0);
  __syncwarp();
  auto add = [&](int32_t kk, T g, int64_t c) {
    if (kk < 0 || kk >= p.k) return;
    if (w) g = g * w[int64_t(kk) * p.ldw + c];
    atomicAdd(&bins[kk], g);
  };
  if constexpr (VEC) {
    for (int64_t c = int64_t(lane) * EPV; c < p.cols; c += 32 * EPV) {
      if constexpr (EPV == 4) {
        const int4 a4 = *reinterpret_cast<const int4*>(arg + c);
        const float4 g4 = *reinterpret_cast<const float4*>(gc + c);
        add(a4.x, g4.x, c); add(a4.y, g4.y, c + 1); add(a4.z, g4.z, c + 2); add(a4.w, g4.w, c + 3);
      } else {
        const int2 a2 = *reinterpret_cast<const int2*>(arg + c);
        const double2 g2 = *reinterpret_cast<const double2*>(gc + c);
        add(a2.x, g2.x, c); add(a2.y, g2.y, c + 1);
      }
    }
  } else {
    for (int64_t c = lane; c < p.cols; c += 32) add(arg[c], gc[c], c);
  }
  __syncwarp();
  for (int64_t i = lane; i < p.k; i += 32) out[i] = p.accumulate ? out[i] + bins[i] : bins[i];
}

// grad_out[k, c] (+)= sum_r [arg[r,c] == k] * gc[r,c] * (w ? w[r*ldw + k] : 1)
// One CTA per 32-column strip; 256 threads = 8 row lanes x 32 columns, eight
// rows per lane in flight.
template <typename T>
__global__ void __launch_bounds__(256) hist_cols_kernel(HistArgs p) {
  extern __shared__ __align__(16) unsigned char hsm[];
  T* bins = reinterpret_cast<T*>(hsm);           // [k][32]
  const int64_t c0 = int64_t(blockIdx.x) * 32, batch = blockIdx.y;
  const int lane = threadIdx.x & 31, rl = threadIdx.x >> 5;
  const T* gc = static_cast<const T*>(p.gc) + batch * p.sc;
  const int32_t* arg = p.arg + batch * p.sc;
  const T* w = p.w ? static_cast<const T*>(p.w) + batch * p.sw : nullptr;
  T* out = static_cast<T*>(p.out) + batch * p.so;
  for (int64_t i = threadIdx.x; i < p.k * 32; i += blockDim.x) bins[i] = T(0);
  __syncthreads();
  const int64_t c = c0 + lane;
  if (c < p.cols) {
    int64_t r = rl;
    for (; r + 56 < p.rows; r += 64) {
      int32_t kk[8];
      T g[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        kk[u] = arg[(r + 8 * u) * p.ldc + c];
        g[u] = gc[(r + 8 * u) * p.ldc + c];
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (kk[u] < 0 || kk[u] >= p.k) continue;
        T v = g[u];
        if (w) v = v * w[(r + 8 * u) * p.ldw + kk[u]];
        atomicAdd(&bins[int64_t(kk[u]) * 32 + lane], v);
      }
    }
    for (; r < p.rows; r += 8) {
      const int32_t kk = arg[r * p.ldc + c];
      if (kk < 0 || kk >= p.k) continue;
      T g = gc[r * p.ldc + c];
      if (w) g = g * w[r * p.ldw + kk];
      atomicAdd(&bins[int64_t(kk) * 32 + lane], g);
    }
  }
  __syncthreads();
  for (int64_t i = threadIdx.x; i < p.k * 32; i += blockDim.x) {
    const int64_t kk = i >> 5, cc = c0 + (i & 31);
    if (cc >= p.cols) continue;
    T* o = out + kk * p.ldo + cc;
    *o = p.accumulate ? *o + bins[i] : bins[i];
  }
}

// Large-K fallback: one thread per C element, global atomics.
// ROWS=true scatters into grad_out[r, k] (row histogram), else grad_out[k, c].
template <typename T, bool ROWS>
__global__ void __launch_bounds__(256) hist_atomic_kernel(HistArgs p) {
  const int64_t total = p.rows * p.cols;
  const int64_t batch = blockIdx.y;
  const T* gc = static_cast<const T*>(p.gc) + batch * p.sc;
  const int32_t* arg = p.arg + batch * p.sc;
  const T* w = p.w ? static_cast<const T*>(p.w) + batch * p.sw : nullptr;
  T* out = static_cast<T*>(p.out) + batch * p.so;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = e / p.cols, c = e % p.cols;
    const int32_t kk = arg[r * p.ldc + c];
    if (kk < 0 || kk >= p.k) continue;
    T g = gc[r * p.ldc + c];
    if (ROWS) {
      if (w) g = g * w[int64_t(kk) * p.ldw + c];
      atomicAdd(out + r * p.ldo + kk, g);
    } else {
      if (w) g = g * w[r * p.ldw + kk];
      atomicAdd(out + int64_t(kk) * p.ldo + c, g);
    }
  }
}

// Zero a (rows x cols, ld) strided-batched matrix.
template <typename T>
__global__ void zero_matrix_kernel(T* out, int64_t rows, int64_t cols, int64_t ld, int64_t stride) {
  T* o = out + int64_t(blockIdx.y) * stride;
  const int64_t total = rows * cols;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += int64_t(gridDim.x) * blockDim.x)
    o[(e / cols) * ld + e % cols] = T(0);
}

}  // namespace tg
