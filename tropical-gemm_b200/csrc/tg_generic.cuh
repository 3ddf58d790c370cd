// Generic tropical GEMM kernel: every (semiring, dtype, argmax) combination,
// arbitrary leading dimensions and strides, strided batch on grid.z.
//
// This is the exact-semantics workhorse used for f64, i64, integer inputs
// outside the fast path's range, and shapes the f32 fast kernel does not
// take.  It restates the reference kernels' arithmetic per product
// (crates/tropical-gemm-cuda/kernels/tropical_gemm.cu:526-639 for argmax,
// :86-189 for values only): k ascending, strict compare, first k wins ties.
//
// Canonical form: row-major A[M,K] (k contiguous), B[K,N] (n contiguous),
// C[M,N].  Column-major callers are mapped onto it by the host as
// C^T = B^T (x) A^T, which leaves every (output, k) product unchanged.
#pragma once
#include "tg_semiring.cuh"

namespace tg {

struct GemmArgs {
  int64_t m, n, k;
  const void* a; int64_t lda, sa;   // sa/sb/sc: batch strides in elements
  const void* b; int64_t ldb, sb;
  void* c;       int64_t ldc, sc;
  int32_t* argmax;
  // Optional device-side gate: when set, the kernel runs only if
  // (*gate != 0) == (gate_run_if_set != 0).  Lets the host enqueue both a
  // fast and an exact kernel behind a device-computed precondition without
  // a host synchronisation.
  const int* gate = nullptr;
  int gate_run_if_set = 0;
  // Accumulate (f32 fast kernels only): every output starts from its current
  // C value (and keeps its argmax unless a product strictly beats it); a
  // winning k is reported as k_offset + k.  Lets a K-sliced problem be
  // computed slice by slice with results identical to one pass.
  int accumulate = 0;
  int32_t k_offset = 0;
};

__device__ __forceinline__ bool gated_off(const GemmArgs& p) {
  return p.gate && ((*p.gate != 0) != (p.gate_run_if_set != 0));
}

constexpr int kGenBM = 64, kGenBN = 64, kGenBK = 16, kGenThreads = 256;

template <int S, typename T, bool ARGMAX>
__global__ void __launch_bounds__(kGenThreads)
generic_gemm_kernel(GemmArgs p) {
  using R = Ring<S, T>;
  if (gated_off(p)) return;
  __shared__ T As[kGenBK][kGenBM];
  __shared__ T Bs[kGenBK][kGenBN];

  const int64_t batch = blockIdx.z;
  const T* __restrict__ A = static_cast<const T*>(p.a) + batch * p.sa;
  const T* __restrict__ B = static_cast<const T*>(p.b) + batch * p.sb;
  T* __restrict__ C = static_cast<T*>(p.c) + batch * p.sc;
  int32_t* __restrict__ IDX = ARGMAX ? p.argmax + batch * p.sc : nullptr;

  const int64_t m0 = int64_t(blockIdx.x) * kGenBM;
  const int64_t n0 = int64_t(blockIdx.y) * kGenBN;
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;  // tx -> columns, ty -> rows

  T acc[4][4];
  int32_t idx[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) { acc[i][j] = R::zero(); idx[i][j] = 0; }

  for (int64_t k0 = 0; k0 < p.k; k0 += kGenBK) {
    // Stage A: 64 rows x 16 k, B: 16 k x 64 cols; 1024 elements each.
#pragma unroll
    for (int e = 0; e < (kGenBM * kGenBK) / kGenThreads; ++e) {
      int lin = tid + e * kGenThreads;
      int r = lin / kGenBK, kk = lin % kGenBK;
      int64_t gr = m0 + r, gk = k0 + kk;
      As[kk][r] = (gr < p.m && gk < p.k) ? A[gr * p.lda + gk] : T(0);
      int kb = lin / kGenBN, cc = lin % kGenBN;
      int64_t gkb = k0 + kb, gc = n0 + cc;
      Bs[kb][cc] = (gkb < p.k && gc < p.n) ? B[gkb * p.ldb + gc] : T(0);
    }
    __syncthreads();
    const int kcount = int((p.k - k0) < kGenBK ? (p.k - k0) : kGenBK);
#pragma unroll 4
    for (int kk = 0; kk < kcount; ++kk) {
      T av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx + 16 * j];
      const int32_t gk = int32_t(k0 + kk);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          T prod = R::mul(av[i], bv[j]);
          if (ARGMAX) {
            if (R::better(prod, acc[i][j])) { acc[i][j] = prod; idx[i][j] = gk; }
          } else {
            acc[i][j] = R::reduce(acc[i][j], prod);
          }
        }
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int64_t gr = m0 + ty + 16 * i;
    if (gr >= p.m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int64_t gc = n0 + tx + 16 * j;
      if (gc >= p.n) continue;
      C[gr * p.ldc + gc] = acc[i][j];
      if (ARGMAX) IDX[gr * p.ldc + gc] = idx[i][j];
    }
  }
}

}  // namespace tg
