// f64 tropical GEMM kernel (also the compute kernel of the i64 path).
//
// FP64 has no paired add and no 3-input max, so this kernel keeps one
// compare per product.  Argmax: add/mul then the strict compare that moves
// value and index (crates/tropical-gemm-cuda/kernels/tropical_gemm.cu:645-758).
// Value-only: the same strict select instead of the reference's fmax/fmin
// (:191-299), which costs about twice as much on sm_100; the results are equal
// (see the zero-sign re-run below).  It wins on tiling too: 128x64x16 CTA tiles, 256 threads, 8x4 outputs per thread
// (the reference uses 32x32 tiles and 4x4 per thread), a 3-stage cp.async
// pipeline, and 16-byte shared-memory fragment loads.  Semantics are the
// reference's bit for bit (same operations in the same k order per output).
#pragma once
#include <type_traits>
#include "tg_semiring.cuh"
#include "tg_generic.cuh"
#include "tg_fast_f32.cuh"   // cp.async helpers

namespace tg {

constexpr int kWBM = 128, kWBN = 64, kWBK = 16, kWThreads = 256, kWStages = 3;
constexpr int kWTN = kWBN / 16;      // outputs per thread along n (8 along m)
constexpr int kWApitch = kWBM + 2;   // As[k][m] (doubles), padded
constexpr int kWBpitch = kWBN + 2;   // Bs[k][n] (doubles), padded; keeps 16-byte alignment
constexpr int kWStage = kWBK * kWApitch + kWBK * kWBpitch;   // doubles
constexpr size_t kWSmem = size_t(kWStages) * kWStage * 8;
static_assert((kWApitch * 8) % 16 == 0 && (kWBK * kWApitch * 8) % 16 == 0, "alignment");

__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src, int bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" :: "r"(dst), "l"(src), "r"(bytes));
}

template <typename CT>
__device__ __forceinline__ void store_w(CT* C, int64_t o, double v) {
  if constexpr (std::is_same<CT, double>::value) C[o] = v; else C[o] = CT(v);
}

// Value-only accumulation with the exact result of CUDA's fmax/fmin fold
// (NaN products ignored, max(+0,-0) = +0, min(+0,-0) = -0) as one
// predicated select: on equal values the max takes the product when its
// sign bit is clear (the min when it is set), which only changes anything
// for a +-0 pair; equal non-zeros have identical encodings.
template <int S>
__device__ __forceinline__ double wide_reduce(double acc, double p) {
  const int ph = __double2hiint(p);
  const bool take = (S == kMinPlus) ? (p < acc || (p == acc && ph < 0)) : (p > acc || (p == acc && ph >= 0));
  return take ? p : acc;
}

// OUTI: C is int64 (the i64 path computes exactly in f64 on converted
// operands).  acc_init: accumulator start (semiring zero, or the i64 sentinel).
template <int S, bool ARGMAX, bool OUTI = false>
__global__ void __launch_bounds__(kWThreads, 1)
wide_f64_kernel(GemmArgs p, double acc_init) {
  using R = Ring<S, double>;
  using CT = typename std::conditional<OUTI, int64_t, double>::type;
  if (gated_off(p)) return;
  extern __shared__ __align__(16) double wsm[];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t batch = blockIdx.z;
  const double* __restrict__ A = static_cast<const double*>(p.a) + batch * p.sa;
  const double* __restrict__ B = static_cast<const double*>(p.b) + batch * p.sb;
  CT* __restrict__ C = static_cast<CT*>(p.c) + batch * p.sc;
  int32_t* __restrict__ IDX = ARGMAX ? p.argmax + batch * p.sc : nullptr;
  const int64_t m0 = int64_t(blockIdx.x) * kWBM, n0 = int64_t(blockIdx.y) * kWBN;
  const int64_t ktiles = (p.k + kWBK - 1) / kWBK;
  const bool bvec = ((reinterpret_cast<uintptr_t>(B) & 15) == 0) && (p.ldb % 2 == 0);

  // staging: A element (row r, k) -> As[k][r] by 8-byte copies;
  // B row k, 2 doubles at n -> Bs[k][n] by 16-byte copies
  auto load = [&](int stage, int64_t kt) {
    double* As = wsm + stage * kWStage;
    double* Bs = As + kWBK * kWApitch;
    const int64_t k0 = kt * kWBK;
#pragma unroll
    for (int e = 0; e < (kWBM * kWBK) / kWThreads; ++e) {
      const int lin = tid + e * kWThreads;
      const int kk = lin & (kWBK - 1), r = lin >> 4;
      const int64_t gr = m0 + r, gk = k0 + kk;
      const bool ok = gr < p.m && gk < p.k;
      cp_async8(smem_u32(As + kk * kWApitch + r), ok ? A + gr * p.lda + gk : A, ok ? 8 : 0);
    }
#pragma unroll
    for (int e = 0; e < (kWBK * kWBN / 2) / kWThreads; ++e) {
      const int lin = tid + e * kWThreads;
      const int kk = lin / (kWBN / 2), c2 = (lin % (kWBN / 2)) * 2;
      const int64_t gk = k0 + kk, gc = n0 + c2;
      if (bvec) {
        int bytes = 0;
        const double* src = B;
        if (gk < p.k && gc < p.n) { bytes = (p.n - gc) >= 2 ? 16 : 8; src = B + gk * p.ldb + gc; }
        cp_async16(smem_u32(Bs + kk * kWBpitch + c2), src, bytes);
      } else {
        const bool ok0 = gk < p.k && gc < p.n, ok1 = gk < p.k && gc + 1 < p.n;
        cp_async8(smem_u32(Bs + kk * kWBpitch + c2), ok0 ? B + gk * p.ldb + gc : B, ok0 ? 8 : 0);
        cp_async8(smem_u32(Bs + kk * kWBpitch + c2 + 1), ok1 ? B + gk * p.ldb + gc + 1 : B, ok1 ? 8 : 0);
      }
    }
  };

  double acc[8][kWTN];
  int32_t idx[ARGMAX ? 8 : 1][ARGMAX ? kWTN : 1];

  // RED: 0 = strict-compare select (argmax, or a value-only fold whose
  // result equals the fmax/fmin fold), 1 = the sign-exact select of wide_reduce
  auto mainloop = [&](auto red_tag) {
    constexpr int RED = decltype(red_tag)::value;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < kWTN; ++j) {
        acc[i][j] = acc_init;
        if (ARGMAX) idx[i][j] = 0;
      }
#pragma unroll
    for (int s = 0; s < kWStages - 1; ++s) {
      if (s < ktiles) load(s, s);
      cp_async_commit();
    }
    for (int64_t t = 0; t < ktiles; ++t) {
      cp_async_wait<kWStages - 2>();
      __syncthreads();
      {
        const int64_t nt = t + kWStages - 1;
        if (nt < ktiles) load(int(nt % kWStages), nt);
        cp_async_commit();
      }
      const double* As = wsm + (t % kWStages) * kWStage;
      const double* Bs = As + kWBK * kWApitch;
      const int kcount = int((p.k - t * kWBK) < kWBK ? (p.k - t * kWBK) : kWBK);
      const int32_t kbase = int32_t(t * kWBK);
      auto step = [&](int kk) {
        double av[8], bv[kWTN];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const double2 a2 = *reinterpret_cast<const double2*>(As + kk * kWApitch + 2 * ty + 32 * q);
          av[2 * q] = a2.x; av[2 * q + 1] = a2.y;
        }
#pragma unroll
        for (int q = 0; q < kWTN / 2; ++q) {
          const double2 b2 = *reinterpret_cast<const double2*>(Bs + kk * kWBpitch + 2 * tx + 32 * q);
          bv[2 * q] = b2.x; bv[2 * q + 1] = b2.y;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < kWTN; ++j) {
            const double prod = R::mul(av[i], bv[j]);
            if (ARGMAX) {
              if (R::better(prod, acc[i][j])) { acc[i][j] = prod; idx[i][j] = kbase + kk; }
            } else if (RED == 0) {
              if (R::better(prod, acc[i][j])) acc[i][j] = prod;
            } else {
              acc[i][j] = wide_reduce<S>(acc[i][j], prod);
            }
          }
      };
      if (kcount == kWBK) {
#pragma unroll
        for (int kk = 0; kk < kWBK; ++kk) step(kk);
      } else {
        for (int kk = 0; kk < kcount; ++kk) step(kk);
      }
    }
    cp_async_wait<0>();
  };

  mainloop(std::integral_constant<int, 0>{});
  // Value-only f64 MaxPlus/MinPlus: the strict select equals the fmax/fmin
  // fold except for the sign of a zero result (fmax(-0, +0) = +0 in either
  // order, the select keeps the first zero seen).  A CTA with any zero result
  // re-runs its tile with the sign-exact select; MaxMul (accumulator starts
  // at +0 and never decreases) and integer outputs need no re-run.
  if constexpr (!ARGMAX && !OUTI && S != kMaxMul) {
    int zero = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < kWTN; ++j) zero |= (acc[i][j] == 0.0);
    if (__syncthreads_or(zero)) {
      __syncthreads();
      mainloop(std::integral_constant<int, 1>{});
    }
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t gr = m0 + 2 * ty + 32 * (i >> 1) + (i & 1);
    if (gr >= p.m) continue;
#pragma unroll
    for (int j = 0; j < kWTN; ++j) {
      const int64_t gc = n0 + 2 * tx + 32 * (j >> 1) + (j & 1);
      if (gc >= p.n) continue;
      store_w(C, gr * p.ldc + gc, acc[i][j]);
      if (ARGMAX) IDX[gr * p.ldc + gc] = idx[i][j];
    }
  }
}

}  // namespace tg
