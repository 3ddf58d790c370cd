// B200 fast path for f32 tropical GEMM (all three semirings, with or
// without argmax).
//
// Why it looks like this (sm_100a, no tensor cores for (max,+)):
//  * Two products per instruction on each SIMT pipe: products come from
//    `add/mul.rn.f32x2` (FMA pipe) on a pair of consecutive k for one
//    output, and both are folded into the accumulator by one 3-input
//    `max/min.f32` (ALU pipe).  Each (output, k) product is one correctly
//    rounded IEEE operation, and max/min is exact, so the value equals the
//    reference's sequential loop whatever the association.
//  * k-paired operands: A is staged row-major (k contiguous) so a k-pair is
//    a natural 64-bit register pair; B is staged k-pair-interleaved
//    ([k/2][n][2]) by 4-byte cp.async, so its k-pair is a register pair too.
//  * 128x128x32 CTA tiles, 256 threads, 8x8 outputs per thread, 3-stage
//    cp.async pipeline, one CTA per SM (register bound).
//
// Kernels:
//  * fast_f32_kernel<S, ARGMAX = false>: values only, one CTA per tile.
//  * fast_f32_kernel<S, ARGMAX = true> (short K; the host picks it for
//    K <= 1024): the pair index of the last strict improvement is kept in
//    registers and the winning k within that pair is settled in the
//    epilogue from the two products reloaded from A and B.
//  * fast_f32_argmax_kernel (tg_fast_f32_argmax.cuh): long K, persistent,
//    argmax by chunk detection resolved inside the next tile's k loop.
#pragma once
#include "tg_semiring.cuh"
#include "tg_generic.cuh"
#include <type_traits>

namespace tg {

constexpr int kFBM = 128, kFBN = 128, kFBK = 32, kFThreads = 256, kFStages = 3;
constexpr int kFApitch = kFBK + 4;                 // floats per staged A row
constexpr int kFAStage = kFBM * kFApitch;          // floats
constexpr int kFBStage = kFBK * kFBN;              // floats
constexpr int kFStageFloats = kFAStage + kFBStage;
constexpr size_t kFSmemValues = size_t(kFStages) * kFStageFloats * 4;
#ifndef TG_K4_UNROLL
#define TG_K4_UNROLL 8
#endif
constexpr int kK4Unroll = TG_K4_UNROLL;   // unrolled 4-k steps of the k-tile loop body

template <int S> struct FastOps;
template <> struct FastOps<kMaxPlus> {
  static __device__ __forceinline__ float zero() { return __int_as_float(0xff800000); }
  static __device__ __forceinline__ void pair(float& lo, float& hi, float a0, float a1, float b0, float b1) {
    unsigned long long pa, pb, s;
    asm("mov.b64 %0, {%1, %2};" : "=l"(pa) : "f"(a0), "f"(a1));
    asm("mov.b64 %0, {%1, %2};" : "=l"(pb) : "f"(b0), "f"(b1));
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(s) : "l"(pa), "l"(pb));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(s));
  }
  static __device__ __forceinline__ float red3(float acc, float x, float y) {
    float r; asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(acc), "f"(x), "f"(y)); return r;
  }
  static __device__ __forceinline__ float mul(float a, float b) { return __fadd_rn(a, b); }
  static __device__ __forceinline__ bool better(float p, float acc) { return p > acc; }
};
template <> struct FastOps<kMinPlus> {
  static __device__ __forceinline__ float zero() { return __int_as_float(0x7f800000); }
  static __device__ __forceinline__ void pair(float& lo, float& hi, float a0, float a1, float b0, float b1) {
    FastOps<kMaxPlus>::pair(lo, hi, a0, a1, b0, b1);
  }
  static __device__ __forceinline__ float red3(float acc, float x, float y) {
    float r; asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(acc), "f"(x), "f"(y)); return r;
  }
  static __device__ __forceinline__ float mul(float a, float b) { return __fadd_rn(a, b); }
  static __device__ __forceinline__ bool better(float p, float acc) { return p < acc; }
};
template <> struct FastOps<kMaxMul> {
  static __device__ __forceinline__ float zero() { return 0.0f; }
  static __device__ __forceinline__ void pair(float& lo, float& hi, float a0, float a1, float b0, float b1) {
    unsigned long long pa, pb, s;
    asm("mov.b64 %0, {%1, %2};" : "=l"(pa) : "f"(a0), "f"(a1));
    asm("mov.b64 %0, {%1, %2};" : "=l"(pb) : "f"(b0), "f"(b1));
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(s) : "l"(pa), "l"(pb));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(s));
  }
  static __device__ __forceinline__ float red3(float acc, float x, float y) {
    return FastOps<kMaxPlus>::red3(acc, x, y);
  }
  static __device__ __forceinline__ float mul(float a, float b) { return __fmul_rn(a, b); }
  static __device__ __forceinline__ bool better(float p, float acc) { return p > acc; }
};

__device__ __forceinline__ int64_t i64min(int64_t a, int64_t b) { return a < b ? a : b; }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" :: "r"(dst), "l"(src), "r"(bytes));
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, int bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" :: "r"(dst), "l"(src), "r"(bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" :: "n"(N));
}

// Per-thread staging of the A side of one k-tile (128 rows x 32 k, row-major,
// kFApitch floats per row), every address term that does not depend on the
// k-tile precomputed.  Thread t copies rows (t>>3) + 32e, e = 0..3, at k
// offset 4*(t&7) as 16-byte cp.async; unaligned A rows (lda % 4 != 0 or a
// misaligned base) use 4-byte copies instead.  Out-of-range rows and k are
// zero-filled (src-size 0); the k tail of the last tile is fixed up by
// fix_k_tail.
struct ALoader {
  const float* src;     // A + (m0 + (t>>3)) * lda + 4*(t&7)
  const float* base;    // A + m0 * lda
  int64_t step;         // 32 * lda
  int64_t k, lda, rows;
  uint32_t dst;         // this thread's stage-0 destination
  uint32_t smem;        // stage-0 A base
  int kq, tid;
  uint32_t rowmask;     // bit e: row (t>>3) + 32e exists
  bool vec;

  __device__ __forceinline__ ALoader(const float* A, int64_t lda_, int64_t m, int64_t k_, int64_t m0, int tid_,
                                     uint32_t smem_a, bool avec) {
    const int ra = tid_ >> 3;
    kq = (tid_ & 7) * 4;
    step = 32 * lda_;
    rowmask = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (m0 + ra + 32 * e < m) rowmask |= 1u << e;
    src = (m0 + ra < m) ? A + (m0 + ra) * lda_ + kq : A;
    base = A + m0 * lda_;
    k = k_;
    lda = lda_;
    rows = m - m0;
    dst = smem_a + uint32_t((ra * kFApitch + kq) * 4);
    smem = smem_a;
    tid = tid_;
    vec = avec;
  }

  __device__ __forceinline__ void load(uint32_t soff, int64_t kt) const {
    const int64_t k0 = kt * kFBK;
    if (!vec) {
#pragma unroll
      for (int e = 0; e < (kFBM * kFBK) / kFThreads; ++e) {
        const int lin = tid + e * kFThreads;
        const int row = lin >> 5, kk = lin & 31;
        const bool ok = row < rows && k0 + kk < k;
        cp_async4(smem + soff + uint32_t((row * kFApitch + kk) * 4), ok ? base + row * lda + k0 + kk : base,
                  ok ? 4 : 0);
      }
      return;
    }
    const float* s = src + k0;
    int bytes = 16;
    if (k0 + kFBK > k) {
      const int64_t rem = k - (k0 + kq);
      bytes = rem >= 4 ? 16 : (rem > 0 ? int(rem) * 4 : 0);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const bool ok = (rowmask >> e) & 1u;
      cp_async16(dst + soff + uint32_t(e * 32 * kFApitch * 4), ok && bytes ? s : src, ok ? bytes : 0);
      s += step;
    }
  }
};

// Per-thread staging of the B side of one k-tile (32 k x 128 n) into the
// k-pair-interleaved layout [k/2][n][2] by 4-byte cp.async: thread t copies
// column t&127 for k rows (t>>7) + 2e, e = 0..15, so its shared-memory
// destinations are 1 KiB apart and its sources 2*ldb apart.  Out-of-range
// columns and k are zero-filled and never stored.
struct BLoader {
  const float* src;     // B + (t>>7) * ldb + n0 + (t&127)
  int64_t step;         // 2 * ldb
  int64_t k;
  uint32_t dst;
  int kpar;
  bool colok;

  __device__ __forceinline__ BLoader(const float* B, int64_t ldb, int64_t n, int64_t k_, int64_t n0, int tid,
                                     uint32_t smem_b) {
    kpar = tid >> 7;
    const int nn = tid & 127;
    colok = (n0 + nn) < n;
    step = 2 * ldb;
    src = colok ? B + int64_t(kpar) * ldb + n0 + nn : B;
    k = k_;
    dst = smem_b + uint32_t((nn * 2 + kpar) * 4);
  }

  __device__ __forceinline__ void load(uint32_t soff, int64_t kt) const {
    const int64_t k0 = kt * kFBK;
#ifdef TG_EXP_B16
    {  // experiment: the cost of four 16-byte copies per thread (wrong layout)
      const float* b0 = src - kpar * (step >> 1);
      const uint32_t d0 = dst - uint32_t(((threadIdx.x & 127) * 2 + kpar) * 4);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int lin = threadIdx.x + e * kFThreads;
        const int kk = lin >> 5, c = (lin & 31) * 4;
        cp_async16(d0 + soff + uint32_t((kk * kFBN + c) * 4), b0 + (k0 + kk) * (step >> 1) + c - (threadIdx.x & 127), 16);
      }
      return;
    }
#endif
    const float* s = src + k0 * (step >> 1);
    if (k0 + kFBK <= k) {
      const int bytes = colok ? 4 : 0;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        cp_async4(dst + soff + uint32_t(e * kFBN * 2 * 4), s, bytes);
        s += colok ? step : 0;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const bool ok = colok && (k0 + kpar + 2 * e < k);
        cp_async4(dst + soff + uint32_t(e * kFBN * 2 * 4), ok ? s : src, ok ? 4 : 0);
        s += colok ? step : 0;
      }
    }
  }
};

// Semiring zero into the A columns k >= K of the last (partial) k-tile, so
// padded k-pairs never produce a winning product.
template <int S>
__device__ __forceinline__ void fix_k_tail(float* stage, int kvalid, int tid) {
  float* As = stage;
  const int width = kFBK - kvalid;
  for (int i = tid; i < kFBM * width; i += kFThreads) {
    int row = i / width, kk = kvalid + i % width;
    As[row * kFApitch + kk] = FastOps<S>::zero();
  }
}

// OUTI: C is int32 (the i32 path computes exactly in f32 on converted
// operands and converts the result back).
template <typename CT>
__device__ __forceinline__ void store_c(CT* C, int64_t o, float v) {
  if constexpr (sizeof(CT) == 4 && !std::is_same<CT, float>::value) C[o] = CT(v); else C[o] = v;
}

// The k loop body over one staged k-tile: this thread's 8x8 outputs, rows
// wm*32 + 4r + lm, columns wn*64 + 16(c>>1) + 2ln + (c&1).  PAIR also keeps,
// per output, the first k of the k-pair that held the last strict
// improvement (kbase = the tile's first k).
template <int S, bool PAIR>
__device__ __forceinline__ void tile_math(const float* stage, int wm, int wn, int lm, int ln, float (&acc)[8][8],
                                          int32_t (&pidx)[PAIR ? 8 : 1][PAIR ? 8 : 1], int64_t kbase) {
  using Op = FastOps<S>;
  const float* Ap = stage + (wm * 32 + lm) * kFApitch;
  const float* Bp = stage + kFAStage + (wn * 64 + 2 * ln) * 2;
#pragma unroll kK4Unroll
  for (int k4 = 0; k4 < kFBK; k4 += 4) {
    float4 a[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) a[r] = *reinterpret_cast<const float4*>(Ap + r * 4 * kFApitch + k4);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float4 bq[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        bq[q] = *reinterpret_cast<const float4*>(Bp + (k4 / 2 + h) * (kFBN * 2) + q * 32);
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const float a0 = h ? a[r].z : a[r].x;
        const float a1 = h ? a[r].w : a[r].y;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float lo, hi;
          if (PAIR) {
            const int32_t kg = int32_t(kbase + k4 + 2 * h);
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              Op::pair(lo, hi, a0, a1, e ? bq[q].z : bq[q].x, e ? bq[q].w : bq[q].y);
              float& av = acc[r][2 * q + e];
              const float nv = Op::red3(av, lo, hi);
              if (Op::better(nv, av)) pidx[r][2 * q + e] = kg;
              av = nv;
            }
          } else {
            Op::pair(lo, hi, a0, a1, bq[q].x, bq[q].y);
            acc[r][2 * q] = Op::red3(acc[r][2 * q], lo, hi);
            Op::pair(lo, hi, a0, a1, bq[q].z, bq[q].w);
            acc[r][2 * q + 1] = Op::red3(acc[r][2 * q + 1], lo, hi);
          }
        }
      }
    }
  }
}

// Values only (ARGMAX = false) or, for short K, argmax by k-pair tracking
// (ARGMAX = true): ~2 more instructions per product than values only, but
// nothing to resolve after the k loop except one reload per output.
// acc_init: accumulator start value (the semiring zero for f32; the
// reference's integer sentinel for the i32 path, whose sentinel operands the
// conversion maps to +-inf).  AVEC: A rows are 16-byte aligned.
template <int S, bool ARGMAX, bool OUTI = false, bool AVEC = true>
__global__ void __launch_bounds__(kFThreads, 1)
fast_f32_kernel(GemmArgs p, float acc_init) {
  using Op = FastOps<S>;
  using CT = typename std::conditional<OUTI, int32_t, float>::type;
  if (gated_off(p)) return;
  extern __shared__ __align__(16) float smem[];
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int lm = lane >> 3, ln = lane & 7;
  const int wm = warp >> 1, wn = warp & 1;

  const int64_t batch = blockIdx.z;
  const float* __restrict__ A = static_cast<const float*>(p.a) + batch * p.sa;
  const float* __restrict__ B = static_cast<const float*>(p.b) + batch * p.sb;
  CT* __restrict__ C = static_cast<CT*>(p.c) + batch * p.sc;
  int32_t* __restrict__ IDX = ARGMAX ? p.argmax + batch * p.sc : nullptr;
  const int64_t m0 = int64_t(blockIdx.x) * kFBM;
  const int64_t n0 = int64_t(blockIdx.y) * kFBN;
  const int64_t ktiles = (p.k + kFBK - 1) / kFBK;
  const int kvalid_last = int(p.k - (ktiles - 1) * kFBK);

  const uint32_t sbase = smem_u32(smem);
  const ALoader la(A, p.lda, p.m, p.k, m0, tid, sbase, AVEC);
  const BLoader lb(B, p.ldb, p.n, p.k, n0, tid, sbase + kFAStage * 4);
  constexpr uint32_t kStageBytes = uint32_t(kFStageFloats * 4);

  float acc[8][8];
  int32_t pidx[ARGMAX ? 8 : 1][ARGMAX ? 8 : 1];
#pragma unroll
  for (int r = 0; r < 8; ++r)
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      acc[r][c] = acc_init;
      if (ARGMAX) pidx[r][c] = -1;
    }

#pragma unroll
  for (int s = 0; s < kFStages - 1; ++s) {
    if (s < ktiles) {
      la.load(s * kStageBytes, s);
      lb.load(s * kStageBytes, s);
    }
    cp_async_commit();
  }
  for (int64_t t = 0; t < ktiles; ++t) {
    cp_async_wait<kFStages - 2>();
    __syncthreads();
    float* stage = smem + (t % kFStages) * kFStageFloats;
    if (t == ktiles - 1 && kvalid_last < kFBK) {
      fix_k_tail<S>(stage, kvalid_last, tid);
      __syncthreads();
    }
    {
      const int64_t nt = t + kFStages - 1;
      if (nt < ktiles) {
        la.load(uint32_t(nt % kFStages) * kStageBytes, nt);
        lb.load(uint32_t(nt % kFStages) * kStageBytes, nt);
      }
      cp_async_commit();
    }
    tile_math<S, ARGMAX>(stage, wm, wn, lm, ln, acc, pidx, t * kFBK);
  }
  cp_async_wait<0>();

#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int64_t gr = m0 + wm * 32 + r * 4 + lm;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int64_t gc = n0 + wn * 64 + 16 * (c >> 1) + 2 * ln + (c & 1);
      if (gr >= p.m || gc >= p.n) continue;
      if (ARGMAX) {
        // pidx: first k of the pair that held the last strict improvement
        // (-1: none, the output is (zero, 0)).  The reference's index is the
        // pair's first k whose product equals the final value; its bits are
        // that product's (the fold may differ in the sign of a zero).
        const int32_t kg = pidx[r][c];
        float v = acc_init;
        int32_t kw = 0;
        if (kg >= 0) {
          const float lo = Op::mul(A[gr * p.lda + kg], B[int64_t(kg) * p.ldb + gc]);
          if (lo == acc[r][c] || kg + 1 >= p.k) {
            v = lo;
            kw = kg;
          } else {
            v = Op::mul(A[gr * p.lda + kg + 1], B[int64_t(kg + 1) * p.ldb + gc]);
            kw = kg + 1;
          }
        }
        store_c(C, gr * p.ldc + gc, v);
        IDX[gr * p.ldc + gc] = kw;
      } else {
        store_c(C, gr * p.ldc + gc, acc[r][c]);
      }
    }
  }
}

}  // namespace tg

#include "tg_fast_f32_argmax.cuh"
