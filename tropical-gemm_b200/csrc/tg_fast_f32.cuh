// B200 fast path for f32 tropical GEMM (all three semirings, with or
// without argmax), one launch for a whole strided batch.
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
//  * Argmax without a per-product compare: the value accumulator runs
//    free over a chunk of L k's; at each chunk boundary one strict compare
//    against the snapshot taken at the previous boundary records the chunk
//    of the last strict improvement (the chunk holding the first k that
//    attains the final value).  After the k loop the CTA buckets its outputs
//    by that chunk, re-streams only the chunks that own outputs, and scans
//    each owned chunk from shared memory for the first k whose product
//    equals the final value -- exactly the reference's winner
//    (tropical_gemm.cu:613-618: strict update, lowest k among ties, index 0
//    when nothing beats the semiring zero), and its exact bits (the sign of
//    a zero included).
#pragma once
#include "tg_semiring.cuh"
#include "tg_generic.cuh"

namespace tg {

constexpr int kFBM = 128, kFBN = 128, kFBK = 32, kFThreads = 256, kFStages = 3;
constexpr int kFApitch = kFBK + 4;                 // floats per staged A row
constexpr int kFAStage = kFBM * kFApitch;          // floats
constexpr int kFBStage = kFBK * kFBN;              // floats
constexpr int kFStageFloats = kFAStage + kFBStage;
constexpr int kFMaxChunks = 1024;
constexpr uint16_t kNoChunk = 0xFFFF;
constexpr uint16_t kResolved = 0xFFFE;
constexpr size_t kFSmemValues = size_t(kFStages) * kFStageFloats * 4;
constexpr size_t kFSmemArgmax = kFSmemValues + 2 * size_t(kFBM * kFBN) * 2 + (kFMaxChunks + 1) * 4;

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

// Stage k-tile `kt` of the CTA's A rows [m0, m0+128) and B cols [n0, n0+128).
// Out-of-range elements are zero-filled (their products are never used or
// are neutralised by fix_k_tail).
__device__ __forceinline__ void fast_load_tile(float* stage, const float* __restrict__ A, const float* __restrict__ B,
                                               const GemmArgs& p, int64_t m0, int64_t n0, int64_t kt, int tid) {
  const int64_t k0 = kt * kFBK;
  float* As = stage;
  float* Bs = stage + kFAStage;
#pragma unroll
  for (int e = 0; e < (kFBM * kFBK / 4) / kFThreads; ++e) {  // 4 x 16B per thread
    int q = tid + e * kFThreads;
    int row = q >> 3, kq = (q & 7) * 4;
    int64_t gr = m0 + row, gk = k0 + kq;
    int bytes = 0;
    const float* src = A;
    if (gr < p.m && gk < p.k) {
      int64_t rem = p.k - gk;
      bytes = rem >= 4 ? 16 : int(rem) * 4;
      src = A + gr * p.lda + gk;
    }
    cp_async16(smem_u32(As + row * kFApitch + kq), src, bytes);
  }
#pragma unroll
  for (int e = 0; e < (kFBK * kFBN) / kFThreads; ++e) {      // 16 x 4B per thread
    int lin = tid + e * kFThreads;
    int kk = lin >> 7, nn = lin & 127;
    int64_t gk = k0 + kk, gc = n0 + nn;
    int bytes = 0;
    const float* src = B;
    if (gk < p.k && gc < p.n) { bytes = 4; src = B + gk * p.ldb + gc; }
    cp_async4(smem_u32(Bs + ((kk >> 1) * kFBN + nn) * 2 + (kk & 1)), src, bytes);
  }
}

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

template <int S, bool ARGMAX>
__global__ void __launch_bounds__(kFThreads, 1)
fast_f32_kernel(GemmArgs p, int tiles_per_chunk) {
  using Op = FastOps<S>;
  extern __shared__ __align__(16) float smem[];
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int lm = lane >> 3, ln = lane & 7;
  const int wm = warp >> 1, wn = warp & 1;

  const int64_t batch = blockIdx.z;
  const float* __restrict__ A = static_cast<const float*>(p.a) + batch * p.sa;
  const float* __restrict__ B = static_cast<const float*>(p.b) + batch * p.sb;
  float* __restrict__ C = static_cast<float*>(p.c) + batch * p.sc;
  int32_t* __restrict__ IDX = ARGMAX ? p.argmax + batch * p.sc : nullptr;
  const int64_t m0 = int64_t(blockIdx.x) * kFBM;
  const int64_t n0 = int64_t(blockIdx.y) * kFBN;
  const int64_t ktiles = (p.k + kFBK - 1) / kFBK;
  const int kvalid_last = int(p.k - (ktiles - 1) * kFBK);

  uint16_t* cid = reinterpret_cast<uint16_t*>(smem + kFStages * kFStageFloats);
  if (ARGMAX) {
    for (int i = tid; i < kFBM * kFBN; i += kFThreads) cid[i] = kNoChunk;
  }

  float acc[8][8];
  float snap[ARGMAX ? 8 : 1][ARGMAX ? 8 : 1];
#pragma unroll
  for (int r = 0; r < 8; ++r)
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      acc[r][c] = Op::zero();
      if (ARGMAX) snap[r][c] = Op::zero();
    }

  // ------------------------------------------------------------ main loop
#pragma unroll
  for (int s = 0; s < kFStages - 1; ++s) {
    if (s < ktiles) fast_load_tile(smem + s * kFStageFloats, A, B, p, m0, n0, s, tid);
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
      int64_t nt = t + kFStages - 1;
      if (nt < ktiles) fast_load_tile(smem + (nt % kFStages) * kFStageFloats, A, B, p, m0, n0, nt, tid);
      cp_async_commit();
    }
    const float* Ap = stage + (wm * 32 + lm) * kFApitch;
    const float* Bp = stage + kFAStage + (wn * 64 + 2 * ln) * 2;
#pragma unroll
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
            Op::pair(lo, hi, a0, a1, bq[q].x, bq[q].y);
            acc[r][2 * q] = Op::red3(acc[r][2 * q], lo, hi);
            Op::pair(lo, hi, a0, a1, bq[q].z, bq[q].w);
            acc[r][2 * q + 1] = Op::red3(acc[r][2 * q + 1], lo, hi);
          }
        }
      }
    }
    if (ARGMAX && ((t + 1) % tiles_per_chunk == 0 || t == ktiles - 1)) {
      const uint16_t chunk = uint16_t(t / tiles_per_chunk);
#pragma unroll
      for (int r = 0; r < 8; ++r)
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          if (Op::better(acc[r][c], snap[r][c])) {
            const int lr = wm * 32 + r * 4 + lm;
            const int lc = wn * 64 + 16 * (c >> 1) + 2 * ln + (c & 1);
            cid[lr * kFBN + lc] = chunk;
          }
          snap[r][c] = acc[r][c];
        }
    }
  }
  cp_async_wait<0>();

  // ------------------------------------------------------------ epilogue
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int lr = wm * 32 + r * 4 + lm;
    const int64_t gr = m0 + lr;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int lc = wn * 64 + 16 * (c >> 1) + 2 * ln + (c & 1);
      const int64_t gc = n0 + lc;
      if (gr >= p.m || gc >= p.n) {
        if (ARGMAX) cid[lr * kFBN + lc] = kNoChunk;   // padding: never resolved
        continue;
      }
      float v = acc[r][c];
      if (ARGMAX) {
        const uint16_t ch = cid[lr * kFBN + lc];
        if (ch == kNoChunk) { v = Op::zero(); IDX[gr * p.ldc + gc] = 0; }
        else IDX[gr * p.ldc + gc] = int32_t(int64_t(ch) * tiles_per_chunk * kFBK);
      }
      C[gr * p.ldc + gc] = v;
    }
  }
  if (!ARGMAX) return;

  // -------------------------------------------- argmax: bucket by chunk
  __syncthreads();
  uint16_t* list = cid + kFBM * kFBN;
  int* off = reinterpret_cast<int*>(list + kFBM * kFBN);   // kFMaxChunks + 1
  const int nchunks = int((ktiles + tiles_per_chunk - 1) / tiles_per_chunk);
  for (int i = tid; i <= nchunks; i += kFThreads) off[i] = 0;
  __syncthreads();
  for (int i = tid; i < kFBM * kFBN; i += kFThreads) {
    const uint16_t ch = cid[i];
    if (ch != kNoChunk) atomicAdd(&off[ch + 1], 1);
  }
  __syncthreads();
  if (warp == 0) {  // inclusive scan of counts -> bucket starts (off[c]..off[c+1])
    int carry = 0;
    for (int base = 1; base <= nchunks; base += 32) {
      int i = base + lane;
      int v = i <= nchunks ? off[i] : 0;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        int u = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += u;
      }
      if (i <= nchunks) off[i] = v + carry;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
  }
  __syncthreads();
  // Scatter: reuse counts as cursors via a second pass with atomics on a
  // copy kept in the scan results (off[c] is the start; use atomicAdd on a
  // running cursor stored in the (now free) first stage buffer).
  int* cursor = reinterpret_cast<int*>(smem);   // stage 0 is idle here
  for (int i = tid; i < nchunks; i += kFThreads) cursor[i] = off[i];
  __syncthreads();
  for (int i = tid; i < kFBM * kFBN; i += kFThreads) {
    const uint16_t ch = cid[i];
    if (ch != kNoChunk) list[atomicAdd(&cursor[ch], 1)] = uint16_t(i);
  }
  __syncthreads();

  // ---------------------------- argmax: re-stream owned chunks and scan
  // Sequence of k-tiles to revisit: all tiles of every chunk that owns at
  // least one output, in ascending k.
  auto next_owned = [&](int c) {
    while (c < nchunks && off[c + 1] == off[c]) ++c;
    return c;
  };
  int ld_chunk = next_owned(0);
  int64_t ld_tile = int64_t(ld_chunk) * tiles_per_chunk;
  auto advance = [&](int& ch, int64_t& tl) {
    ++tl;
    if (tl >= int64_t(ch + 1) * tiles_per_chunk || tl >= ktiles) {
      ch = next_owned(ch + 1);
      tl = int64_t(ch) * tiles_per_chunk;
    }
  };
  int64_t issued = 0;
#pragma unroll
  for (int s = 0; s < kFStages - 1; ++s) {
    if (ld_chunk < nchunks) {
      fast_load_tile(smem + (issued % kFStages) * kFStageFloats, A, B, p, m0, n0, ld_tile, tid);
      advance(ld_chunk, ld_tile);
    }
    ++issued;
    cp_async_commit();
  }
  int cur_chunk = next_owned(0);
  int64_t cur_tile = int64_t(cur_chunk) * tiles_per_chunk;
  for (int64_t it = 0; cur_chunk < nchunks; ++it) {
    cp_async_wait<kFStages - 2>();
    __syncthreads();
    float* stage = smem + (it % kFStages) * kFStageFloats;
    if (ld_chunk < nchunks) {
      fast_load_tile(smem + (issued % kFStages) * kFStageFloats, A, B, p, m0, n0, ld_tile, tid);
      advance(ld_chunk, ld_tile);
    }
    ++issued;
    cp_async_commit();

    const float* As = stage;
    const float* Bs = stage + kFAStage;
    const int64_t k0 = cur_tile * kFBK;
    const int kcount = int((p.k - k0) < kFBK ? (p.k - k0) : kFBK);
    const int beg = off[cur_chunk], end = off[cur_chunk + 1];
    for (int e = beg + tid; e < end; e += kFThreads) {
      const int o = list[e];
      if (cid[o] == kResolved) continue;
      const int lr = o >> 7, lc = o & 127;
      const int64_t gofs = (m0 + lr) * p.ldc + (n0 + lc);
      const float v = C[gofs];
      for (int kk = 0; kk < kcount; ++kk) {
        const float prod = Op::mul(As[lr * kFApitch + kk], Bs[((kk >> 1) * kFBN + lc) * 2 + (kk & 1)]);
        if (prod == v) {
          C[gofs] = prod;
          IDX[gofs] = int32_t(k0 + kk);
          cid[o] = kResolved;
          break;
        }
      }
    }
    advance(cur_chunk, cur_tile);
  }
  cp_async_wait<0>();
}

}  // namespace tg
