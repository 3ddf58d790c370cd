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
//  * Short K (the host picks PAIR for K <= 1024, where the re-stream's fixed
//    cost per output would dominate): the 4-k group of the last strict
//    improvement is kept in registers and the winning k within that group is
//    settled in the epilogue from the four products reloaded from A and B.
#pragma once
#include "tg_semiring.cuh"
#include "tg_generic.cuh"
#include <type_traits>
#include <cuda.h>

namespace tg {

constexpr int kFBM = 128, kFBN = 128, kFBK = 32, kFThreads = 256, kFStages = 3;
constexpr int kFApitch = kFBK + 4;                 // floats per staged A row
constexpr int kFAStage = kFBM * kFApitch;          // floats
constexpr int kFBStage = kFBK * kFBN;              // floats
constexpr int kFStageFloats = kFAStage + kFBStage;
constexpr int kFMaxChunks = 1024;
constexpr uint16_t kNoChunk = 0xFFFF;              // output never beat the semiring zero
constexpr size_t kFSmemValues = size_t(kFStages) * kFStageFloats * 4;
// Argmax kernel shared-memory map.  During the k loop: the three pipeline
// stages and one chunk id (u16) per CTA output.  After the outputs are
// bucketed by chunk, kRStages ring slots (overlaying stages and chunk ids)
// re-stream the owned chunks -- three two-tile chunks resident or in flight,
// so the scan of one chunk overlaps the copies of the next two; the bucketed
// list and its u16 offsets sit above the ring.
constexpr int kRStages = 6;
constexpr int kRAFloats = kFBM * kFBK;                     // A slot: 128 rows x 32 k, 16-byte groups swizzled
constexpr int kRStageFloats = kRAFloats + kFBK * kFBN;     // + B slot: 32 k x 128 n, swizzled
constexpr size_t kOffCid = kFSmemValues;
constexpr size_t kOffList = size_t(kRStages) * kRStageFloats * 4;
constexpr size_t kOffOff = kOffList + size_t(kFBM * kFBN) * 2;
constexpr size_t kOffBar = (kOffOff + size_t(kFMaxChunks + 1) * 2 + 7) & ~size_t(7);   // ring mbarriers (TMA)
constexpr size_t kFSmemArgmax = kOffBar + size_t(kRStages) * 8;
static_assert(kOffCid + size_t(kFBM * kFBN) * 2 <= kOffList, "chunk ids overlap the list");
static_assert(size_t(2 * (kFMaxChunks + 1)) * 4 <= kOffCid, "bucket counters overlap the chunk ids");
static_assert(kFSmemArgmax <= 232448, "argmax kernel exceeds shared memory");
static_assert(kFBM * kFBN <= 65535, "u16 bucket offsets");

// Ring-slot element positions.  Rows keep their natural length (no padding);
// instead the 16-byte groups of a row are XOR-swizzled by the row index, so
// the scan's column reads (4 lanes on consecutive k of one output, 8 outputs
// per warp) spread over the banks.
__device__ __forceinline__ int ring_a(int r, int k) { return r * kFBK + ((((k >> 2) ^ (r & 7)) << 2) | (k & 3)); }
__device__ __forceinline__ int ring_b(int k, int n) {   // four 32-column boxes of 128-byte rows
  return kRAFloats + (n >> 5) * (kFBK * 32) + k * 32 + (((((n >> 2) & 7) ^ (k & 7)) << 2) | (n & 3));
}

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

// ---- TMA re-stream of the ring (bulk tensor copies completing on an
// mbarrier per ring slot; no multicast).  The ring's A slot (128 rows x 32 k,
// 128-byte rows) and B slot (four 32 k x 32 n boxes) use the hardware's
// 128-byte swizzle, which is the XOR pattern of ring_a / ring_b below.
__device__ __forceinline__ void mbar_init(uint32_t bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" :: "r"(bar), "r"(count));
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" :: "r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void tma_load3(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];\n"
      :: "r"(dst), "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar) : "memory");
}
// Waits for phase `parity` of the barrier, giving up after a bounded number
// of polls (returns false then; the caller marks its outputs).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  for (int i = 0; i < (1 << 22); ++i) {
    uint32_t done;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(done) : "r"(bar), "r"(parity) : "memory");
    if (done) return true;
  }
  return false;
}

// Per-thread staging of k-tiles into one pipeline stage, with every address
// term that does not depend on the tile precomputed once per CTA.
//  A: 128 rows x 32 k as 16-byte cp.async; thread t copies rows
//     (t>>3) + 32e, e = 0..3, at k offset 4*(t&7).
//  B: 32 k x 128 n as 4-byte cp.async into the k-pair-interleaved layout;
//     thread t copies column t&127 for rows (t>>7) + 2e, e = 0..15, so its
//     shared-memory destinations are 1 KiB apart and its sources 2*ldb apart.
// Out-of-range rows/columns are zero-filled (src-size 0) and never stored;
// the k tail of the last tile is fixed up by fix_k_tail.
struct TileLoader {
  const float* a_src;   // A + (m0 + (t>>3)) * lda + 4*(t&7)
  const float* b_src;   // B + (t>>7) * ldb + n0 + (t&127)
  int64_t a_step;       // 32 * lda
  int64_t b_step;       // 2 * ldb
  int64_t k;
  uint32_t a_dst, b_dst;
  int a_kq, b_kpar;
  uint32_t a_rowmask;   // bit e: row (t>>3) + 32e exists
  bool b_colok;
  // A rows not 16-byte aligned (lda % 4 != 0 or a misaligned base): 4-byte copies
  bool a_vec;
  const float* a_base;  // A + m0 * lda
  int64_t a_lda, a_rows;
  uint32_t a_smem;      // stage-0 A base
  int tid_;

  __device__ __forceinline__ TileLoader(const float* A, const float* B, const GemmArgs& p, int64_t m0, int64_t n0,
                                        int tid, const float* smem_base, bool avec = true) {
    const int ra = tid >> 3;
    a_kq = (tid & 7) * 4;
    a_step = 32 * p.lda;
    a_rowmask = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (m0 + ra + 32 * e < p.m) a_rowmask |= 1u << e;
    a_src = (m0 + ra < p.m) ? A + (m0 + ra) * p.lda + a_kq : A;
    b_kpar = tid >> 7;
    const int nn = tid & 127;
    b_colok = (n0 + nn) < p.n;
    b_step = 2 * p.ldb;
    b_src = b_colok ? B + int64_t(b_kpar) * p.ldb + n0 + nn : B;
    k = p.k;
    a_dst = smem_u32(smem_base) + uint32_t((ra * kFApitch + a_kq) * 4);
    a_vec = avec;
    a_base = A + m0 * p.lda;
    a_lda = p.lda;
    a_rows = p.m - m0;
    a_smem = smem_u32(smem_base);
    tid_ = tid;
    b_dst = smem_u32(smem_base + kFAStage) + uint32_t((nn * 2 + b_kpar) * 4);
  }

  __device__ __forceinline__ void load(int stage, int64_t kt) const {
    const uint32_t soff = uint32_t(stage) * uint32_t(kFStageFloats * 4);
    load_a_at(soff, kt);
    load_b(soff, kt);
  }

  __device__ __forceinline__ void load_a_at(uint32_t soff, int64_t kt) const {
    const int64_t k0 = kt * kFBK;
    const bool interior = k0 + kFBK <= k;
    if (!a_vec) {
#pragma unroll
      for (int e = 0; e < (kFBM * kFBK) / kFThreads; ++e) {
        const int lin = tid_ + e * kFThreads;
        const int row = lin >> 5, kk = lin & 31;
        const bool ok = row < a_rows && k0 + kk < k;
        cp_async4(a_smem + soff + uint32_t((row * kFApitch + kk) * 4), ok ? a_base + row * a_lda + k0 + kk : a_base,
                  ok ? 4 : 0);
      }
      return;
    }
    {
      const float* src = a_src + k0;
      int bytes = 16;
      if (!interior) {
        const int64_t rem = k - (k0 + a_kq);
        bytes = rem >= 4 ? 16 : (rem > 0 ? int(rem) * 4 : 0);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const bool ok = (a_rowmask >> e) & 1u;
        cp_async16(a_dst + soff + uint32_t(e * 32 * kFApitch * 4), ok && bytes ? src : a_src, ok ? bytes : 0);
        src += a_step;
      }
    }
  }

  __device__ __forceinline__ void load_b(uint32_t soff, int64_t kt) const {
    const int64_t k0 = kt * kFBK;
    const bool interior = k0 + kFBK <= k;
    {
      const float* src = b_src + k0 * (b_step >> 1);
      if (interior) {
        const int bytes = b_colok ? 4 : 0;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          cp_async4(b_dst + soff + uint32_t(e * kFBN * 2 * 4), src, bytes);
          src += b_colok ? b_step : 0;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const bool ok = b_colok && (k0 + b_kpar + 2 * e < k);
          cp_async4(b_dst + soff + uint32_t(e * kFBN * 2 * 4), ok ? src : b_src, ok ? 4 : 0);
          src += b_colok ? b_step : 0;
        }
      }
    }
  }
};

// Re-stream staging of one k-tile into a ring slot (layout of ring_a /
// ring_b).  16-byte copies when rows are 16-byte aligned, 4-byte copies
// otherwise; out-of-range elements are zero-filled (the scan masks k >= K).
struct RingLoader {
  const float* A;   // row m0 of this batch's A
  const float* B;   // this batch's B
  int64_t rows, cols, kdim, lda, ldb, n0;
  int tid;
  bool a_vec, b_vec;
  uint32_t base;
  __device__ __forceinline__ RingLoader(const float* A_, const float* B_, const GemmArgs& p, int64_t m0, int64_t n0_,
                                        int tid_, const float* smem_base, bool avec, bool bvec)
      : A(A_ + m0 * p.lda), B(B_), rows(p.m - m0), cols(p.n - n0_), kdim(p.k), lda(p.lda), ldb(p.ldb), n0(n0_),
        tid(tid_), a_vec(avec), b_vec(bvec), base(smem_u32(smem_base)) {}
  __device__ __forceinline__ void load(int slot, int64_t kt) const {
    const uint32_t sb = base + uint32_t(slot) * uint32_t(kRStageFloats * 4);
    const int64_t k0 = kt * kFBK;
    if (a_vec) {
#pragma unroll
      for (int e = 0; e < (kFBM * kFBK / 4) / kFThreads; ++e) {
        const int lin = tid + e * kFThreads;
        const int r = lin >> 3, kq = (lin & 7) * 4;
        const int64_t rem = kdim - (k0 + kq);
        const int bytes = r < rows ? (rem >= 4 ? 16 : (rem > 0 ? int(rem) * 4 : 0)) : 0;
        cp_async16(sb + uint32_t(ring_a(r, kq) * 4), bytes ? A + r * lda + k0 + kq : A, bytes);
      }
    } else {
#pragma unroll
      for (int e = 0; e < (kFBM * kFBK) / kFThreads; ++e) {
        const int lin = tid + e * kFThreads;
        const int r = lin >> 5, kk = lin & 31;
        const bool ok = r < rows && k0 + kk < kdim;
        cp_async4(sb + uint32_t(ring_a(r, kk) * 4), ok ? A + r * lda + k0 + kk : A, ok ? 4 : 0);
      }
    }
    if (b_vec) {
#pragma unroll
      for (int e = 0; e < (kFBK * kFBN / 4) / kFThreads; ++e) {
        const int lin = tid + e * kFThreads;
        const int kk = lin >> 5, c = (lin & 31) * 4;
        const int64_t rem = cols - c;
        const int bytes = k0 + kk < kdim ? (rem >= 4 ? 16 : (rem > 0 ? int(rem) * 4 : 0)) : 0;
        cp_async16(sb + uint32_t(ring_b(kk, c) * 4), bytes ? B + (k0 + kk) * ldb + n0 + c : B, bytes);
      }
    } else {
#pragma unroll
      for (int e = 0; e < (kFBK * kFBN) / kFThreads; ++e) {
        const int lin = tid + e * kFThreads;
        const int kk = lin >> 7, c = lin & 127;
        const bool ok = k0 + kk < kdim && c < cols;
        cp_async4(sb + uint32_t(ring_b(kk, c) * 4), ok ? B + (k0 + kk) * ldb + n0 + c : B, ok ? 4 : 0);
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

// The 16 products a scan lane owns in a full two-tile chunk: k = sub + 4i
// of each tile (i = 0..7), for output (lr, lc) of the ring slots st0, st1.
// The swizzled positions (ring_a / ring_b) are taken apart once per output:
// A's 16-byte group index is i ^ (lr & 7), and B's XOR key k & 7 is sub or
// sub + 4 by the parity of i, so each load is a base plus an immediate.
template <int S>
__device__ __forceinline__ void chunk_products(const float* st0, const float* st1, int lr, int lc, int sub,
                                               float (&pv)[16]) {
  using Op = FastOps<S>;
  const int ax = lr & 7, abase = lr * kFBK + sub;
  int aoff[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) aoff[i] = abase + ((i ^ ax) << 2);
  const int yb = (lc >> 2) & 7;
  const int bbase = kRAFloats + (lc >> 5) * (kFBK * 32) + sub * 32 + (lc & 3);
  const int b_even = bbase + ((yb ^ sub) << 2), b_odd = bbase + ((yb ^ (sub + 4)) << 2);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int bo = ((i & 1) ? b_odd : b_even) + 128 * i;
    pv[i] = Op::mul(st0[aoff[i]], st0[bo]);
    pv[8 + i] = Op::mul(st1[aoff[i]], st1[bo]);
  }
}

// OUTI: C is int32 (the i32 path computes exactly in f32 on converted
// operands and converts the result back).  acc_init: accumulator start value
// (the semiring zero for f32; the reference's integer sentinel for i32 --
// the sentinel operands themselves are mapped to +-inf by the conversion).
template <typename CT>
__device__ __forceinline__ void store_c(CT* C, int64_t o, float v) {
  if constexpr (sizeof(CT) == 4 && !std::is_same<CT, float>::value) C[o] = CT(v); else C[o] = v;
}

// The k loop body over one staged k-tile: this thread's 8x8 outputs, rows
// wm*32 + 4r + lm, columns wn*64 + 16(c>>1) + 2ln + (c&1).
template <int S, int KUNROLL = kFBK / 4>   // KUNROLL: 4-k steps unrolled per loop trip
__device__ __forceinline__ void tile_math(const float* a_stage, const float* b_stage, int wm, int wn, int lm, int ln,
                                          float (&acc)[8][8]) {
  using Op = FastOps<S>;
  const float* Ap = a_stage + (wm * 32 + lm) * kFApitch;
  const float* Bp = b_stage + (wn * 64 + 2 * ln) * 2;
#pragma unroll KUNROLL
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
}

// Argmax tracked per 4-k group (short K): both k-pairs
// of a group are folded into an output back to back (FADD2, FMNMX3, FADD2,
// FMNMX3), then one strict compare against the value before the group
// records the group of the last strict improvement -- 6 instructions per 4
// products (values only: 4).  The epilogue resolves the winning k inside
// that group from A (global) and B (the resident panel, or global).
// UNROLL: 4-k groups per unrolled body.  The whole k-tile (8) for K > 256;
// 2 for the resident-panel kernel (K <= 256), whose epilogue and k loop do
// not fit the instruction cache together (no-instruction stalls 0.65 per
// issue fully unrolled; config 3 forward 0.540 -> 0.526 ms).
template <int S, int UNROLL = 8>
__device__ __forceinline__ void tile_math_g4(const float* a_stage, const float* b_stage, int wm, int wn, int lm,
                                             int ln, float (&acc)[8][8], int32_t (&pidx)[8][8], int64_t kbase) {
  using Op = FastOps<S>;
  const float* Ap = a_stage + (wm * 32 + lm) * kFApitch;
  const float* Bp = b_stage + (wn * 64 + 2 * ln) * 2;
#pragma unroll UNROLL
  for (int k4 = 0; k4 < kFBK; k4 += 4) {
    float4 a[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) a[r] = *reinterpret_cast<const float4*>(Ap + r * 4 * kFApitch + k4);
    float4 b0[4], b1[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      b0[q] = *reinterpret_cast<const float4*>(Bp + (k4 / 2) * (kFBN * 2) + q * 32);
      b1[q] = *reinterpret_cast<const float4*>(Bp + (k4 / 2 + 1) * (kFBN * 2) + q * 32);
    }
    const int32_t kg = int32_t(kbase + k4);
#pragma unroll
    for (int r = 0; r < 8; ++r) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float l0, h0, l1, h1;
          Op::pair(l0, h0, a[r].x, a[r].y, e ? b0[q].z : b0[q].x, e ? b0[q].w : b0[q].y);
          Op::pair(l1, h1, a[r].z, a[r].w, e ? b1[q].z : b1[q].x, e ? b1[q].w : b1[q].y);
          float& av = acc[r][2 * q + e];
          const float nv = Op::red3(Op::red3(av, l0, h0), l1, h1);
          if (Op::better(nv, av)) pidx[r][2 * q + e] = kg;
          av = nv;
        }
      }
    }
  }
}

// PAIR (with ARGMAX, for short K): instead of chunk detection + re-stream,
// track the winner per 4-k group in registers (tile_math_g4): 1.5
// instructions per product instead of ~1, but no re-stream, whose cost per
// output does not shrink with K.
// AVEC: A rows are 16-byte aligned (else A is staged by 4-byte copies).
// BPANEL (PAIR, K <= kPanelMaxK): B's whole 128-column panel stays resident
// in shared memory (each k-tile's B lands in its own panel slice, A alone
// cycles through the stages), so the epilogue reads the winning group's B
// values from shared memory instead of scattered global loads.
constexpr int kPanelMaxK = 256;
constexpr size_t kFSmemPanel = size_t(kFStages) * kFAStage * 4 + size_t(kPanelMaxK) * kFBN * 4;
static_assert(kFSmemPanel <= 232448, "B-panel kernel exceeds shared memory");

template <int S, bool ARGMAX, bool OUTI = false, bool PAIR = false, bool AVEC = true, bool BPANEL = false>
__global__ void __launch_bounds__(kFThreads, 1)
fast_f32_kernel(GemmArgs p, int tiles_per_chunk, int b_vec, float acc_init, const __grid_constant__ CUtensorMap tma_a,
                const __grid_constant__ CUtensorMap tma_b, int use_tma) {
  using Op = FastOps<S>;
  using CT = typename std::conditional<OUTI, int32_t, float>::type;
  if (gated_off(p)) return;
  extern __shared__ __align__(16) float smem[];
  unsigned char* sbytes = reinterpret_cast<unsigned char*>(smem);
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

  const TileLoader ldr(A, B, p, m0, n0, tid, smem, AVEC);
  uint16_t* cid = reinterpret_cast<uint16_t*>(sbytes + kOffCid);
  if (ARGMAX && !PAIR) {
    for (int i = tid; i < kFBM * kFBN; i += kFThreads) cid[i] = kNoChunk;
  }

  float acc[8][8];
  float snap[ARGMAX && !PAIR ? 8 : 1][ARGMAX && !PAIR ? 8 : 1];
  int32_t pidx[PAIR ? 8 : 1][PAIR ? 8 : 1];
#pragma unroll
  for (int r = 0; r < 8; ++r)
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      acc[r][c] = acc_init;
      if constexpr (!OUTI) {
        if (p.accumulate) {   // start from the current C (a previous K slice's result)
          const int64_t gr = m0 + wm * 32 + r * 4 + lm, gc = n0 + wn * 64 + 16 * (c >> 1) + 2 * ln + (c & 1);
          if (gr < p.m && gc < p.n) acc[r][c] = C[gr * p.ldc + gc];
        }
      }
      if (ARGMAX && !PAIR) snap[r][c] = acc[r][c];
      if (PAIR) pidx[r][c] = -1;
    }

  // ------------------------------------------------------------ main loop
  // stage layout: [A | B] per stage, or (BPANEL) three A stages then the B panel
  auto load_tile = [&](int stg, int64_t kt) {
    if constexpr (BPANEL) {
      ldr.load_a_at(uint32_t(stg) * uint32_t(kFAStage * 4), kt);
      ldr.load_b(uint32_t((kFStages - 1) * kFAStage + int(kt) * kFBStage) * 4u, kt);
    } else {
      ldr.load(stg, kt);
    }
  };
#pragma unroll
  for (int s = 0; s < kFStages - 1; ++s) {
    if (s < ktiles) load_tile(s, s);
    cp_async_commit();
  }
  for (int64_t t = 0; t < ktiles; ++t) {
    cp_async_wait<kFStages - 2>();
    __syncthreads();
    float* stage = smem + (t % kFStages) * (BPANEL ? kFAStage : kFStageFloats);
    const float* bstage = BPANEL ? smem + kFStages * kFAStage + t * kFBStage : stage + kFAStage;
    if (t == ktiles - 1 && kvalid_last < kFBK) {
      fix_k_tail<S>(stage, kvalid_last, tid);
      __syncthreads();
    }
    {
      int64_t nt = t + kFStages - 1;
      if (nt < ktiles) load_tile(int(nt % kFStages), nt);
      cp_async_commit();
    }
    if constexpr (PAIR) tile_math_g4<S, BPANEL ? 2 : 8>(stage, bstage, wm, wn, lm, ln, acc, pidx, t * kFBK);
    else tile_math<S>(stage, bstage, wm, wn, lm, ln, acc);
    if (ARGMAX && !PAIR && ((t + 1) % tiles_per_chunk == 0 || t == ktiles - 1)) {
      // chunk boundary: remember the chunk of each output's latest strict improvement
      const uint16_t chunk = uint16_t(t / tiles_per_chunk);
#pragma unroll
      for (int r = 0; r < 8; ++r)
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          if (Op::better(acc[r][c], snap[r][c]))
            cid[(wm * 32 + r * 4 + lm) * kFBN + wn * 64 + 16 * (c >> 1) + 2 * ln + (c & 1)] = chunk;
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
        if (ARGMAX && !PAIR) cid[lr * kFBN + lc] = kNoChunk;   // padding: never resolved
        continue;
      }
      if (PAIR) {
        // pidx: first k of the pair that held the last strict improvement
        // (-1: none, the output is (zero, 0)).  The reference's index is the
        // pair's first k whose product equals the final value; its bits are
        // that product's (the fold may differ in the sign of a zero).
        const int32_t kg = pidx[r][c];
        float v = acc_init;
        int32_t kw = 0;
        if (kg < 0 && p.accumulate) continue;   // nothing beat the previous slices: keep C and argmax
        if (kg >= 0) {
          // kg: first k of the 4-k group of the last strict improvement; the
          // winner is the group's first k whose product equals the final value
          float bv[4];
          if constexpr (BPANEL) {   // two k-pairs of column lc in the resident panel ([k/2][n][2])
            const float* pan = smem + kFStages * kFAStage + (kg >> 1) * (kFBN * 2) + lc * 2;
            const float2 bb0 = *reinterpret_cast<const float2*>(pan);
            const float2 bb1 = *reinterpret_cast<const float2*>(pan + kFBN * 2);
            bv[0] = bb0.x; bv[1] = bb0.y; bv[2] = bb1.x; bv[3] = bb1.y;
          } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) bv[i] = kg + i < p.k ? B[int64_t(kg + i) * p.ldb + gc] : 0.f;
          }
          // A's four values: one 16-byte load (kg is a multiple of 4 and
          // AVEC rows are 16-byte aligned) unless the group is K's tail
          const float* ar = A + gr * p.lda + kg;
          float av4[4];
          if (AVEC && kg + 4 <= p.k) {
            const float4 a4 = *reinterpret_cast<const float4*>(ar);
            av4[0] = a4.x; av4[1] = a4.y; av4[2] = a4.z; av4[3] = a4.w;
          } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) av4[i] = kg + i < p.k ? ar[i] : 0.f;
          }
          v = acc[r][c];
          kw = kg;
#pragma unroll
          for (int i = 3; i >= 0; --i) {
            if (kg + i < p.k) {
              const float pr = Op::mul(av4[i], bv[i]);
              if (pr == acc[r][c]) {
                v = pr;
                kw = kg + i;
              }
            }
          }
        }
        store_c(C, gr * p.ldc + gc, v);
        IDX[gr * p.ldc + gc] = kw + (kg >= 0 ? p.k_offset : 0);
      } else if (!ARGMAX) {
        store_c(C, gr * p.ldc + gc, acc[r][c]);
      } else if (cid[lr * kFBN + lc] == kNoChunk && !p.accumulate) {   // nothing beat the zero: (zero, index 0)
        store_c(C, gr * p.ldc + gc, acc_init);
        IDX[gr * p.ldc + gc] = 0;
      }
    }
  }
  if (!ARGMAX || PAIR) return;

  // -------------------------------------------- argmax: bucket by chunk
  __syncthreads();
  uint16_t* list = reinterpret_cast<uint16_t*>(sbytes + kOffList);
  uint16_t* off = reinterpret_cast<uint16_t*>(sbytes + kOffOff);
  int* cnt = reinterpret_cast<int*>(smem);            // the stages are idle after the k loop
  int* cursor = cnt + (kFMaxChunks + 1);
  const int nchunks = int((ktiles + tiles_per_chunk - 1) / tiles_per_chunk);
  for (int i = tid; i <= nchunks; i += kFThreads) cnt[i] = 0;
  __syncthreads();
  for (int i = tid; i < kFBM * kFBN; i += kFThreads) {
    const uint16_t ch = cid[i];
    if (ch != kNoChunk) atomicAdd(&cnt[ch + 1], 1);
  }
  __syncthreads();
  if (warp == 0) {  // inclusive scan of counts: bucket c is list[off[c], off[c+1])
    int carry = 0;
    for (int base = 1; base <= nchunks; base += 32) {
      int i = base + lane;
      int v = i <= nchunks ? cnt[i] : 0;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        int u = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += u;
      }
      if (i <= nchunks) cnt[i] = v + carry;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
  }
  __syncthreads();
  for (int i = tid; i <= nchunks; i += kFThreads) {
    off[i] = uint16_t(cnt[i]);
    if (i < nchunks) cursor[i] = cnt[i];
  }
  __syncthreads();
  for (int i = tid; i < kFBM * kFBN; i += kFThreads) {
    const uint16_t ch = cid[i];
    if (ch != kNoChunk) list[atomicAdd(&cursor[ch], 1)] = uint16_t(i);
  }
  __syncthreads();

  // ---------------------- argmax: re-stream the chunks that own outputs
  // Every output of chunk c had its last strict improvement in c, so its
  // final value is the max (min) of its products over c, and its reference
  // index is the first k of c whose product equals that value.  Tiles of the
  // owned chunks stream through a kRStages-deep ring (the chunk ids and the
  // counters are dead now); a chunk is scanned once all its tiles have landed.
  const RingLoader rl(A, B, p, m0, n0, tid, smem, AVEC, b_vec != 0);
  auto next_owned = [&](int c) {
    while (c < nchunks && off[c + 1] == off[c]) ++c;
    return c;
  };
  int ld_chunk = next_owned(0);
  int64_t ld_tile = int64_t(ld_chunk) * tiles_per_chunk;
  int64_t issued = 0;
  // TMA ring: slot base 1024-byte aligned for the 128-byte swizzle
  const bool tma = use_tma != 0 && (smem_u32(smem) & 1023) == 0;
  const uint32_t bars = smem_u32(sbytes + kOffBar);
  if (tma && tid == 0) {
    for (int s2 = 0; s2 < kRStages; ++s2) mbar_init(bars + 8 * s2, 1);
    fence_proxy_async();
  }
  if (tma) __syncthreads();
  auto issue_until = [&](int64_t limit) {
    if (tma && tid == 0) fence_proxy_async();   // the slots' earlier generic accesses come first
    while (ld_chunk < nchunks && issued < limit) {
      if (tma) {
        if (tid == 0) {
          const int slot = int(issued % kRStages);
          const uint32_t sb = smem_u32(smem + slot * kRStageFloats), bar = bars + 8 * slot;
          mbar_expect_tx(bar, uint32_t(kRStageFloats * 4));
          tma_load3(sb, &tma_a, int(ld_tile * kFBK), int(m0), int(batch), bar);
#pragma unroll
          for (int j = 0; j < kFBN / 32; ++j)
            tma_load3(sb + uint32_t((kRAFloats + j * kFBK * 32) * 4), &tma_b, int(n0) + 32 * j, int(ld_tile * kFBK),
                      int(batch), bar);
        }
      } else {
        rl.load(int(issued % kRStages), ld_tile);
        cp_async_commit();
      }
      ++issued;
      ++ld_tile;
      if (ld_tile >= int64_t(ld_chunk + 1) * tiles_per_chunk || ld_tile >= ktiles) {
        ld_chunk = next_owned(ld_chunk + 1);
        ld_tile = int64_t(ld_chunk) * tiles_per_chunk;
      }
    }
  };
  issue_until(kRStages);
  int64_t seq0 = 0;   // ring sequence number of the current chunk's first tile
  const int grp = tid >> 2, sub = tid & 3;
  // a full chunk = two k-tiles with every k < K
  auto full_chunk = [&](int cc) {
    const int64_t tt = int64_t(cc) * tiles_per_chunk;
    return tiles_per_chunk == 2 && tt + 2 <= ktiles && (tt + 2) * kFBK <= p.k;
  };
  for (int c = next_owned(0); c < nchunks; c = next_owned(c + 1)) {
    const int64_t t0 = int64_t(c) * tiles_per_chunk;
    const int nt = int(i64min(tiles_per_chunk, ktiles - t0));
    {
      // Two full owned chunks resident in the ring at once (4 of its 6
      // slots): scanned in one round with four entries per lane group, one
      // barrier for both -- the scan is latency-bound per round, not
      // throughput-bound.
      const int c2 = next_owned(c + 1);
      if (c2 < nchunks && full_chunk(c) && full_chunk(c2) && issued >= seq0 + 4) {
        const int64_t need2 = seq0 + 4;
        bool landed = true;
        if (tma) {
          for (int64_t q = seq0; q < need2; ++q)
            landed = mbar_wait(bars + 8 * uint32_t(q % kRStages), uint32_t((q / kRStages) & 1)) && landed;
        } else {
          const int64_t pending = issued - need2;
          if (pending >= 2) cp_async_wait<2>();
          else if (pending == 1) cp_async_wait<1>();
          else cp_async_wait<0>();
        }
        __syncthreads();
        if (!__syncthreads_and(landed)) {   // a copy never arrived: mark both chunks' outputs, stop
          for (int e = off[c] + tid; e < off[c2 + 1]; e += kFThreads) {
            const int o = list[e];
            IDX[(m0 + (o >> 7)) * p.ldc + (n0 + (o & 127))] = -2;
          }
          return;
        }
        issue_until(seq0 + kRStages);
        const int beg = off[c], mid = off[c + 1], end = off[c2 + 1];
        const int64_t t0b = int64_t(c2) * tiles_per_chunk;
        constexpr int kE4 = 4;
        for (int e0 = beg; e0 < end; e0 += kE4 * (kFThreads / 4)) {
#pragma unroll
          for (int u = 0; u < kE4; ++u) {
            const int e = e0 + u * (kFThreads / 4) + grp;
            const bool act = e < end;
            const bool second = e >= mid;
            const int o = act ? list[e] : 0;
            const int lr = o >> 7, lc = o & 127;
            const int s0 = int((seq0 + (second ? 2 : 0)) % kRStages);
            const float* st0 = smem + s0 * kRStageFloats;
            const float* st1 = smem + (s0 + 1 >= kRStages ? s0 + 1 - kRStages : s0 + 1) * kRStageFloats;
            float pv[16];
            chunk_products<S>(st0, st1, lr, lc, sub, pv);
            float m = Op::red3(Op::red3(Op::red3(pv[0], pv[1], pv[2]), Op::red3(pv[3], pv[4], pv[5]),
                                        Op::red3(pv[6], pv[7], pv[8])),
                               Op::red3(Op::red3(pv[9], pv[10], pv[11]), Op::red3(pv[12], pv[13], pv[14]), pv[15]),
                               pv[15]);
            float x = __shfl_xor_sync(0xffffffffu, m, 1);
            m = Op::red3(m, x, x);
            x = __shfl_xor_sync(0xffffffffu, m, 2);
            m = Op::red3(m, x, x);
            unsigned mask = 0;
#pragma unroll
            for (int q = 0; q < 16; ++q) mask |= (pv[q] == m) ? (1u << q) : 0u;
            unsigned kf = 0xFFFFFFFFu;
            if (mask) {
              const int q = __ffs(mask) - 1;
              kf = unsigned(32 * (q >> 3) + sub + 4 * (q & 7));
            }
            unsigned first = min(kf, __shfl_xor_sync(0xffffffffu, kf, 1));
            first = min(first, __shfl_xor_sync(0xffffffffu, first, 2));
            if (act && first != 0xFFFFFFFFu && kf == first) {
              const float* st = first >= unsigned(kFBK) ? st1 : st0;
              const int kk = int(first) & (kFBK - 1);
              const float v = Op::mul(st[ring_a(lr, kk)], st[ring_b(kk, lc)]);
              const int64_t gofs = (m0 + lr) * p.ldc + (n0 + lc);
              store_c(C, gofs, v);
              IDX[gofs] = int32_t((second ? t0b : t0) * kFBK + first) + p.k_offset;
            }
          }
        }
        seq0 = need2;
        c = c2;
        continue;
      }
    }
    const int64_t need = seq0 + nt;
    if (issued < need) {   // chunks longer than two tiles: make room, then issue the rest
      __syncthreads();
      issue_until(need);
    }
    bool landed = true;
    if (tma) {
      for (int64_t q = seq0; q < need; ++q)
        landed = mbar_wait(bars + 8 * uint32_t(q % kRStages), uint32_t((q / kRStages) & 1)) && landed;
    } else {
      const int64_t pending = issued - need;   // groups allowed to stay in flight
      if (pending >= 4) cp_async_wait<4>();
      else if (pending == 3) cp_async_wait<3>();
      else if (pending == 2) cp_async_wait<2>();
      else if (pending == 1) cp_async_wait<1>();
      else cp_async_wait<0>();
    }
    __syncthreads();
    if (!__syncthreads_and(landed)) {   // a copy never arrived: mark the chunk's outputs, stop
      for (int e = off[c] + tid; e < off[c + 1]; e += kFThreads) {
        const int o = list[e];
        IDX[(m0 + (o >> 7)) * p.ldc + (n0 + (o & 127))] = -2;
      }
      return;
    }
    // every thread is past the previous chunk: its ring slots may be refilled
    issue_until(seq0 + kRStages);
    const int beg = off[c], end = off[c + 1];
    const int slot0 = int(seq0 % kRStages);
    const int klast = int(i64min(kFBK, p.k - (t0 + nt - 1) * kFBK));   // valid k in the chunk's last tile
    // 64 groups of 4 lanes; lane `sub` owns k = sub, sub+4, ..., sub+28 of
    // every tile of the chunk.  Pass 1: group max of the products; pass 2:
    // lowest k whose product equals it.  Trip counts are block-uniform, so
    // every lane reaches the shuffles.  Each group handles two entries per
    // round (independent chains for ILP); the products of pass 1 stay in
    // registers for pass 2.
    if (nt == 2 && klast == kFBK) {
      // Full two-tile chunk: no k-range masks; pass 1 is a max3 tree, pass 2
      // a 16-bit equality mask whose lowest set bit is the lane's first
      // winning k (bit order = k order).
      const float* st0 = smem + slot0 * kRStageFloats;
      const float* st1 = smem + (slot0 + 1 >= kRStages ? slot0 + 1 - kRStages : slot0 + 1) * kRStageFloats;
      for (int e0 = beg; e0 < end; e0 += 2 * (kFThreads / 4)) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int e = e0 + u * (kFThreads / 4) + grp;
          const bool act = e < end;
          const int o = act ? list[e] : 0;
          const int lr = o >> 7, lc = o & 127;
          float pv[16];
          chunk_products<S>(st0, st1, lr, lc, sub, pv);
          float m = Op::red3(Op::red3(Op::red3(pv[0], pv[1], pv[2]), Op::red3(pv[3], pv[4], pv[5]),
                                      Op::red3(pv[6], pv[7], pv[8])),
                             Op::red3(Op::red3(pv[9], pv[10], pv[11]), Op::red3(pv[12], pv[13], pv[14]), pv[15]),
                             pv[15]);
          float x = __shfl_xor_sync(0xffffffffu, m, 1);
          m = Op::red3(m, x, x);
          x = __shfl_xor_sync(0xffffffffu, m, 2);
          m = Op::red3(m, x, x);
          unsigned mask = 0;
#pragma unroll
          for (int q = 0; q < 16; ++q) mask |= (pv[q] == m) ? (1u << q) : 0u;
          unsigned kf = 0xFFFFFFFFu;
          if (mask) {
            const int q = __ffs(mask) - 1;
            kf = unsigned(32 * (q >> 3) + sub + 4 * (q & 7));
          }
          unsigned first = min(kf, __shfl_xor_sync(0xffffffffu, kf, 1));
          first = min(first, __shfl_xor_sync(0xffffffffu, first, 2));
          if (act && first != 0xFFFFFFFFu && kf == first) {
            const float* st = first >= unsigned(kFBK) ? st1 : st0;
            const int kk = int(first) & (kFBK - 1);
            const float v = Op::mul(st[ring_a(lr, kk)], st[ring_b(kk, lc)]);
            const int64_t gofs = (m0 + lr) * p.ldc + (n0 + lc);
            store_c(C, gofs, v);
            IDX[gofs] = int32_t(t0 * kFBK + first) + p.k_offset;
          }
        }
      }
      seq0 = need;
      continue;
    }
    constexpr int kE = 2;
    for (int e0 = beg; e0 < end; e0 += kE * (kFThreads / 4)) {
      int o[kE];
      bool active[kE];
      float pr[kE][4][8];
      float best[kE];
#pragma unroll
      for (int u = 0; u < kE; ++u) {
        const int e = e0 + u * (kFThreads / 4) + grp;
        active[u] = e < end;
        o[u] = active[u] ? list[e] : 0;
        best[u] = Op::zero();
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (j < nt) {
          const int slot = slot0 + j >= kRStages ? slot0 + j - kRStages : slot0 + j;
          const float* st = smem + slot * kRStageFloats;
          const int kc = j == nt - 1 ? klast : kFBK;
#pragma unroll
          for (int u = 0; u < kE; ++u) {
            const int lr = o[u] >> 7, lc = o[u] & 127;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              pr[u][j][i] = Op::mul(st[ring_a(lr, sub + 4 * i)], st[ring_b(sub + 4 * i, lc)]);
              if (sub + 4 * i < kc && Op::better(pr[u][j][i], best[u])) best[u] = pr[u][j][i];
            }
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kE; ++u)
#pragma unroll
        for (int d = 1; d < 4; d <<= 1) {
          const float other = __shfl_xor_sync(0xffffffffu, best[u], d);
          if (Op::better(other, best[u])) best[u] = other;
        }
      unsigned cand[kE], first[kE];
      float cp[kE];
#pragma unroll
      for (int u = 0; u < kE; ++u) { cand[u] = 0xFFFFFFFFu; cp[u] = 0.f; }
#pragma unroll
      for (int j = 3; j >= 0; --j) {
        if (j < nt) {
          const int kc = j == nt - 1 ? klast : kFBK;
#pragma unroll
          for (int u = 0; u < kE; ++u)
#pragma unroll
            for (int i = 7; i >= 0; --i)
              if (sub + 4 * i < kc && pr[u][j][i] == best[u]) {
                cand[u] = unsigned(j * kFBK + sub + 4 * i);
                cp[u] = pr[u][j][i];
              }
        }
      }
#pragma unroll
      for (int u = 0; u < kE; ++u) {
        first[u] = cand[u];
#pragma unroll
        for (int d = 1; d < 4; d <<= 1) first[u] = min(first[u], __shfl_xor_sync(0xffffffffu, first[u], d));
        if (active[u] && first[u] != 0xFFFFFFFFu && cand[u] == first[u]) {
          const int64_t gofs = (m0 + (o[u] >> 7)) * p.ldc + (n0 + (o[u] & 127));
          store_c(C, gofs, cp[u]);
          IDX[gofs] = int32_t(t0 * kFBK + first[u]) + p.k_offset;
        }
      }
    }
    seq0 = need;
  }
  cp_async_wait<0>();
}

}  // namespace tg
