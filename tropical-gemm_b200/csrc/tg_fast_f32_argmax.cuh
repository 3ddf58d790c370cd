// f32 tropical GEMM with argmax for long K: a persistent kernel whose argmax
// bookkeeping rides inside the k loop of the next tile.
//
// The value accumulator of every output runs free (FADD2 + 3-input max, as
// in the values-only kernel).  At every chunk boundary (tpc k-tiles) one
// strict compare of the running value against the snapshot taken at the
// previous boundary records, in shared memory, the chunk of the output's
// last strict improvement: the chunk holding the first k that attains the
// final value.  The reference's winner (tropical_gemm.cu:613-618: strict
// update, lowest k among ties, index 0 when nothing beats the semiring
// zero) is therefore the first k of that chunk whose product is the chunk's
// extreme, and its value bits are that product's (the sign of a zero
// included).
//
// Resolving it needs the chunk's operands again.  Each CTA walks a
// contiguous range of tiles, n fastest, so consecutive tiles share their A
// row panel.  While tile i streams its k-tiles, every stage also carries the
// B columns of tile i-1 (in natural [k][n] layout), and the outputs of tile
// i-1 bucketed under the chunk being staged are scanned right there, before
// the k-tile's arithmetic: one thread per output, the extreme of the 32
// products and the first k attaining it, the running (value, k) of a chunk
// kept in registers between its k-tiles (in C and argmax for outputs past
// the first 256 of a chunk).  So the operands of a chunk are fetched once
// more for B only, and the scan shares the SM with the next tile's
// arithmetic instead of running after it.  A CTA's last tile, and a tile
// followed by one from another row panel, get a drain pass that stages only
// A and the old B columns and scans.
//
// Shared memory: three stages of [A 128x36 | B 32x128 (k-pair interleaved)
// | B_prev 32x128] floats, one u16 chunk id per output of the current tile,
// the previous tile's outputs bucketed by chunk (u16 list + u16 offsets) and
// the bucket counters: 225,288 bytes, one CTA per SM.
#pragma once

namespace tg {

constexpr int kPStageFloats = kFAStage + 2 * kFBStage;
constexpr int kPBprev = kFAStage + kFBStage;                // B_prev offset in a stage (floats)
constexpr int kFMaxChunks = 1024;
constexpr uint16_t kNoChunk = 0xFFFF;                       // output never beat the semiring zero
constexpr size_t kPOffCid = size_t(kFStages) * kPStageFloats * 4;
constexpr size_t kPOffList = kPOffCid + size_t(kFBM * kFBN) * 2;
constexpr size_t kPOffOff = kPOffList + size_t(kFBM * kFBN) * 2;
constexpr size_t kPOffCnt = kPOffOff + ((size_t(kFMaxChunks + 1) * 2 + 3) & ~size_t(3));
constexpr size_t kFSmemArgmax = kPOffCnt + size_t(kFMaxChunks + 1) * 4;
static_assert(kFSmemArgmax <= 232448, "argmax kernel exceeds shared memory");
static_assert(kFBM * kFBN <= 65535, "u16 bucket offsets");

// Staging of one k-tile of B (32 k x 128 n) in natural layout [k][n]: four
// 16-byte cp.async per thread when B rows are 16-byte aligned, sixteen
// 4-byte ones otherwise; out-of-range elements are zero-filled.
struct BNatLoader {
  const float* base;    // B + n0
  int64_t ldb, k, cols;
  uint32_t dst;         // stage-0 B_prev base
  int tid;
  bool vec;
  __device__ __forceinline__ BNatLoader(const float* B, int64_t ldb_, int64_t n, int64_t k_, int64_t n0, int tid_,
                                        uint32_t smem_b, bool bvec)
      : base(B + n0), ldb(ldb_), k(k_), cols(n - n0), dst(smem_b), tid(tid_), vec(bvec) {}
  __device__ __forceinline__ void load(uint32_t soff, int64_t kt) const {
    const int64_t k0 = kt * kFBK;
    if (vec) {
#pragma unroll
      for (int e = 0; e < (kFBK * kFBN / 4) / kFThreads; ++e) {
        const int lin = tid + e * kFThreads;
        const int kk = lin >> 5, c = (lin & 31) * 4;
        const int64_t rem = cols - c;
        const int bytes = k0 + kk < k ? (rem >= 4 ? 16 : (rem > 0 ? int(rem) * 4 : 0)) : 0;
        cp_async16(dst + soff + uint32_t((kk * kFBN + c) * 4), bytes ? base + (k0 + kk) * ldb + c : base, bytes);
      }
    } else {
#pragma unroll
      for (int e = 0; e < (kFBK * kFBN) / kFThreads; ++e) {
        const int lin = tid + e * kFThreads;
        const int kk = lin >> 7, c = lin & 127;
        const bool ok = k0 + kk < k && c < cols;
        cp_async4(dst + soff + uint32_t((kk * kFBN + c) * 4), ok ? base + (k0 + kk) * ldb + c : base, ok ? 4 : 0);
      }
    }
  }
};

struct TileAt {
  int64_t batch, m0, n0;
};
__device__ __forceinline__ TileAt tile_at(int64_t tau, int64_t tiles_m, int64_t tiles_n) {
  const int64_t per = tiles_m * tiles_n;
  const int64_t b = tau / per, r = tau - b * per;
  const int64_t mt = r / tiles_n;
  return TileAt{b, mt * kFBM, (r - mt * tiles_n) * kFBN};
}

// The extreme of the 32 products of output (lr, lc) over the staged k-tile
// and, when it strictly beats `best`, the first k attaining it (its exact
// bits and index kb + i).
template <int S>
__device__ __forceinline__ void scan_ktile(const float* stage, int lr, int lc, int32_t kb, float& best, int32_t& bk) {
  using Op = FastOps<S>;
  const float* ar = stage + lr * kFApitch;
  const float* bc = stage + kPBprev + lc;
  float pr[kFBK];
#pragma unroll
  for (int q = 0; q < kFBK / 4; ++q) {
    const float4 a4 = *reinterpret_cast<const float4*>(ar + 4 * q);
    pr[4 * q + 0] = Op::mul(a4.x, bc[(4 * q + 0) * kFBN]);
    pr[4 * q + 1] = Op::mul(a4.y, bc[(4 * q + 1) * kFBN]);
    pr[4 * q + 2] = Op::mul(a4.z, bc[(4 * q + 2) * kFBN]);
    pr[4 * q + 3] = Op::mul(a4.w, bc[(4 * q + 3) * kFBN]);
  }
  float m4[4];
#pragma unroll
  for (int g = 0; g < 4; ++g) {   // four independent folds of eight
    float m = Op::red3(pr[8 * g], pr[8 * g + 1], pr[8 * g + 2]);
    m = Op::red3(m, pr[8 * g + 3], pr[8 * g + 4]);
    m4[g] = Op::red3(m, Op::red3(pr[8 * g + 5], pr[8 * g + 6], pr[8 * g + 7]), pr[8 * g + 7]);
  }
  const float m = Op::red3(Op::red3(m4[0], m4[1], m4[2]), m4[3], m4[3]);
  if (Op::better(m, best)) {
    unsigned mask = 0;
#pragma unroll
    for (int i = 0; i < kFBK; ++i) mask |= (pr[i] == m ? 1u : 0u) << i;
    const int f = __ffs(mask) - 1;
    best = Op::mul(ar[f], bc[f * kFBN]);
    bk = kb + f;
  }
}

// One grid of min(#tiles, #SMs) CTAs; CTA b owns tiles [b*T/G, (b+1)*T/G)
// of the batch-major, then m, then n tile order.  tpc: k-tiles per chunk
// (ceil(ktiles / tpc) <= kFMaxChunks).  b_vec: B rows 16-byte aligned.
template <int S, bool OUTI = false, bool AVEC = true>
__global__ void __launch_bounds__(kFThreads, 1)
fast_f32_argmax_kernel(GemmArgs p, int64_t nbatch, int tpc, int b_vec, float acc_init) {
  using Op = FastOps<S>;
  using CT = typename std::conditional<OUTI, int32_t, float>::type;
  if (gated_off(p)) return;
  extern __shared__ __align__(16) float smem[];
  unsigned char* sbytes = reinterpret_cast<unsigned char*>(smem);
  uint16_t* cid = reinterpret_cast<uint16_t*>(sbytes + kPOffCid);
  uint16_t* list = reinterpret_cast<uint16_t*>(sbytes + kPOffList);
  uint16_t* off = reinterpret_cast<uint16_t*>(sbytes + kPOffOff);
  int* cnt = reinterpret_cast<int*>(sbytes + kPOffCnt);
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int lm = lane >> 3, ln = lane & 7;
  const int wm = warp >> 1, wn = warp & 1;

  const int64_t tiles_m = (p.m + kFBM - 1) / kFBM, tiles_n = (p.n + kFBN - 1) / kFBN;
  const int64_t ntiles = nbatch * tiles_m * tiles_n;
  const int64_t G = gridDim.x;
  const int64_t t_end = (int64_t(blockIdx.x) + 1) * ntiles / G;
  int64_t next_tile = int64_t(blockIdx.x) * ntiles / G;
  int64_t last_tile = -1;   // tile whose outputs wait for resolution
  const int64_t ktiles = (p.k + kFBK - 1) / kFBK;
  const int kvalid_last = int(p.k - (ktiles - 1) * kFBK);
  const int nchunks = int((ktiles + tpc - 1) / tpc);
  const uint32_t sbase = smem_u32(smem);
  constexpr uint32_t kStageBytes = uint32_t(kPStageFloats * 4);

  for (int i = tid; i < kFBM * kFBN; i += kFThreads) cid[i] = kNoChunk;

  // Pass sequence: (cur, prv) = (tile computed, tile resolved); -1 = none.
  // A pass always stages A of one row panel (cur's, or prv's in a drain).
  int64_t cur = -1, prv = -1;
  auto advance = [&]() -> bool {
    if (next_tile < t_end) {
      if (last_tile >= 0) {
        const TileAt x = tile_at(last_tile, tiles_m, tiles_n), y = tile_at(next_tile, tiles_m, tiles_n);
        if (x.batch != y.batch || x.m0 != y.m0) {   // another row panel: drain first
          cur = -1;
          prv = last_tile;
          last_tile = -1;
          return true;
        }
      }
      cur = next_tile;
      prv = last_tile;
      last_tile = next_tile;
      ++next_tile;
      return true;
    }
    if (last_tile >= 0) {
      cur = -1;
      prv = last_tile;
      last_tile = -1;
      return true;
    }
    return false;
  };
  // Issues the loads of k-tile kt of pass (c, q) into stage `stage`.
  auto issue = [&](int64_t c, int64_t q, int stage, int64_t kt) {
    const TileAt at = tile_at(c >= 0 ? c : q, tiles_m, tiles_n);
    const uint32_t soff = uint32_t(stage) * kStageBytes;
    const ALoader la(static_cast<const float*>(p.a) + at.batch * p.sa, p.lda, p.m, p.k, at.m0, tid, sbase, AVEC);
    la.load(soff, kt);
    if (c >= 0) {
      const BLoader lb(static_cast<const float*>(p.b) + at.batch * p.sb, p.ldb, p.n, p.k, at.n0, tid,
                       sbase + kFAStage * 4);
      lb.load(soff, kt);
    }
    if (q >= 0) {
      const TileAt pq = tile_at(q, tiles_m, tiles_n);
      const BNatLoader lp(static_cast<const float*>(p.b) + pq.batch * p.sb, p.ldb, p.n, p.k, pq.n0, tid,
                          sbase + kPBprev * 4, b_vec != 0);
      lp.load(soff, kt);
    }
  };

  bool have = advance();
  if (have) {
#pragma unroll
    for (int s = 0; s < kFStages - 1; ++s) {
      if (s < ktiles) issue(cur, prv, s, s);
      cp_async_commit();
    }
  }
  __syncthreads();

  float acc[8][8], snap[8][8];
  int32_t pidx_unused[1][1];
#ifdef TG_EXP_CLK
  long long dbg[4] = {0, 0, 0, 0};
#endif
  while (have) {
    const bool has_cur = cur >= 0, has_prv = prv >= 0;
    const TileAt cc = tile_at(has_cur ? cur : 0, tiles_m, tiles_n);
    const TileAt pc = tile_at(has_prv ? prv : 0, tiles_m, tiles_n);
    // stage loaders of this pass (the tile coordinates change per pass)
    const TileAt at = has_cur ? cc : pc;
    const ALoader la(static_cast<const float*>(p.a) + at.batch * p.sa, p.lda, p.m, p.k, at.m0, tid, sbase, AVEC);
    const BLoader lb(static_cast<const float*>(p.b) + cc.batch * p.sb, p.ldb, p.n, p.k, cc.n0, tid,
                     sbase + kFAStage * 4);
    const BNatLoader lp(static_cast<const float*>(p.b) + pc.batch * p.sb, p.ldb, p.n, p.k, pc.n0, tid,
                        sbase + kPBprev * 4, b_vec != 0);
    CT* const Cp = static_cast<CT*>(p.c) + pc.batch * p.sc;
    int32_t* const Ip = p.argmax + pc.batch * p.sc;
#pragma unroll
    for (int r = 0; r < 8; ++r)
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        acc[r][c] = acc_init;
        snap[r][c] = acc_init;
      }
    float rs_best = Op::zero();   // running (value, k) of this thread's first entry of the chunk
    int32_t rs_k = 0;

    for (int64_t t = 0; t < ktiles; ++t) {
#ifdef TG_EXP_CLK
      long long c0 = clock64();
#endif
      cp_async_wait<kFStages - 2>();
      __syncthreads();
#ifdef TG_EXP_CLK
      long long c1 = clock64();
      if (has_cur && has_prv) dbg[0] += c1 - c0;
#endif
      float* stage = smem + (t % kFStages) * kPStageFloats;
      if (t == ktiles - 1 && kvalid_last < kFBK) {
        fix_k_tail<S>(stage, kvalid_last, tid);
        __syncthreads();
      }
      {
        const int64_t nt = t + kFStages - 1;
        if (nt < ktiles) {
          const uint32_t soff = uint32_t(nt % kFStages) * kStageBytes;
          la.load(soff, nt);
          if (has_cur) lb.load(soff, nt);
#ifndef TG_EXP_NOBP
          if (has_prv) lp.load(soff, nt);
#endif
        }
        cp_async_commit();
      }

#ifndef TG_EXP_NOSCAN
      if (has_prv) {
#else
      if (false) {
#endif
        // Resolve the previous tile's outputs whose chunk is being staged
        // (the staged A columns k >= K hold the semiring zero: no product
        // there beats anything).
        const int c = int(t / tpc);
        const bool first = (t % tpc) == 0;
        const bool last = (t % tpc) == tpc - 1 || t == ktiles - 1;
        const int beg = off[c], end = off[c + 1];
        const int32_t kb = int32_t(t * kFBK);
        for (int e = beg + tid; e < end; e += kFThreads) {
          const bool round0 = e < beg + kFThreads;
          const int o = list[e];
          const int lr = o >> 7, lc = o & 127;
          const int64_t gofs = (pc.m0 + lr) * p.ldc + (pc.n0 + lc);
          float best = Op::zero();
          int32_t bk = 0;
          if (!first) {
            if (round0) {
              best = rs_best;
              bk = rs_k;
            } else {
              best = reinterpret_cast<const float*>(Cp)[gofs];
              bk = Ip[gofs];
            }
          }
          scan_ktile<S>(stage, lr, lc, kb, best, bk);
          if (last) {
            store_c(Cp, gofs, best);
            Ip[gofs] = bk;
          } else if (round0) {
            rs_best = best;
            rs_k = bk;
          } else {
            reinterpret_cast<float*>(Cp)[gofs] = best;
            Ip[gofs] = bk;
          }
        }
      }

#ifdef TG_EXP_CLK
      long long c2 = clock64();
      if (has_cur && has_prv) dbg[1] += c2 - c1;
#endif
      if (has_cur) tile_math<S, false>(stage, wm, wn, lm, ln, acc, pidx_unused, 0);
#ifdef TG_EXP_CLK
      long long c3 = clock64();
      if (has_cur && has_prv) dbg[2] += c3 - c2;
      if (!has_cur) dbg[3] += c3 - c0;
#endif

      if (has_cur && ((t + 1) % tpc == 0 || t == ktiles - 1)) {
        // chunk boundary: remember the chunk of each output's latest strict improvement
        const uint16_t chunk = uint16_t(t / tpc);
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
    __syncthreads();   // every stage and the previous tile's bucket list are free now

    // Start the next pass's first stages, then settle this tile while they land.
    have = advance();
    if (have) {
#pragma unroll
      for (int s = 0; s < kFStages - 1; ++s) {
        if (s < ktiles) issue(cur, prv, s, s);
        cp_async_commit();
      }
    }
    if (!has_cur) continue;

    CT* const Cc = static_cast<CT*>(p.c) + cc.batch * p.sc;
    int32_t* const Ic = p.argmax + cc.batch * p.sc;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int lr = wm * 32 + r * 4 + lm;
      const int64_t gr = cc.m0 + lr;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int lc = wn * 64 + 16 * (c >> 1) + 2 * ln + (c & 1);
        const int64_t gc = cc.n0 + lc;
        if (gr >= p.m || gc >= p.n) {
          cid[lr * kFBN + lc] = kNoChunk;   // padding: never resolved
        } else if (cid[lr * kFBN + lc] == kNoChunk) {   // nothing beat the zero: (zero, index 0)
          store_c(Cc, gr * p.ldc + gc, acc_init);
          Ic[gr * p.ldc + gc] = 0;
        }
      }
    }
    // Bucket this tile's outputs by chunk: bucket c is list[off[c], off[c+1]).
    for (int i = tid; i <= nchunks; i += kFThreads) cnt[i] = 0;
    __syncthreads();
    for (int i = tid; i < kFBM * kFBN; i += kFThreads) {
      const uint16_t ch = cid[i];
      if (ch != kNoChunk) atomicAdd(&cnt[ch + 1], 1);
    }
    __syncthreads();
    if (warp == 0) {  // inclusive scan of the counts
      int carry = 0;
      for (int b0 = 1; b0 <= nchunks; b0 += 32) {
        const int i = b0 + lane;
        int v = i <= nchunks ? cnt[i] : 0;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
          const int u = __shfl_up_sync(0xffffffffu, v, d);
          if (lane >= d) v += u;
        }
        if (i <= nchunks) cnt[i] = v + carry;
        carry += __shfl_sync(0xffffffffu, v, 31);
      }
    }
    __syncthreads();
    for (int i = tid; i <= nchunks; i += kFThreads) off[i] = uint16_t(cnt[i]);
    __syncthreads();
    for (int i = tid; i < kFBM * kFBN; i += kFThreads) {
      const uint16_t ch = cid[i];
      if (ch != kNoChunk) {
        list[atomicAdd(&cnt[ch], 1)] = uint16_t(i);
        cid[i] = kNoChunk;
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
#ifdef TG_EXP_CLK
  // experiment only: per-warp cycle sums (wait+barrier, scan, math, drain) into argmax[]
  if (lane == 0)
    for (int i = 0; i < 4; ++i) p.argmax[(int64_t(blockIdx.x) * 8 + warp) * 4 + i] = int32_t(dbg[i] >> 8);
#endif
}

}  // namespace tg
