// f32 tropical GEMM with argmax for long K, persistent, with the argmax
// resolution of one tile fused into the k loop of the next.
//
// What is computed is the chunked kernel's (tg_fast_f32.cuh): the value
// accumulators run free (FADD2 + 3-input max), a strict compare at every
// chunk boundary (every two k-tiles) records the chunk of each output's last
// strict improvement, and the winner -- the reference's first k attaining
// the extreme (tropical_gemm.cu:613-618), with that product's bits -- is the
// first strict extreme of that chunk's products.
//
// How it runs (one CTA of 256 threads per SM):
//  * the CTA walks a contiguous range of tiles, n fastest, so consecutive
//    tiles share their A row panel;
//  * each pipeline stage holds A's k-tile (16-byte cp.async by every
//    thread), B's k-tile (one TMA box of a k-pair-interleaved copy of B) and
//    the previous tile's columns of B for the same k (one TMA box of a
//    transposed copy of B, 128-byte swizzled); both copies are made by one
//    pass over B (copy_b_kernel) before the launch;
//  * while k-tile t of tile i is folded, the outputs of tile i-1 whose
//    chunk is t's are scanned from the same stage -- A is shared because
//    both tiles lie in one row panel -- so the chunk kernel's post-loop
//    re-stream of A and B disappears.  Eight lanes scan one output, four k
//    each, from one 128-byte A row and one 128-byte B^T row (no bank
//    conflicts); a group max and a ballot give the first k of the extreme;
//  * a CTA's last tile, and a tile followed by one from another row panel,
//    get a drain pass that stages only A and the old B columns and scans.
// No TMA multicast.  Every wait on a TMA barrier is bounded: on a timeout
// the kernel stops waiting and marks the outputs it resolves with index -2.
#pragma once

namespace tg {

constexpr int kXStageFloats = kFAStage + 2 * kFBStage;   // A | B (k-pair interleaved) | B_prev^T (128 n x 32 k, swizzled)
constexpr int kXBprev = kFAStage + kFBStage;
constexpr size_t kXOffCid = size_t(kFStages) * kXStageFloats * 4;
constexpr size_t kXOffList = kXOffCid + size_t(kFBM * kFBN) * 2;
constexpr size_t kXOffOff = kXOffList + size_t(kFBM * kFBN) * 2;
constexpr size_t kXOffCnt = kXOffOff + ((size_t(kFMaxChunks + 1) * 2 + 7) & ~size_t(7));
constexpr size_t kXOffBar = (kXOffCnt + size_t(kFMaxChunks + 1) * 4 + 7) & ~size_t(7);   // mbarriers: 8-byte aligned
constexpr size_t kXOffDead = kXOffBar + size_t(kFStages) * 8;                           // set when a TMA wait timed out
constexpr size_t kFSmemFused = kXOffDead + 8;
static_assert(kFSmemFused <= 232448, "fused argmax kernel exceeds shared memory");
static_assert(kXOffBar % 8 == 0 && kXOffCnt % 4 == 0, "barrier / counter alignment");
static_assert((kXStageFloats * 4) % 1024 == 0 && (kFAStage * 4) % 128 == 0 && (kXBprev * 4) % 1024 == 0,
              "TMA destinations");

// Both copies of B the kernel reads, from one pass over B (K x N, ldb, batch
// stride sb) in 32 x 32 blocks staged through shared memory:
//  * il: k-pair-interleaved [K2][np][2] (K2 = ceil(K/2), np >= N a multiple
//    of 4), coalesced float2 stores along n;
//  * bt: transposed [N][kp] (kp >= K a multiple of 4), coalesced along k.
// Everything outside B is zero.  Grid: (ceil(np/32), k blocks, batch).
static __global__ void copy_b_kernel(const float* __restrict__ b, int64_t k, int64_t n, int64_t ldb, int64_t sb,
                                     float* __restrict__ il, int64_t np, float* __restrict__ bt, int64_t kp) {
  __shared__ float blk[32][33];
  const int64_t k2n = (k + 1) / 2;
  const float* bb = b + int64_t(blockIdx.z) * sb;
  float2* ilb = reinterpret_cast<float2*>(il + int64_t(blockIdx.z) * k2n * np * 2);
  float* btb = bt + int64_t(blockIdx.z) * n * kp;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 256 threads: 8 rows per pass
  const int64_t n0 = int64_t(blockIdx.x) * 32;
  for (int64_t k0 = int64_t(blockIdx.y) * 32; k0 < kp; k0 += int64_t(gridDim.y) * 32) {
    for (int r = ty; r < 32; r += 8) {
      const int64_t kk = k0 + r, nn = n0 + tx;
      blk[r][tx] = (kk < k && nn < n) ? bb[kk * ldb + nn] : 0.f;
    }
    __syncthreads();
    for (int r = ty; r < 32; r += 8) {   // transposed: row n0 + r, k = k0 + tx
      const int64_t nn = n0 + r, kk = k0 + tx;
      if (nn < n && kk < kp) btb[nn * kp + kk] = blk[tx][r];
    }
    for (int r = ty; r < 16; r += 8) {   // interleaved: k-pair row k0/2 + r, column n0 + tx
      const int64_t k2 = k0 / 2 + r, c = n0 + tx;
      if (k2 < k2n && c < np) ilb[k2 * np + c] = make_float2(blk[2 * r][tx], blk[2 * r + 1][tx]);
    }
    __syncthreads();
  }
}

struct XTile {
  int64_t batch, m0, n0;
};
__device__ __forceinline__ XTile x_tile(int64_t tau, int64_t tiles_m, int64_t tiles_n) {
  const int64_t per = tiles_m * tiles_n;
  const int64_t b = tau / per, r = tau - b * per;
  const int64_t mt = r / tiles_n;
  return XTile{b, mt * kFBM, (r - mt * tiles_n) * kFBN};
}

// The pass sequence of one CTA: (cur, prv) = (tile folded, tile resolved),
// -1 = none.
struct XPasses {
  int64_t tiles_m, tiles_n, next_tile, t_end, last_tile = -1, cur = -1, prv = -1;
  __device__ __forceinline__ bool advance() {
    if (next_tile < t_end) {
      if (last_tile >= 0) {
        const XTile x = x_tile(last_tile, tiles_m, tiles_n), y = x_tile(next_tile, tiles_m, tiles_n);
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
  }
};

struct FusedArgs {
  GemmArgs p;
  int64_t nbatch;
  float acc_init;
};

template <int S>
__global__ void __launch_bounds__(kFThreads, 1)
fast_f32_argmax_fused_kernel(FusedArgs w, const __grid_constant__ CUtensorMap tm_bil,
                             const __grid_constant__ CUtensorMap tm_bt) {
  using Op = FastOps<S>;
  const GemmArgs& p = w.p;
  if (gated_off(p)) return;
  extern __shared__ __align__(1024) float x_smem[];
  float* smem = x_smem;
  unsigned char* sbytes = reinterpret_cast<unsigned char*>(smem);
  uint16_t* cid = reinterpret_cast<uint16_t*>(sbytes + kXOffCid);
  uint16_t* list = reinterpret_cast<uint16_t*>(sbytes + kXOffList);
  uint16_t* off = reinterpret_cast<uint16_t*>(sbytes + kXOffOff);
  int* cnt = reinterpret_cast<int*>(sbytes + kXOffCnt);
  int* dead = reinterpret_cast<int*>(sbytes + kXOffDead);
  const uint32_t bars = smem_u32(sbytes + kXOffBar);
  const uint32_t sbase = smem_u32(smem);
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int lm = lane >> 3, ln = lane & 7;
  const int wm = warp >> 1, wn = warp & 1;

  XPasses ps;
  ps.tiles_m = (p.m + kFBM - 1) / kFBM;
  ps.tiles_n = (p.n + kFBN - 1) / kFBN;
  const int64_t ntiles = w.nbatch * ps.tiles_m * ps.tiles_n;
  ps.next_tile = int64_t(blockIdx.x) * ntiles / gridDim.x;
  ps.t_end = (int64_t(blockIdx.x) + 1) * ntiles / gridDim.x;
  const int ktiles = int((p.k + kFBK - 1) / kFBK);   // the host keeps K below 2^30
  const int nchunks = (ktiles + 1) / 2;   // the host keeps this within kFMaxChunks
  const int kvalid_last = int(p.k - (ktiles - 1) * kFBK);
  for (int i = tid; i < kFBM * kFBN; i += kFThreads) cid[i] = kNoChunk;
  if (tid == 0) {
    *dead = (sbase & 1023) ? 1 : 0;   // the swizzled TMA destination needs 1024-byte alignment
    for (int s = 0; s < kFStages; ++s) mbar_init(bars + 8 * s, 1);
    fence_proxy_async();
  }
  __syncthreads();

  uint32_t uses[kFStages] = {0, 0, 0};
  // Per-pass load plan, decoded once per pass (not per k-tile): this
  // thread's A source rows, and the TMA coordinates of B and B^T.
  struct Plan {
    const float* a;        // A + batch * sa + (m0 + r0) * lda + kq0 (row r0 = tid / 8 of the copy loop)
    uint32_t rowmask;      // bit e: row r0 + 32 e exists
    int bx, bz, px, pz;    // B_il box (2 n0, batch), B^T box (n0, batch) of the previous tile; bx < 0: no B, px < 0: no B^T
  };
  auto plan = [&](int64_t c, int64_t q) {
    Plan pl;
    const XTile at = x_tile(c >= 0 ? c : (q >= 0 ? q : 0), ps.tiles_m, ps.tiles_n);
    const int r0 = tid >> 3;
    pl.a = static_cast<const float*>(p.a) + at.batch * p.sa + (at.m0 + r0) * p.lda + (tid & 7) * 4;
    pl.rowmask = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (at.m0 + r0 + 32 * e < p.m) pl.rowmask |= 1u << e;
    pl.bx = c >= 0 ? int(2 * at.n0) : -1;
    pl.bz = int(at.batch);
    if (q >= 0) {
      const XTile pq = x_tile(q, ps.tiles_m, ps.tiles_n);
      pl.px = int(pq.n0);
      pl.pz = int(pq.batch);
    } else {
      pl.px = -1;
      pl.pz = 0;
    }
    return pl;
  };
  // Loads of k-tile kt into stage st: A by cp.async (four 16-byte copies per
  // thread, rows r0 + 32 e), B and B^T by TMA on the stage barrier.
  const int kq0 = (tid & 7) * 4;
  const uint32_t a_dst0 = uint32_t(((tid >> 3) * kFApitch + kq0) * 4);
  auto issue = [&](const Plan& pl, int st, int kt) {
    const uint32_t sb = sbase + uint32_t(st) * uint32_t(kXStageFloats * 4);
    const int64_t k0 = int64_t(kt) * kFBK;
    const int64_t rem = p.k - (k0 + kq0);
    const int kbytes = rem >= 4 ? 16 : (rem > 0 ? int(rem) * 4 : 0);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int bytes = (pl.rowmask >> e) & 1 ? kbytes : 0;
      cp_async16(sb + a_dst0 + uint32_t(e * 32 * kFApitch * 4), bytes ? pl.a + 32 * e * p.lda + k0 : p.a, bytes);
    }
    cp_async_commit();
    if (tid == 0 && !*dead) {
      const uint32_t bar = bars + 8 * st;
      fence_proxy_async();   // the stage's earlier generic accesses come first
      mbar_expect_tx(bar, uint32_t((pl.bx >= 0 ? kFBStage * 4 : 0) + (pl.px >= 0 ? kFBStage * 4 : 0)));
      if (pl.bx >= 0)   // k-pair rows [16 kt, 16 kt + 16) x columns [2 n0, 2 n0 + 256) of the interleaved copy
        tma_load3(sb + uint32_t(kFAStage * 4), &tm_bil, pl.bx, int(16 * kt), pl.bz, bar);
      if (pl.px >= 0)   // rows [n0, n0 + 128) x k [k0, k0 + 32) of B^T, 128-byte swizzle (ring_a's layout)
        tma_load3(sb + uint32_t(kXBprev * 4), &tm_bt, int(k0), pl.px, pl.pz, bar);
    }
  };

  float acc[8][8], snap[8][8];
  bool have = ps.advance();
  Plan pl_next = plan(ps.cur, ps.prv);
  if (have) {
#pragma unroll
    for (int s = 0; s < kFStages - 1; ++s)
      if (s < ktiles) issue(pl_next, s, s);
      else cp_async_commit();
  }
  while (have) {
    const int64_t c_cur = ps.cur, c_prv = ps.prv;
    const Plan pl = pl_next;
    const XTile cc = x_tile(c_cur >= 0 ? c_cur : 0, ps.tiles_m, ps.tiles_n);
    const XTile pc = x_tile(c_prv >= 0 ? c_prv : 0, ps.tiles_m, ps.tiles_n);
#pragma unroll
    for (int r = 0; r < 8; ++r)
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        acc[r][c] = w.acc_init;
        snap[r][c] = w.acc_init;
      }
    float* const Cq = static_cast<float*>(p.c) + pc.batch * p.sc + pc.m0 * p.ldc + pc.n0;
    int32_t* const Iq = p.argmax + pc.batch * p.sc + pc.m0 * p.ldc + pc.n0;
    bool deferred = false;   // the load of k-tile t + 1 waits for this step (its stage held k-tile t - 2)
    for (int t = 0; t < ktiles; ++t) {
      const int st = t % kFStages;
      float* stage = smem + st * kXStageFloats;
      cp_async_wait<kFStages - 2>();   // this thread's A copies of stage t have landed
      if (t == ktiles - 1 && kvalid_last < kFBK) {
        // the k tail of A holds the semiring zero: no product there wins
        __syncthreads();
        const int width = kFBK - kvalid_last;
        for (int i = tid; i < kFBM * width; i += kFThreads)
          stage[(i / width) * kFApitch + kvalid_last + i % width] = Op::zero();
      }
      __syncthreads();   // stage t complete (A) and every thread done with the stages it frees
      if (!*dead && !mbar_wait(bars + 8 * st, uses[st] & 1)) *dead = 1;   // after a timeout: no more waits
      ++uses[st];
      // A chunk is two k-tiles (t - 1, t) and is scanned at its second one,
      // so the load that would overwrite k-tile t - 1 is issued a step later.
      const bool chunk_end = (t & 1) || t == ktiles - 1;
      const bool scan = c_prv >= 0 && chunk_end;
      if (deferred) issue(pl, (t + 1) % kFStages, t + 1);
      deferred = scan && (t & 1) && t + 2 < ktiles;
      if (t + 2 < ktiles && !deferred) issue(pl, (t + 2) % kFStages, t + 2);
      else cp_async_commit();
      if (scan) {
        // Resolve the previous tile's outputs of this chunk: eight lanes per
        // output, four k of each k-tile per lane, so each A row and B^T row
        // is one conflict-free 128-byte read; a group extreme and two
        // ballots give the first k attaining it.
        const bool two = t & 1;
        const float* s0 = smem + ((t + kFStages - 1) % kFStages) * kXStageFloats;   // k-tile t - 1
        const int ch = t >> 1;
        const int beg = off[ch], end = off[ch + 1];
        const int32_t kb0 = int32_t(ch) * (2 * kFBK);
        const int grp = lane >> 3, sub = lane & 7;
        const bool dd = *dead;
        for (int e0 = beg; e0 < end; e0 += kFThreads / 8) {   // uniform trip count: the shuffles see every lane
          const int e = e0 + warp * 4 + grp;
          const bool active = e < end;
          const int o = list[active ? e : beg];
          const int lr = o >> 7, lc = o & 127;
          const int ao = lr * kFApitch + 4 * sub, bo = kXBprev + ring_a(lc, 4 * sub);
          const float4 a1 = *reinterpret_cast<const float4*>(stage + ao);
          const float4 b1 = *reinterpret_cast<const float4*>(stage + bo);
          float q0 = Op::zero(), q1 = q0, q2 = q0, q3 = q0;
          if (two) {
            const float4 a0 = *reinterpret_cast<const float4*>(s0 + ao);
            const float4 b0 = *reinterpret_cast<const float4*>(s0 + bo);
            q0 = Op::mul(a0.x, b0.x); q1 = Op::mul(a0.y, b0.y);
            q2 = Op::mul(a0.z, b0.z); q3 = Op::mul(a0.w, b0.w);
          }
          const float r0 = Op::mul(a1.x, b1.x), r1 = Op::mul(a1.y, b1.y);
          const float r2 = Op::mul(a1.z, b1.z), r3 = Op::mul(a1.w, b1.w);
          float m = Op::red3(Op::red3(Op::red3(q0, q1, q2), q3, r0), r1, r2);
          m = Op::red3(m, r3, r3);
#pragma unroll
          for (int d = 4; d >= 1; d >>= 1) {
            const float x = __shfl_xor_sync(0xffffffffu, m, d);
            m = Op::red3(m, x, x);
          }
          const uint32_t bq = (q0 == m ? 1u : 0u) | (q1 == m ? 2u : 0u) | (q2 == m ? 4u : 0u) | (q3 == m ? 8u : 0u);
          const uint32_t br = (r0 == m ? 1u : 0u) | (r1 == m ? 2u : 0u) | (r2 == m ? 4u : 0u) | (r3 == m ? 8u : 0u);
          const uint32_t gq = (__ballot_sync(0xffffffffu, active && bq) >> (grp * 8)) & 0xffu;
          const uint32_t gr = (__ballot_sync(0xffffffffu, active && br) >> (grp * 8)) & 0xffu;
          // first k: k-tile t - 1 before k-tile t, lanes in k order, bits in k order
          const int src = __ffs(gq ? gq : (gr ? gr : 1u)) - 1;
          const uint32_t fb = __shfl_sync(0xffffffffu, gq ? bq : br, grp * 8 + src);
          const int32_t kw = kb0 + (gq || !two ? 0 : kFBK) + 4 * src + __ffs(fb ? fb : 1u) - 1;
          float pw = m;
          if (__any_sync(0xffffffffu, m == 0.f)) {   // the winning product's own zero sign
            const uint32_t mb = gq ? bq : br;
            const int f = __ffs(mb ? mb : 1u) - 1;
            const float pf = gq ? (f == 0 ? q0 : f == 1 ? q1 : f == 2 ? q2 : q3)
                                : (f == 0 ? r0 : f == 1 ? r1 : f == 2 ? r2 : r3);
            pw = __shfl_sync(0xffffffffu, pf, grp * 8 + src);
          }
          if (active && sub == 0) {
            const int64_t go = int64_t(lr) * p.ldc + lc;
            Cq[go] = pw;
            Iq[go] = dd ? -2 : kw;
          }
        }
      }
      if (c_cur >= 0) {
        // (four k at a time per loop trip: a body half the size of the fully
        // unrolled one leaves instruction-cache room for the scan; measured faster)
        tile_math<S, 4>(stage, stage + kFAStage, wm, wn, lm, ln, acc);
        if (chunk_end) {
          // chunk boundary: remember the chunk of each output's latest strict improvement
          const uint16_t chunk = uint16_t(t >> 1);
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
    }
    cp_async_wait<0>();
    __syncthreads();   // every stage and the previous tile's bucket list are free
    have = ps.advance();
    if (have) {   // start the next pass's first stages, then finish this tile
      pl_next = plan(ps.cur, ps.prv);
#pragma unroll
      for (int s = 0; s < kFStages - 1; ++s)
        if (s < ktiles) issue(pl_next, s, s);
        else cp_async_commit();
    }
    if (c_cur < 0) continue;
    float* const Cc = static_cast<float*>(p.c) + cc.batch * p.sc;
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
          Cc[gr * p.ldc + gc] = w.acc_init;
          Ic[gr * p.ldc + gc] = 0;
        }
      }
    }
    // bucket the tile's outputs by chunk: bucket c is list[off[c], off[c+1]);
    // the chunk ids are reset for the next tile
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
}

}  // namespace tg
