// Register-only micro-benchmark of the SIMT instruction forms a tropical
// (max,+) GEMM can be built from on sm_100a.  It is measurement code, not part
// of the engine: bench.py (--case pipe_rates, and every default run) loads it
// to put a measured instruction-mix ceiling beside the pipe-count roofline.
//
// Every variant keeps 64 independent accumulators per thread (the engine's
// 8x8 outputs per thread) and operands in registers, so nothing but issue,
// operand dispatch and pipe throughput limits it.  A "product" is one
// tropical multiply (one add) folded into an accumulator (one max); variants
// that only add or only fold count the operation they perform.  The rate is
// products per clock per SM, from clock64() stamps of each CTA and the SM it
// ran on, so it does not depend on the clock frequency.
#include <cstdint>
#include <vector>
#include <algorithm>
#include <cuda_runtime.h>
#include "../tg_fast_f32.cuh"

namespace {

__device__ __forceinline__ unsigned long long pk(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void upk(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long fadd2(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float fmax2(float a, float b) {
  float r;
  asm("max.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float fadd(float a, float b) {
  float r;
  asm("add.rn.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Variants (products per thread per iteration in brackets):
//  0 pair        FADD2 + FMNMX3 per output and k-pair (the engine's loop)  [128]
//  1 fadd2       FADD2 alone                                               [128]
//  2 fmnmx3      FMNMX3 alone (2 folds each)                               [128]
//  3 fadd        scalar FADD alone                                         [64]
//  4 fmnmx       2-input FMNMX alone                                       [64]
//  5 fadd_fmnmx3 two scalar FADD + one FMNMX3 per output and k-pair        [128]
//  6 fadd2_fmnmx FADD2 + two 2-input FMNMX per output and k-pair           [128]
//  7 fadd_fmnmx  scalar FADD + 2-input FMNMX per product (the reference's
//                value-only form)                                          [64]
//  8, 9          the engine's k-tile body from shared memory (below)
template <int V>
__global__ void __launch_bounds__(256) pipe_kernel(int iters, long long* stamps, float* sink) {
  __shared__ __align__(16) float sm[2048];
  for (int i = threadIdx.x; i < 2048; i += blockDim.x) sm[i] = -1e-3f * float(i % 13 + 1);
  float acc[64];
  const float seed = float(threadIdx.x) * 1e-3f;
#pragma unroll
  for (int i = 0; i < 64; ++i) acc[i] = seed + float(i) * 0.25f;
  unsigned long long B[8];
  float bs[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    bs[q] = -1e-3f * float(q + 1);
    B[q] = pk(bs[q], -2e-3f * float(q + 1));
  }
  float4 pre[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) pre[q] = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncthreads();
  long long t0 = clock64();
  for (int it = 0; it < iters; ++it) {
    if (V >= 15) {
      // variant 0 with the B pairs reloaded from shared memory every
      // iteration: 15 by four 16-byte loads, 16 by eight 8-byte loads,
      // 17 by four 16-byte loads issued one iteration ahead
      const int base = ((it & 7) * 64 + (threadIdx.x & 7) * 4) % 2048;
      float4 bq[4];
      if (V == 15) {
#pragma unroll
        for (int q = 0; q < 4; ++q) bq[q] = *reinterpret_cast<const float4*>(sm + (base + q * 32) % 2048);
      } else if (V == 16) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 x = *reinterpret_cast<const float2*>(sm + (base + q * 32) % 2048);
          const float2 y = *reinterpret_cast<const float2*>(sm + (base + q * 32 + 2) % 2048);
          bq[q] = make_float4(x.x, x.y, y.x, y.y);
        }
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) bq[q] = pre[q];
        const int nb = (((it + 1) & 7) * 64 + (threadIdx.x & 7) * 4) % 2048;
#pragma unroll
        for (int q = 0; q < 4; ++q) pre[q] = *reinterpret_cast<const float4*>(sm + (nb + q * 32) % 2048);
      }
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const unsigned long long A = pk(acc[r * 8], acc[r * 8 + 1]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float lo, hi;
          upk(fadd2(A, pk(bq[q].x, bq[q].y)), lo, hi);
          acc[r * 8 + 2 * q] = fmax3(acc[r * 8 + 2 * q], lo, hi);
          upk(fadd2(A, pk(bq[q].z, bq[q].w)), lo, hi);
          acc[r * 8 + 2 * q + 1] = fmax3(acc[r * 8 + 2 * q + 1], lo, hi);
        }
      }
    } else if (V == 0 || V == 5 || V == 6) {
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const float a0 = acc[r * 8], a1 = acc[r * 8 + 1];
        const unsigned long long A = pk(a0, a1);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          float lo, hi;
          if (V == 5) {
            lo = fadd(a0, bs[c]);
            hi = fadd(a1, bs[(c + 1) & 7]);
          } else {
            upk(fadd2(A, B[c]), lo, hi);
          }
          if (V == 6) acc[r * 8 + c] = fmax2(fmax2(acc[r * 8 + c], lo), hi);
          else acc[r * 8 + c] = fmax3(acc[r * 8 + c], lo, hi);
        }
      }
    } else if (V == 1) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        unsigned long long p = pk(acc[2 * i], acc[2 * i + 1]);
        upk(fadd2(p, B[i & 7]), acc[2 * i], acc[2 * i + 1]);
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        unsigned long long p = pk(acc[2 * i], acc[2 * i + 1]);
        upk(fadd2(p, B[(i + 3) & 7]), acc[2 * i], acc[2 * i + 1]);
      }
    } else if (V == 2) {
#pragma unroll
      for (int i = 0; i < 64; ++i) acc[i] = fmax3(acc[i], bs[i & 7], bs[(i + 1) & 7]);
    } else if (V == 3) {
#pragma unroll
      for (int i = 0; i < 64; ++i) acc[i] = fadd(acc[i], bs[i & 7]);
    } else if (V == 4) {
#pragma unroll
      for (int i = 0; i < 64; ++i) acc[i] = fmax2(acc[i], bs[i & 7]);
    } else if (V == 7) {
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const float a0 = acc[r * 8];
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[r * 8 + c] = fmax2(acc[r * 8 + c], fadd(a0, bs[c]));
      }
    }
  }
  __syncthreads();
  long long t1 = clock64();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 64; ++i) s += acc[i];
  sink[blockIdx.x * blockDim.x + threadIdx.x] = s;
  if (threadIdx.x == 0) {
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    stamps[3 * blockIdx.x] = smid;
    stamps[3 * blockIdx.x + 1] = t0;
    stamps[3 * blockIdx.x + 2] = t1;
  }
}

// Variants 18-22: f64 forms (32 accumulators of 4 rows x 8 columns per
// thread, operands in registers; a product is one f64 add folded into its
// accumulator):
//  18 DADD alone; 19 fmax alone; 20 DADD + fmax (the reference's value-only
//  form); 21 DADD + strict compare-and-select (the engine's f64 fold);
//  22 DADD + compare + value and index selects (the argmax form).
template <int V>
__global__ void __launch_bounds__(256) pipe64_kernel(int iters, long long* stamps, float* sink) {
  double acc[4][8];
  int idx[4][8];
  double a[4], b[8];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    a[r] = -1e-3 * double(r + 1) + 1e-6 * threadIdx.x;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      acc[r][c] = 0.25 * double(r * 8 + c);
      idx[r][c] = 0;
    }
  }
#pragma unroll
  for (int c = 0; c < 8; ++c) b[c] = -2e-3 * double(c + 1);
  __syncthreads();
  long long t0 = clock64();
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const double ar = V == 18 || V == 19 ? 0.0 : acc[r][0] + a[r];   // keeps the chain loop-carried
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        double& x = acc[r][c];
        if (V == 18) {
          x = x + b[c];
        } else if (V == 19) {
          x = fmax(x, b[c] + ar);
        } else {
          const double pr = ar + b[c];
          if (V == 20) x = fmax(x, pr);
          else if (V == 21) x = pr > x ? pr : x;
          else {
            const bool w = pr > x;
            x = w ? pr : x;
            idx[r][c] = w ? it : idx[r][c];
          }
        }
      }
    }
  }
  __syncthreads();
  long long t1 = clock64();
  double sum = 0.0;
  int si = 0;
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      sum += acc[r][c];
      si += idx[r][c];
    }
  sink[blockIdx.x * blockDim.x + threadIdx.x] = float(sum) + float(si);
  if (threadIdx.x == 0) {
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    stamps[3 * blockIdx.x] = smid;
    stamps[3 * blockIdx.x + 1] = t0;
    stamps[3 * blockIdx.x + 2] = t1;
  }
}

// Variants 8 and 9: the engine's own k-tile body (tg::tile_math, MaxPlus,
// values only) over one shared-memory stage that never changes; 9 adds the
// k loop's barrier per k-tile.  Products per iteration: 64 outputs x 32 k.
template <int V>
__global__ void __launch_bounds__(256, 1) body_kernel(int iters, long long* stamps, float* sink) {
  extern __shared__ __align__(16) float stage[];
  for (int i = threadIdx.x; i < tg::kFStageFloats; i += blockDim.x) stage[i] = float((i * 37) % 101) * 0.01f;
  __syncthreads();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float acc[8][8];
#pragma unroll
  for (int r = 0; r < 8; ++r)
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[r][c] = -1e30f;
  long long t0 = clock64();
  for (int it = 0; it < iters; ++it) {
    if (V == 9) __syncthreads();
    tg::tile_math<tg::kMaxPlus>(stage, stage + tg::kFAStage, warp >> 1, warp & 1, lane >> 3, lane & 7, acc);
  }
  __syncthreads();
  long long t1 = clock64();
  float s = 0.f;
#pragma unroll
  for (int r = 0; r < 8; ++r)
#pragma unroll
    for (int c = 0; c < 8; ++c) s += acc[r][c];
  sink[blockIdx.x * blockDim.x + threadIdx.x] = s;
  if (threadIdx.x == 0) {
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    stamps[3 * blockIdx.x] = smid;
    stamps[3 * blockIdx.x + 1] = t0;
    stamps[3 * blockIdx.x + 2] = t1;
  }
}

// Variants 10-12: alternative orders of the same k-tile body (each with the
// barrier per k-tile), to see which operand order the SIMT pipes prefer.
//  10: B pair outer (each B k-pair register pair feeds eight FADD2 in a row)
//  11: two k-pairs per output back to back (two independent FADD2, then two FMNMX3)
//  12: two k-pairs folded by a 3-input max tree (t = max(lo0, hi0, lo1); acc = max(acc, t, hi1))
//  13: B staged as one float4 of four k per column with its two k-pairs swapped,
//      so each FADD2 pairs A's (x,y) with B's (z,w) registers and vice versa
//  14: as 13 without the swap (A's (x,y) with B's (x,y))
//  15-17: variant 0 with its B pairs reloaded from shared memory every
//      iteration (16-byte loads / 8-byte loads / 16-byte loads one iteration ahead)
__device__ __forceinline__ void fadd2s(float& lo, float& hi, float a0, float a1, float b0, float b1) {
  tg::FastOps<tg::kMaxPlus>::pair(lo, hi, a0, a1, b0, b1);
}
__device__ __forceinline__ float mx3(float a, float b, float c) { return tg::FastOps<tg::kMaxPlus>::red3(a, b, c); }

template <int V>
__device__ __forceinline__ void alt_body(const float* stage, int wm, int wn, int lm, int ln, float (&acc)[8][8]) {
  const float* Ap = stage + (wm * 32 + lm) * tg::kFApitch;
  const float* Bp = stage + tg::kFAStage + (wn * 64 + 2 * ln) * 2;
#pragma unroll
  for (int k4 = 0; k4 < tg::kFBK; k4 += 4) {
    float4 a[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) a[r] = *reinterpret_cast<const float4*>(Ap + r * 4 * tg::kFApitch + k4);
    if (V == 13 || V == 14) {
      // one float4 of B per column holding four k (k-pair order swapped for 13),
      // the thread's columns wn*64 + ln + 8c
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float4 b = *reinterpret_cast<const float4*>(stage + tg::kFAStage + ((k4 / 4) * tg::kFBN + wn * 64 + ln + 8 * c) * 4);
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          float l0, h0, l1, h1;
          if (V == 13) {
            fadd2s(l0, h0, a[r].x, a[r].y, b.z, b.w);
            fadd2s(l1, h1, a[r].z, a[r].w, b.x, b.y);
          } else {
            fadd2s(l0, h0, a[r].x, a[r].y, b.x, b.y);
            fadd2s(l1, h1, a[r].z, a[r].w, b.z, b.w);
          }
          acc[r][c] = mx3(mx3(acc[r][c], l0, h0), l1, h1);
        }
      }
    } else if (V == 10) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float4 bq[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) bq[q] = *reinterpret_cast<const float4*>(Bp + (k4 / 2 + h) * (tg::kFBN * 2) + q * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int e = 0; e < 2; ++e)
#pragma unroll
            for (int r = 0; r < 8; ++r) {
              float lo, hi;
              fadd2s(lo, hi, h ? a[r].z : a[r].x, h ? a[r].w : a[r].y, e ? bq[q].z : bq[q].x, e ? bq[q].w : bq[q].y);
              acc[r][2 * q + e] = mx3(acc[r][2 * q + e], lo, hi);
            }
      }
    } else {
      float4 b0[4], b1[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        b0[q] = *reinterpret_cast<const float4*>(Bp + (k4 / 2) * (tg::kFBN * 2) + q * 32);
        b1[q] = *reinterpret_cast<const float4*>(Bp + (k4 / 2 + 1) * (tg::kFBN * 2) + q * 32);
      }
#pragma unroll
      for (int r = 0; r < 8; ++r)
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            float l0, h0, l1, h1;
            fadd2s(l0, h0, a[r].x, a[r].y, e ? b0[q].z : b0[q].x, e ? b0[q].w : b0[q].y);
            fadd2s(l1, h1, a[r].z, a[r].w, e ? b1[q].z : b1[q].x, e ? b1[q].w : b1[q].y);
            if (V == 11) {
              acc[r][2 * q + e] = mx3(mx3(acc[r][2 * q + e], l0, h0), l1, h1);
            } else {
              acc[r][2 * q + e] = mx3(acc[r][2 * q + e], mx3(l0, h0, l1), h1);
            }
          }
    }
  }
}

template <int V>
__global__ void __launch_bounds__(256, 1) alt_kernel(int iters, long long* stamps, float* sink) {
  extern __shared__ __align__(16) float stage[];
  for (int i = threadIdx.x; i < tg::kFStageFloats; i += blockDim.x) stage[i] = float((i * 37) % 101) * 0.01f;
  __syncthreads();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float acc[8][8];
#pragma unroll
  for (int r = 0; r < 8; ++r)
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[r][c] = -1e30f;
  long long t0 = clock64();
  for (int it = 0; it < iters; ++it) {
    __syncthreads();
    alt_body<V>(stage, warp >> 1, warp & 1, lane >> 3, lane & 7, acc);
  }
  __syncthreads();
  long long t1 = clock64();
  float s = 0.f;
#pragma unroll
  for (int r = 0; r < 8; ++r)
#pragma unroll
    for (int c = 0; c < 8; ++c) s += acc[r][c];
  sink[blockIdx.x * blockDim.x + threadIdx.x] = s;
  if (threadIdx.x == 0) {
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    stamps[3 * blockIdx.x] = smid;
    stamps[3 * blockIdx.x + 1] = t0;
    stamps[3 * blockIdx.x + 2] = t1;
  }
}

constexpr int kVariants = 23;
constexpr int kProducts[kVariants] = {128, 128, 128, 64, 64, 128, 128, 64, 64 * tg::kFBK, 64 * tg::kFBK,
                                      64 * tg::kFBK, 64 * tg::kFBK, 64 * tg::kFBK, 64 * tg::kFBK, 64 * tg::kFBK,
                                      128, 128, 128, 32, 32, 32, 32, 32};

template <int V>
cudaError_t launch(int blocks, int threads, int iters, long long* st, float* sink) {
  if constexpr (V >= 18) {
    pipe64_kernel<V><<<blocks, threads>>>(iters, st, sink);
  } else if constexpr (V >= 15) {
    pipe_kernel<V><<<blocks, threads>>>(iters, st, sink);
  } else if constexpr (V >= 10) {
    alt_kernel<V><<<blocks, threads, tg::kFStageFloats * 4>>>(iters, st, sink);
  } else if constexpr (V >= 8) {
    body_kernel<V><<<blocks, threads, tg::kFStageFloats * 4>>>(iters, st, sink);
  } else {
    pipe_kernel<V><<<blocks, threads>>>(iters, st, sink);
  }
  return cudaGetLastError();
}

}  // namespace

extern "C" int tg_probe_variant_count(void) { return kVariants; }

// Runs `variant` with `blocks_per_sm` CTAs of `threads` threads on every SM
// for `iters` iterations; writes products per clock per SM (mean over SMs)
// and the kernel's wall time in ms.  Returns 0 or a CUDA error code.
extern "C" int tg_probe_pipe_rate(int variant, int blocks_per_sm, int threads, int iters, double* per_clk_sm,
                                  double* ms) {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int blocks = sms * blocks_per_sm;
  long long* st = nullptr;
  float* sink = nullptr;
  cudaError_t e = cudaMalloc(&st, sizeof(long long) * 3 * blocks);
  if (e == cudaSuccess) e = cudaMalloc(&sink, sizeof(float) * blocks * threads);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  if (e == cudaSuccess) {
    using L = cudaError_t (*)(int, int, int, long long*, float*);
    const L table[kVariants] = {launch<0>, launch<1>, launch<2>, launch<3>, launch<4>,
                                launch<5>, launch<6>, launch<7>, launch<8>, launch<9>,
                                launch<10>, launch<11>, launch<12>, launch<13>, launch<14>,
                                launch<15>, launch<16>, launch<17>, launch<18>, launch<19>,
                                launch<20>, launch<21>, launch<22>};
    if (variant < 0 || variant >= kVariants) variant = 0;
    const L fn = table[variant];
    e = fn(blocks, threads, 8, st, sink);   // warm-up
    cudaEventRecord(e0);
    if (e == cudaSuccess) e = fn(blocks, threads, iters, st, sink);
    cudaEventRecord(e1);
    if (e == cudaSuccess) e = cudaEventSynchronize(e1);
  }
  if (e == cudaSuccess) {
    float t = 0.f;
    cudaEventElapsedTime(&t, e0, e1);
    *ms = t;
    std::vector<long long> h(3 * blocks);
    e = cudaMemcpy(h.data(), st, sizeof(long long) * 3 * blocks, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) {
      // per SM: products of all its CTAs over the span from the first start to the last end
      std::vector<long long> lo(1024, -1), hi(1024, -1);
      std::vector<int> nb(1024, 0);
      for (int b = 0; b < blocks; ++b) {
        const int sm = int(h[3 * b]) & 1023;
        if (lo[sm] < 0 || h[3 * b + 1] < lo[sm]) lo[sm] = h[3 * b + 1];
        hi[sm] = std::max(hi[sm], h[3 * b + 2]);
        nb[sm]++;
      }
      double sum = 0;
      int used = 0;
      for (int s = 0; s < 1024; ++s)
        if (nb[s]) {
          sum += double(nb[s]) * threads * double(iters) * kProducts[variant] / double(hi[s] - lo[s]);
          ++used;
        }
      *per_clk_sm = used ? sum / used : 0.0;
    }
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaFree(st);
  cudaFree(sink);
  return int(e);
}
