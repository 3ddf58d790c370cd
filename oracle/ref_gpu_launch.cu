// Host launchers for the reference's own CUDA kernels, compiled unmodified
// from the reference source tree (REF_CU is its path, given by oracle/Makefile).
//
// TEST INFRASTRUCTURE ONLY: the GPU parity tests and the reference arm of
// bench.py use this to run the reference kernels on the same box; nothing in
// the product links it.  Launch geometry restates
// crates/tropical-gemm-cuda/src/context.rs:125-150 (f32/i32: 64x64 tiles,
// 16x16 threads; f64/i64: 32x32 tiles, 8x8 threads) and the batched grid of
// crates/tropical-gemm-cuda/src/kernels.rs:512-515.  All matrices are
// column-major, as the reference kernels expect.
#include REF_CU
#include <cuda_runtime.h>

#define REF_NAME(S, T, SUF) tropical_##S##_##T##_nn##SUF

extern "C" int ref_gemm(int semiring, int dtype, int with_argmax, int m, int n, int k, const void* a,
                        const void* b, void* c, int* argmax, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  const bool wide = (dtype == 1 || dtype == 3);
  const unsigned tile = wide ? 32u : 64u;
  const unsigned grid = ((unsigned(m) + tile - 1) / tile) * ((unsigned(n) + tile - 1) / tile);
  const dim3 block = wide ? dim3(8, 8) : dim3(16, 16);
#define L(S, T, CT)                                                                                      \
  if (with_argmax)                                                                                       \
    REF_NAME(S, T, _with_argmax)<<<grid, block, 0, st>>>((const CT*)a, (const CT*)b, (CT*)c, argmax, m, n, k); \
  else                                                                                                   \
    REF_NAME(S, T, )<<<grid, block, 0, st>>>((const CT*)a, (const CT*)b, (CT*)c, m, n, k);
#define SEMI(T, CT)                                  \
  switch (semiring) {                                \
    case 0: { L(maxplus, T, CT) break; }             \
    case 1: { L(minplus, T, CT) break; }             \
    case 2: { L(maxmul, T, CT) break; }              \
    default: return -1;                              \
  }
  switch (dtype) {
    case 0: SEMI(f32, float) break;
    case 1: SEMI(f64, double) break;
    case 2: SEMI(i32, int) break;
    case 3: SEMI(i64, long long) break;
    default: return -1;
  }
  return (int)cudaGetLastError();
}

extern "C" int ref_gemm_batched_argmax_f32(int semiring, int batch, int m, int n, int k, const float* a,
                                           const float* b, float* c, int* argmax, int stride_a, int stride_b,
                                           int stride_c, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 grid(((unsigned(m) + 63) / 64) * ((unsigned(n) + 63) / 64), 1, unsigned(batch));
  const dim3 block(16, 16);
  switch (semiring) {
    case 0: tropical_maxplus_f32_nn_batched_with_argmax<<<grid, block, 0, st>>>(a, b, c, argmax, m, n, k, stride_a, stride_b, stride_c); break;
    case 1: tropical_minplus_f32_nn_batched_with_argmax<<<grid, block, 0, st>>>(a, b, c, argmax, m, n, k, stride_a, stride_b, stride_c); break;
    case 2: tropical_maxmul_f32_nn_batched_with_argmax<<<grid, block, 0, st>>>(a, b, c, argmax, m, n, k, stride_a, stride_b, stride_c); break;
    default: return -1;
  }
  return (int)cudaGetLastError();
}

// grad buffers must be zeroed by the caller (the reference allocates zeros).
extern "C" int ref_backward(int want_a, int dtype, const void* grad_c, const int* argmax, void* grad, int m, int n,
                            int k, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned total = unsigned(m) * unsigned(n);
  const unsigned grid = (total + 255) / 256;
  if (dtype == 0) {
    if (want_a) tropical_backward_a_f32<<<grid, 256, 0, st>>>((const float*)grad_c, argmax, (float*)grad, m, n, k);
    else tropical_backward_b_f32<<<grid, 256, 0, st>>>((const float*)grad_c, argmax, (float*)grad, m, n, k);
  } else {
    if (want_a) tropical_backward_a_f64<<<grid, 256, 0, st>>>((const double*)grad_c, argmax, (double*)grad, m, n, k);
    else tropical_backward_b_f64<<<grid, 256, 0, st>>>((const double*)grad_c, argmax, (double*)grad, m, n, k);
  }
  return (int)cudaGetLastError();
}
