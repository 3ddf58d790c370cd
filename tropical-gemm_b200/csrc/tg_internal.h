// Host-side declarations shared by the engine's translation units (not part
// of the C ABI).  tg_api.cu holds the ABI entry points, the error state and
// the per-device configuration; tg_gemm_{maxplus,minplus,maxmul}.cu
// instantiate the kernel dispatch of one semiring each (so they compile in
// parallel); tg_backward.cu holds the backward dispatch.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include "../../include/tropical_gemm_b200.h"
#include "tg_generic.cuh"

namespace tgi {

struct Problem {
  tg::GemmArgs g;
  int64_t batch;
};

// Records a formatted message for tg_last_error() and returns s.
tg_status fail(tg_status s, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
void clear_error();
// TG_ERR_CUDA with the launch error, if the last launch failed.
tg_status check_launch(const char* what);
// Dynamic shared-memory opt-in of `kern` on the current device, once.
tg_status ensure_smem(const void* kern, size_t smem);
// SM count of the current device (cached).
int sm_count();
// Stream-ordered scratch from the library's own memory pool on the current
// device (the i32 / i64 conversion copies).
cudaError_t scratch_alloc(void** p, size_t bytes, cudaStream_t st);
void scratch_free(void* p, cudaStream_t st);

bool fast_f32_ok(const Problem& P);

// A 3-D f32 tensor map (inner, rows, batch) with a (box_inner x box_rows x 1)
// box, 128-byte swizzle (or none) and zero fill out of bounds, for TMA loads.
// False when the driver entry point is missing or the layout is not
// encodable (16-byte aligned base and strides are the caller's check).
bool encode_tma_f32(const void* base, int64_t inner, int64_t rows, int64_t ld, int64_t batch, int64_t bstride,
                    uint32_t box_inner, uint32_t box_rows, CUtensorMap* out, bool swizzle = true);
// Registers per thread the kernel launches with (0 when unknown).
int kernel_regs(const void* kern);

// One semiring's dispatch over the four dtypes (canonical row-major problem).
template <int S> tg_status dispatch(tg_dtype dtype, const Problem& P, cudaStream_t st);
// The i32 path of one semiring with its scratch supplied by the caller.
template <int S> tg_status noalloc_i32(const Problem& P, cudaStream_t st, unsigned char* ws);

tg_status backward_impl(bool want_a, tg_semiring semiring, tg_dtype dtype, tg_layout layout,
                        int64_t batch, int64_t m, int64_t n, int64_t k,
                        const void* grad_c, int64_t ldc, int64_t sc, const int32_t* argmax,
                        const void* w, int64_t ldw, int64_t sw,
                        void* grad, int64_t ldg, int64_t sg, int accumulate, void* stream);

}  // namespace tgi
