/*
 * tropical_gemm_b200.h -- C ABI of the B200-native tropical GEMM engine.
 *
 * C = A (x) B over a tropical semiring, optionally with the argmax index of
 * the winning k for every output, plus the argmax-scatter backward pass.
 *
 * Conventions shared by every entry point
 *   - All pointers are device pointers (cudaMalloc / torch CUDA storage),
 *     except where a comment says otherwise.  The library never allocates
 *     outputs: the caller passes C, argmax and gradient buffers.
 *   - `stream` is a cudaStream_t passed as void*; NULL means the legacy
 *     default stream.  Every call is stream-ordered and asynchronous: no
 *     host synchronisation happens inside the library.
 *   - Leading dimensions (lda/ldb/ldc) are in elements.  For TG_ROW_MAJOR
 *     A is M x K with A[i,k] at a[i*lda + k]; for TG_COL_MAJOR A[i,k] is at
 *     a[k*lda + i] (the column-major convention of the reference's Rust
 *     GPU API).  The same layout applies to B, C and argmax.
 *   - argmax is int32 with the same leading dimension as C; NULL selects
 *     the plain (value-only) GEMM.
 *   - Semantics follow the reference bit for bit: k is visited in
 *     ascending order, the accumulator starts at the semiring zero with
 *     index 0, and a product replaces it only when strictly better, so the
 *     lowest k among ties wins and outputs that nothing beats keep index 0.
 *     Integer MaxPlus/MinPlus use the sentinels -46340/+46340 (i32) and
 *     -3037000499/+3037000499 (i64) with the reference's saturating add.
 *   - Return value: TG_OK or an error code; tg_last_error() gives a
 *     human-readable message for the calling thread.
 */
#ifndef TROPICAL_GEMM_B200_H
#define TROPICAL_GEMM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum { TG_MAXPLUS = 0, TG_MINPLUS = 1, TG_MAXMUL = 2 } tg_semiring;
typedef enum { TG_F32 = 0, TG_F64 = 1, TG_I32 = 2, TG_I64 = 3 } tg_dtype;
typedef enum { TG_ROW_MAJOR = 0, TG_COL_MAJOR = 1 } tg_layout;

typedef enum {
  TG_OK = 0,
  TG_ERR_INVALID_ARGUMENT = 1,  /* null pointer, negative size, bad enum   */
  TG_ERR_DIMENSION_MISMATCH = 2,/* leading dimension too small, etc.       */
  TG_ERR_UNSUPPORTED = 3,       /* combination not provided (e.g. int grad) */
  TG_ERR_CUDA = 4,              /* a CUDA runtime call failed              */
  TG_ERR_NO_DEVICE = 5          /* no CUDA device visible                  */
} tg_status;

/* Library version string, e.g. "0.2.0-b200". */
const char* tg_version(void);

/* Message describing the last failing call on this thread ("" if none). */
const char* tg_last_error(void);

/* Number of visible CUDA devices (0 when none); never fails.
 * Replaces cuda_device_count (crates/tropical-gemm-cuda/src/lib.rs:63). */
int tg_device_count(void);

/* C = A (x) B, optionally with argmax.
 * Replaces CudaKernel::launch_gemm and CudaKernelWithArgmax::launch_gemm_with_argmax
 * (crates/tropical-gemm-cuda/src/kernels.rs:22-27, :202-207), the free functions
 * tropical_matmul_gpu[_with_argmax] / tropical_gemm_gpu[_with_argmax]
 * (crates/tropical-gemm-cuda/src/lib.rs:221, :256, :354, :392), and the DLPack
 * launchers launch_gemm_external[_with_argmax]_f32 (kernels.rs:388-473).
 * M, N or K equal to 0 is accepted: with K == 0 every output is the semiring
 * zero with index 0; with M or N == 0 nothing is written. */
tg_status tg_gemm(tg_semiring semiring, tg_dtype dtype, tg_layout layout,
                  int64_t m, int64_t n, int64_t k,
                  const void* a, int64_t lda,
                  const void* b, int64_t ldb,
                  void* c, int64_t ldc,
                  int32_t* argmax,
                  void* stream);

/* Strided batched GEMM: for p in [0, batch) computes
 * C[p] = A[p] (x) B[p] with A[p] = a + p*stride_a (elements), etc.;
 * argmax uses stride_c.  One launch for the whole batch.
 * Replaces launch_gemm_external_batched_with_argmax_f32 (kernels.rs:498-550)
 * and tropical_matmul_gpu_strided_batched[_with_argmax]
 * (crates/tropical-gemm-cuda/src/lib.rs:486, :563, :1007). */
tg_status tg_gemm_strided_batched(tg_semiring semiring, tg_dtype dtype, tg_layout layout,
                                  int64_t batch, int64_t m, int64_t n, int64_t k,
                                  const void* a, int64_t lda, int64_t stride_a,
                                  const void* b, int64_t ldb, int64_t stride_b,
                                  void* c, int64_t ldc, int64_t stride_c,
                                  int32_t* argmax,
                                  void* stream);

/* Accumulating f32 GEMM over one K slice: every output starts from its
 * current value in C (and keeps its argmax) unless a product of this slice
 * strictly beats it; a winning k is written as k_offset + k.  Computing
 * K = [0, k1) with tg_gemm and then [k1, k2), ... with this call (A's and
 * B's slices, k_offset = slice start) gives results identical to one
 * tg_gemm over the whole K, so a caller can overlap the transfer of B's next
 * K slice with the arithmetic of the current one.  f32 only (others:
 * TG_ERR_UNSUPPORTED); argmax may be null (values only).  No reference
 * counterpart: the reference computes whole products in one launch
 * (kernels.rs:388-434); this is the building block of the pipelined sharded
 * GEMM. */
tg_status tg_gemm_accumulate(tg_semiring semiring, tg_layout layout,
                             int64_t m, int64_t n, int64_t k,
                             const float* a, int64_t lda,
                             const float* b, int64_t ldb,
                             float* c, int64_t ldc,
                             int32_t* argmax, int32_t k_offset,
                             void* stream);

/* Broadcast callback for tg_sharded_gemm: make the `bytes` bytes of device
 * memory at `buf` equal to rank `root`'s copy, enqueued on `stream` (for
 * example ncclBroadcast on the caller's communicator, so the library links no
 * collective library of its own).  Returns 0 on success. */
typedef int (*tg_broadcast_fn)(void* buf, size_t bytes, int root, void* stream, void* ctx);

/* One rank's part of a row-sharded GEMM across GPUs: B (k x n, row-major,
 * leading dimension ldb, one buffer per rank on its device) is made whole by
 * bcast(b, ..., root, stream, bcast_ctx), then this rank computes its own
 * m_local rows C_local = A_local (x) B (row-major, like tg_gemm with
 * TG_ROW_MAJOR).  C and argmax stay sharded: no reduction.  Every rank must
 * call it (m_local may be 0: the rank still takes part in the broadcast).
 * Column-major callers shard columns instead: pass the transposed problem
 * (B^T rows, A^T broadcast).  No reference counterpart: the reference has no
 * multi-GPU path; this is the sharded entry its CUDA crate would bind for one
 * process per GPU. */
tg_status tg_sharded_gemm(tg_semiring semiring, tg_dtype dtype,
                          int64_t m_local, int64_t n, int64_t k,
                          const void* a_local, int64_t lda,
                          void* b, int64_t ldb,
                          void* c_local, int64_t ldc,
                          int32_t* argmax_local,
                          int root, tg_broadcast_fn bcast, void* bcast_ctx,
                          void* stream);

/* Backward pass w.r.t. A:
 *   grad_a[i, argmax[i,j]] += grad_c[i,j] * w[i,j]
 * where w = 1 for MaxPlus/MinPlus and w = B[argmax[i,j], j] for MaxMul
 * (the multiplicative rule of pytorch.py:521-548; pass b for MaxMul, NULL
 * otherwise).  Indices outside [0, K) are skipped, as in the reference kernel.
 * accumulate == 0 overwrites grad_a (no pre-zeroing needed); != 0 adds into it.
 * Float types only.  Replaces tropical_backward_a_gpu_kernel
 * (crates/tropical-gemm-cuda/src/lib.rs:841-882) and the torch scatter_add_
 * backward (crates/tropical-gemm-python/python/tropical_gemm/pytorch.py:386-403). */
tg_status tg_backward_a(tg_semiring semiring, tg_dtype dtype, tg_layout layout,
                        int64_t batch, int64_t m, int64_t n, int64_t k,
                        const void* grad_c, int64_t ldc, int64_t stride_c,
                        const int32_t* argmax,
                        const void* b, int64_t ldb, int64_t stride_b,
                        void* grad_a, int64_t lda, int64_t stride_a,
                        int accumulate, void* stream);

/* Backward pass w.r.t. B:
 *   grad_b[argmax[i,j], j] += grad_c[i,j] * w[i,j]
 * with w = 1, or A[i, argmax[i,j]] for MaxMul (pass a).  Same conventions
 * as tg_backward_a.  Replaces tropical_backward_b_gpu_kernel
 * (crates/tropical-gemm-cuda/src/lib.rs:901-942). */
tg_status tg_backward_b(tg_semiring semiring, tg_dtype dtype, tg_layout layout,
                        int64_t batch, int64_t m, int64_t n, int64_t k,
                        const void* grad_c, int64_t ldc, int64_t stride_c,
                        const int32_t* argmax,
                        const void* a, int64_t lda, int64_t stride_a,
                        void* grad_b, int64_t ldb, int64_t stride_b,
                        int accumulate, void* stream);

/* Integer (i32) C = A (x) B, optionally with argmax, that allocates nothing.
 * No counterpart in the reference: it is an addition of this library.
 * For callers that cannot allocate device memory at call time -- e.g. a host
 * framework that has reserved the GPU's memory for its own pool, or a
 * serving / real-time loop that forbids cudaMalloc after start-up because an
 * allocation can block, fail or synchronise.  Same arguments and results as
 * tg_gemm with dtype TG_I32 (one matrix, no batch).  Its scratch (A and B as
 * f32, rows padded to 4 elements, plus a 256-byte header) lives in a fixed
 * 64 MiB device array that every GPU loading this library keeps until the
 * process exits; larger problems are rejected with TG_ERR_UNSUPPORTED and a
 * message (use tg_gemm for them).  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress); make that first call before
 * any stream capture.  All calls share the one array and it keeps the last
 * call's contents: calls that overlap on the GPU (different streams, or
 * different host threads on the same device) race and must be serialised by
 * the caller. */
tg_status tg_gemm_i32_noalloc(tg_semiring semiring, tg_layout layout,
                              int64_t m, int64_t n, int64_t k,
                              const void* a, int64_t lda,
                              const void* b, int64_t ldb,
                              void* c, int64_t ldc,
                              int32_t* argmax,
                              void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TROPICAL_GEMM_B200_H */
