// C ABI of the engine: validation, layout mapping, error state and the
// per-device configuration.  Declarations and per-function contracts live in
// include/tropical_gemm_b200.h; the kernel dispatch is in tg_dispatch.cuh.
//
// Host-side responsibilities (the reference's cu/src/{kernels,lib}.rs):
//  * shape / leading-dimension / pointer checks with error codes instead
//    of Rust `Result`s (crates/tropical-gemm-cuda/src/error.rs:8-29);
//  * column-major callers become the canonical row-major problem
//    C^T = B^T (x) A^T by swapping operands and M <-> N -- the same trick
//    the reference applies for row-major DLPack tensors (kernels.rs:416-430),
//    here in the opposite direction;
//  * stream-ordered launches only: no synchronisation.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <algorithm>
#include <mutex>
#include <set>
#include <utility>
#include <cuda_runtime.h>
#include "../../include/tropical_gemm_b200.h"
#include "tg_internal.h"
#include "tg_semiring.cuh"
#include "tg_fast_f32.cuh"

namespace {
thread_local std::string g_last_error;
}  // namespace

namespace tgi {

tg_status fail(tg_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return s;
}

void clear_error() { g_last_error.clear(); }

tg_status check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(TG_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return TG_OK;
}

bool fast_f32_ok(const Problem& P) {
  const auto& g = P.g;
  // any A alignment: the kernel switches to 4-byte copies for unaligned rows
  if (g.k >= (int64_t(1) << 31)) return false;
  // argmax: the re-stream ring holds whole chunks of <= 4 k-tiles (1024 chunks)
  if (g.argmax && (g.k + tg::kFBK - 1) / tg::kFBK > int64_t(4) * tg::kFMaxChunks) return false;
  return true;
}

// Per-device launch configuration, set up once per (device, kernel) under a
// lock: the dynamic shared-memory opt-in, the SM count, the scratch pool.
std::mutex g_cfg_mu;
std::set<std::pair<int, const void*>> g_cfg_done;
int g_sm_count[64] = {0};

tg_status ensure_smem(const void* kern, size_t smem) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(TG_ERR_NO_DEVICE, "no current CUDA device");
  std::lock_guard<std::mutex> lock(g_cfg_mu);
  if (g_cfg_done.count({dev, kern})) return TG_OK;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return fail(TG_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  g_cfg_done.insert({dev, kern});
  return TG_OK;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

bool encode_tma_f32(const void* base, int64_t inner, int64_t rows, int64_t ld, int64_t batch, int64_t bstride,
                    uint32_t box_inner, uint32_t box_rows, CUtensorMap* out, bool swizzle) {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
    cudaGetLastError();
  });
  if (!fn) return false;
  const cuuint64_t dims[3] = {cuuint64_t(inner), cuuint64_t(rows), cuuint64_t(batch)};
  const cuuint64_t strides[2] = {cuuint64_t(ld) * 4, cuuint64_t(batch > 1 ? bstride : ld * rows) * 4};
  const cuuint32_t box[3] = {box_inner, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int kernel_regs(const void* kern) {
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return fa.numRegs;
}

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_cfg_mu);
  if (dev < 0 || dev >= 64) return 148;
  if (!g_sm_count[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      return 148;
    }
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

// Stream-ordered scratch comes from a memory pool the library creates on
// each device (never the device's default pool, whose settings belong to
// the application).  Its release threshold is 4 GiB, so freed scratch stays
// mapped for the next call instead of going back to the OS at every
// synchronisation (an i32 call at 4096^3: 7.6 -> 6.3 ms; the two copies of B
// the fused argmax kernel takes at N = 32768, K = 8192 are 2 GiB).
cudaMemPool_t g_pool[64] = {};

cudaError_t scratch_alloc(void** p, size_t bytes, cudaStream_t st) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  cudaMemPool_t pool;
  {
    std::lock_guard<std::mutex> lock(g_cfg_mu);
    if (!g_pool[dev]) {
      cudaMemPoolProps props;
      std::memset(&props, 0, sizeof(props));
      props.allocType = cudaMemAllocationTypePinned;
      props.handleTypes = cudaMemHandleTypeNone;
      props.location.type = cudaMemLocationTypeDevice;
      props.location.id = dev;
      cudaMemPool_t np;
      e = cudaMemPoolCreate(&np, &props);
      if (e != cudaSuccess) return e;
      uint64_t thr = uint64_t(4) << 30;
      cudaMemPoolSetAttribute(np, cudaMemPoolAttrReleaseThreshold, &thr);
      g_pool[dev] = np;
    }
    pool = g_pool[dev];
  }
  return cudaMallocFromPoolAsync(p, bytes, pool, st);
}

void scratch_free(void* p, cudaStream_t st) { cudaFreeAsync(p, st); }

size_t dtype_size(tg_dtype t) {
  switch (t) {
    case TG_F32: case TG_I32: return 4;
    case TG_F64: case TG_I64: return 8;
  }
  return 0;
}

tg_status gemm_impl(tg_semiring semiring, tg_dtype dtype, tg_layout layout, int64_t batch,
                    int64_t m, int64_t n, int64_t k, const void* a, int64_t lda, int64_t sa,
                    const void* b, int64_t ldb, int64_t sb, void* c, int64_t ldc, int64_t sc,
                    int32_t* argmax, void* stream) {
  clear_error();
  if (semiring < TG_MAXPLUS || semiring > TG_MAXMUL) return fail(TG_ERR_INVALID_ARGUMENT, "unknown semiring %d", int(semiring));
  if (dtype_size(dtype) == 0) return fail(TG_ERR_INVALID_ARGUMENT, "unknown dtype %d", int(dtype));
  if (layout != TG_ROW_MAJOR && layout != TG_COL_MAJOR) return fail(TG_ERR_INVALID_ARGUMENT, "unknown layout %d", int(layout));
  if (batch < 0 || m < 0 || n < 0 || k < 0) return fail(TG_ERR_INVALID_ARGUMENT, "negative size (batch=%lld m=%lld n=%lld k=%lld)", (long long)batch, (long long)m, (long long)n, (long long)k);
  if (batch == 0 || m == 0 || n == 0) return TG_OK;
  if (!c) return fail(TG_ERR_INVALID_ARGUMENT, "C is null");
  if (k > 0 && (!a || !b)) return fail(TG_ERR_INVALID_ARGUMENT, "A or B is null");
  if (k >= (int64_t(1) << 31)) return fail(TG_ERR_UNSUPPORTED, "K=%lld exceeds the int32 argmax range", (long long)k);
  // Leading-dimension checks in the caller's layout.
  const bool row = layout == TG_ROW_MAJOR;
  const int64_t need_lda = row ? k : m, need_ldb = row ? n : k, need_ldc = row ? n : m;
  if (k > 0 && lda < std::max<int64_t>(1, need_lda)) return fail(TG_ERR_DIMENSION_MISMATCH, "lda=%lld < %lld", (long long)lda, (long long)need_lda);
  if (k > 0 && ldb < std::max<int64_t>(1, need_ldb)) return fail(TG_ERR_DIMENSION_MISMATCH, "ldb=%lld < %lld", (long long)ldb, (long long)need_ldb);
  if (ldc < std::max<int64_t>(1, need_ldc)) return fail(TG_ERR_DIMENSION_MISMATCH, "ldc=%lld < %lld", (long long)ldc, (long long)need_ldc);
  if (batch > 1 && (sa < 0 || sb < 0 || sc < 0)) return fail(TG_ERR_INVALID_ARGUMENT, "negative batch stride");

  Problem P;
  P.batch = batch;
  if (row) {
    P.g = tg::GemmArgs{m, n, k, a, lda, sa, b, ldb, sb, c, ldc, sc, argmax};
  } else {  // C^T (N x M, row-major, ldc) = B^T (N x K, ldb) (x) A^T (K x M, lda)
    P.g = tg::GemmArgs{n, m, k, b, ldb, sb, a, lda, sa, c, ldc, sc, argmax};
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (semiring) {
    case TG_MAXPLUS: return dispatch<tg::kMaxPlus>(dtype, P, st);
    case TG_MINPLUS: return dispatch<tg::kMinPlus>(dtype, P, st);
    case TG_MAXMUL: return dispatch<tg::kMaxMul>(dtype, P, st);
  }
  return fail(TG_ERR_INVALID_ARGUMENT, "unknown semiring %d", int(semiring));
}

}  // namespace tgi

using namespace tgi;

extern "C" {

const char* tg_version(void) { return "0.2.0-b200"; }
const char* tg_last_error(void) { return g_last_error.c_str(); }

int tg_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) { cudaGetLastError(); return 0; }
  return n;
}

tg_status tg_gemm(tg_semiring semiring, tg_dtype dtype, tg_layout layout, int64_t m, int64_t n, int64_t k,
                  const void* a, int64_t lda, const void* b, int64_t ldb, void* c, int64_t ldc,
                  int32_t* argmax, void* stream) {
  return gemm_impl(semiring, dtype, layout, 1, m, n, k, a, lda, 0, b, ldb, 0, c, ldc, 0, argmax, stream);
}

tg_status tg_gemm_strided_batched(tg_semiring semiring, tg_dtype dtype, tg_layout layout, int64_t batch,
                                  int64_t m, int64_t n, int64_t k, const void* a, int64_t lda, int64_t stride_a,
                                  const void* b, int64_t ldb, int64_t stride_b, void* c, int64_t ldc,
                                  int64_t stride_c, int32_t* argmax, void* stream) {
  return gemm_impl(semiring, dtype, layout, batch, m, n, k, a, lda, stride_a, b, ldb, stride_b, c, ldc, stride_c,
                   argmax, stream);
}

tg_status tg_backward_a(tg_semiring semiring, tg_dtype dtype, tg_layout layout, int64_t batch, int64_t m, int64_t n,
                        int64_t k, const void* grad_c, int64_t ldc, int64_t stride_c, const int32_t* argmax,
                        const void* b, int64_t ldb, int64_t stride_b, void* grad_a, int64_t lda, int64_t stride_a,
                        int accumulate, void* stream) {
  return backward_impl(true, semiring, dtype, layout, batch, m, n, k, grad_c, ldc, stride_c, argmax, b, ldb, stride_b,
                       grad_a, lda, stride_a, accumulate, stream);
}

tg_status tg_backward_b(tg_semiring semiring, tg_dtype dtype, tg_layout layout, int64_t batch, int64_t m, int64_t n,
                        int64_t k, const void* grad_c, int64_t ldc, int64_t stride_c, const int32_t* argmax,
                        const void* a, int64_t lda, int64_t stride_a, void* grad_b, int64_t ldb, int64_t stride_b,
                        int accumulate, void* stream) {
  return backward_impl(false, semiring, dtype, layout, batch, m, n, k, grad_c, ldc, stride_c, argmax, a, lda, stride_a,
                       grad_b, ldb, stride_b, accumulate, stream);
}

tg_status tg_gemm_accumulate(tg_semiring semiring, tg_layout layout, int64_t m, int64_t n, int64_t k, const float* a,
                             int64_t lda, const float* b, int64_t ldb, float* c, int64_t ldc, int32_t* argmax,
                             int32_t k_offset, void* stream) {
  clear_error();
  if (semiring < TG_MAXPLUS || semiring > TG_MAXMUL) return fail(TG_ERR_INVALID_ARGUMENT, "unknown semiring %d", int(semiring));
  if (layout != TG_ROW_MAJOR && layout != TG_COL_MAJOR) return fail(TG_ERR_INVALID_ARGUMENT, "unknown layout %d", int(layout));
  if (m < 0 || n < 0 || k < 0) return fail(TG_ERR_INVALID_ARGUMENT, "negative size (m=%lld n=%lld k=%lld)", (long long)m, (long long)n, (long long)k);
  if (k_offset < 0 || int64_t(k_offset) + k >= (int64_t(1) << 31)) return fail(TG_ERR_INVALID_ARGUMENT, "k_offset %d out of range", int(k_offset));
  if (m == 0 || n == 0 || k == 0) return TG_OK;   // an empty slice changes nothing
  if (!c || !a || !b) return fail(TG_ERR_INVALID_ARGUMENT, "null operand");
  const bool row = layout == TG_ROW_MAJOR;
  const int64_t need_lda = row ? k : m, need_ldb = row ? n : k, need_ldc = row ? n : m;
  if (lda < need_lda) return fail(TG_ERR_DIMENSION_MISMATCH, "lda=%lld < %lld", (long long)lda, (long long)need_lda);
  if (ldb < need_ldb) return fail(TG_ERR_DIMENSION_MISMATCH, "ldb=%lld < %lld", (long long)ldb, (long long)need_ldb);
  if (ldc < need_ldc) return fail(TG_ERR_DIMENSION_MISMATCH, "ldc=%lld < %lld", (long long)ldc, (long long)need_ldc);
  Problem P;
  P.batch = 1;
  P.g = row ? tg::GemmArgs{m, n, k, a, lda, 0, b, ldb, 0, c, ldc, 0, argmax}
            : tg::GemmArgs{n, m, k, b, ldb, 0, a, lda, 0, c, ldc, 0, argmax};
  P.g.accumulate = 1;
  P.g.k_offset = k_offset;
  if (!fast_f32_ok(P)) return fail(TG_ERR_UNSUPPORTED, "K=%lld is beyond the accumulating kernel's range", (long long)k);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (semiring) {
    case TG_MAXPLUS: return dispatch<tg::kMaxPlus>(TG_F32, P, st);
    case TG_MINPLUS: return dispatch<tg::kMinPlus>(TG_F32, P, st);
    default: return dispatch<tg::kMaxMul>(TG_F32, P, st);
  }
}

tg_status tg_sharded_gemm(tg_semiring semiring, tg_dtype dtype, int64_t m_local, int64_t n, int64_t k,
                          const void* a_local, int64_t lda, void* b, int64_t ldb, void* c_local, int64_t ldc,
                          int32_t* argmax_local, int root, tg_broadcast_fn bcast, void* bcast_ctx, void* stream) {
  clear_error();
  if (semiring < TG_MAXPLUS || semiring > TG_MAXMUL) return fail(TG_ERR_INVALID_ARGUMENT, "unknown semiring %d", int(semiring));
  if (dtype < TG_F32 || dtype > TG_I64) return fail(TG_ERR_INVALID_ARGUMENT, "unknown dtype %d", int(dtype));
  if (m_local < 0 || n < 0 || k < 0)
    return fail(TG_ERR_INVALID_ARGUMENT, "negative size (m_local=%lld n=%lld k=%lld)", (long long)m_local, (long long)n,
                (long long)k);
  if (!bcast) return fail(TG_ERR_INVALID_ARGUMENT, "broadcast callback is null");
  if (root < 0) return fail(TG_ERR_INVALID_ARGUMENT, "negative root rank %d", root);
  // B must reach every rank even when this rank owns no rows
  if (k > 0 && n > 0) {
    if (!b) return fail(TG_ERR_INVALID_ARGUMENT, "B is null");
    if (ldb < n) return fail(TG_ERR_DIMENSION_MISMATCH, "ldb=%lld < n=%lld", (long long)ldb, (long long)n);
    const size_t elem = (dtype == TG_F64 || dtype == TG_I64) ? 8 : 4;
    const size_t bytes = (size_t(k - 1) * size_t(ldb) + size_t(n)) * elem;
    const int rc = bcast(b, bytes, root, stream, bcast_ctx);
    if (rc != 0) return fail(TG_ERR_CUDA, "broadcast callback failed (code %d)", rc);
  }
  return tg_gemm(semiring, dtype, TG_ROW_MAJOR, m_local, n, k, a_local, lda, b, ldb, c_local, ldc, argmax_local,
                 stream);
}

}  // extern "C"

// --------------------------------------------------------------------------
// Allocation-free variant of the i32 GEMM.
//
// Some callers cannot allocate device memory at call time: a host framework
// that has already reserved the GPU's memory for its own pool, or a serving
// or real-time loop that forbids cudaMalloc/cudaMallocAsync after start-up
// (an allocation can block, fail under memory pressure, or synchronise).
// tg_gemm_i32_noalloc gives them the i32 GEMM without any allocation: its
// scratch (the f32 copies of A and B plus the range flag) lives in the
// fixed array below, which every GPU that loads this library keeps for the
// life of the process.
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;   // 64 MiB per device
static __device__ __align__(256) unsigned char tg_noalloc_scratch[kNoAllocScratchBytes];

// Device address of tg_noalloc_scratch, looked up once per device (the
// symbol's host-side name is not a device address).
void* noalloc_scratch_address(int dev, tg_status* st) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  if (dev < 0 || dev >= 64) { *st = fail(TG_ERR_UNSUPPORTED, "device ordinal %d out of range", dev); return nullptr; }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, tg_noalloc_scratch);
    if (e != cudaSuccess) {
      *st = fail(TG_ERR_CUDA, "cudaGetSymbolAddress(tg_noalloc_scratch): %s", cudaGetErrorString(e));
      return nullptr;
    }
    addr[dev] = p;
  }
  *st = TG_OK;
  return addr[dev];
}

}  // namespace

extern "C" tg_status tg_gemm_i32_noalloc(tg_semiring semiring, tg_layout layout, int64_t m, int64_t n, int64_t k,
                                         const void* a, int64_t lda, const void* b, int64_t ldb, void* c,
                                         int64_t ldc, int32_t* argmax, void* stream) {
  clear_error();
  if (semiring < TG_MAXPLUS || semiring > TG_MAXMUL) return fail(TG_ERR_INVALID_ARGUMENT, "unknown semiring %d", int(semiring));
  if (layout != TG_ROW_MAJOR && layout != TG_COL_MAJOR) return fail(TG_ERR_INVALID_ARGUMENT, "unknown layout %d", int(layout));
  if (m < 0 || n < 0 || k < 0) return fail(TG_ERR_INVALID_ARGUMENT, "negative size (m=%lld n=%lld k=%lld)", (long long)m, (long long)n, (long long)k);
  if (m == 0 || n == 0) return TG_OK;
  if (!c) return fail(TG_ERR_INVALID_ARGUMENT, "C is null");
  if (k > 0 && (!a || !b)) return fail(TG_ERR_INVALID_ARGUMENT, "A or B is null");
  const bool row = layout == TG_ROW_MAJOR;
  const int64_t need_lda = row ? k : m, need_ldb = row ? n : k, need_ldc = row ? n : m;
  if (k > 0 && lda < std::max<int64_t>(1, need_lda)) return fail(TG_ERR_DIMENSION_MISMATCH, "lda=%lld < %lld", (long long)lda, (long long)need_lda);
  if (k > 0 && ldb < std::max<int64_t>(1, need_ldb)) return fail(TG_ERR_DIMENSION_MISMATCH, "ldb=%lld < %lld", (long long)ldb, (long long)need_ldb);
  if (ldc < std::max<int64_t>(1, need_ldc)) return fail(TG_ERR_DIMENSION_MISMATCH, "ldc=%lld < %lld", (long long)ldc, (long long)need_ldc);
  Problem P;
  P.batch = 1;
  P.g = row ? tg::GemmArgs{m, n, k, a, lda, 0, b, ldb, 0, c, ldc, 0, argmax}
            : tg::GemmArgs{n, m, k, b, ldb, 0, a, lda, 0, c, ldc, 0, argmax};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (k == 0 || !fast_f32_ok(P)) {   // no scratch needed: semiring zero and index 0, or the exact kernel
    switch (semiring) {
      case TG_MAXPLUS: return dispatch<tg::kMaxPlus>(TG_I32, P, st);
      case TG_MINPLUS: return dispatch<tg::kMinPlus>(TG_I32, P, st);
      default: return dispatch<tg::kMaxMul>(TG_I32, P, st);
    }
  }
  const int64_t lda_f = (P.g.k + 3) & ~int64_t(3), ldb_f = (P.g.n + 3) & ~int64_t(3);
  const double need = 256.0 + 4.0 * (double(P.g.m) * double(lda_f) + double(P.g.k) * double(ldb_f));
  if (need > double(kNoAllocScratchBytes))
    return fail(TG_ERR_UNSUPPORTED,
                "tg_gemm_i32_noalloc: A and B need %.0f bytes of scratch as f32 (rows padded to 4 elements), "
                "more than the fixed %zu-byte scratch; use tg_gemm instead",
                need, kNoAllocScratchBytes);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(TG_ERR_NO_DEVICE, "no current CUDA device");
  tg_status s;
  unsigned char* ws = static_cast<unsigned char*>(noalloc_scratch_address(dev, &s));
  if (!ws) return s;
  switch (semiring) {
    case TG_MAXPLUS: return noalloc_i32<tg::kMaxPlus>(P, st, ws);
    case TG_MINPLUS: return noalloc_i32<tg::kMinPlus>(P, st, ws);
    default: return noalloc_i32<tg::kMaxMul>(P, st, ws);
  }
}
