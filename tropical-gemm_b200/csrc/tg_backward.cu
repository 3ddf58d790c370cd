// Backward dispatch: gradient histograms keyed by the forward argmax
// (tg_backward.cuh), with the batch chunked over grid.y.
#include <algorithm>
#include "tg_internal.h"
#include "tg_backward.cuh"

namespace tgi {

template <typename T>
tg_status hist_launch(bool rows_kind, const tg::HistArgs& h, int64_t batch, cudaStream_t st) {
  int dev = 0;
  cudaGetDevice(&dev);
  int max_optin = 0;
  cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const size_t bins = rows_kind ? size_t(h.k) * sizeof(T) : size_t(h.k) * 32 * sizeof(T);
  for (int64_t b0 = 0; b0 < batch; b0 += 65535) {
    const int64_t nb = std::min<int64_t>(65535, batch - b0);
    tg::HistArgs g = h;
    g.gc = static_cast<const T*>(h.gc) + b0 * h.sc;
    g.arg = h.arg + b0 * h.sc;
    if (h.w) g.w = static_cast<const T*>(h.w) + b0 * h.sw;
    g.out = static_cast<T*>(h.out) + b0 * h.so;
    const size_t wbins = size_t(h.k) * sizeof(T) * 8;   // one warp per row, 8 rows per CTA
    if (rows_kind && wbins <= size_t(max_optin) && (h.rows + 7) / 8 <= 0x7fffffff) {
      constexpr int64_t epv = 16 / sizeof(T);
      // 16-byte grad_C loads (and 4 * epv-byte argmax loads) on every row
      const bool vec = (reinterpret_cast<uintptr_t>(g.gc) & 15) == 0 &&
                       (reinterpret_cast<uintptr_t>(g.arg) & (4 * epv - 1)) == 0 && h.cols % epv == 0 &&
                       h.ldc % epv == 0 && (nb == 1 || h.sc % epv == 0);
      auto kern = vec ? tg::hist_rows_warp_kernel<T, true> : tg::hist_rows_warp_kernel<T, false>;
      if (wbins > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(wbins));
      kern<<<dim3(unsigned((h.rows + 7) / 8), unsigned(nb)), 256, wbins, st>>>(g);
    } else if (bins <= size_t(max_optin) && (rows_kind ? h.rows <= 0x7fffffff : (h.cols + 31) / 32 <= 0x7fffffff)) {
      if (rows_kind) {
        auto kern = tg::hist_rows_kernel<T>;
        if (bins > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bins));
        kern<<<dim3(unsigned(h.rows), unsigned(nb)), 256, bins, st>>>(g);
      } else {
        auto kern = tg::hist_cols_kernel<T>;
        if (bins > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bins));
        kern<<<dim3(unsigned((h.cols + 31) / 32), unsigned(nb)), 256, bins, st>>>(g);
      }
    } else {
      const int64_t out_rows = rows_kind ? h.rows : h.k, out_cols = rows_kind ? h.k : h.cols;
      if (!h.accumulate)
        tg::zero_matrix_kernel<T><<<dim3(1024, unsigned(nb)), 256, 0, st>>>(static_cast<T*>(g.out), out_rows, out_cols, h.ldo, h.so);
      if (rows_kind) tg::hist_atomic_kernel<T, true><<<dim3(2048, unsigned(nb)), 256, 0, st>>>(g);
      else tg::hist_atomic_kernel<T, false><<<dim3(2048, unsigned(nb)), 256, 0, st>>>(g);
    }
    tg_status s = check_launch("backward launch");
    if (s != TG_OK) return s;
  }
  return TG_OK;
}

tg_status backward_impl(bool want_a, tg_semiring semiring, tg_dtype dtype, tg_layout layout,
                        int64_t batch, int64_t m, int64_t n, int64_t k,
                        const void* grad_c, int64_t ldc, int64_t sc, const int32_t* argmax,
                        const void* w, int64_t ldw, int64_t sw,
                        void* grad, int64_t ldg, int64_t sg, int accumulate, void* stream) {
  clear_error();
  if (semiring < TG_MAXPLUS || semiring > TG_MAXMUL) return fail(TG_ERR_INVALID_ARGUMENT, "unknown semiring %d", int(semiring));
  if (dtype != TG_F32 && dtype != TG_F64) return fail(TG_ERR_UNSUPPORTED, "backward is defined for f32/f64 only");
  if (layout != TG_ROW_MAJOR && layout != TG_COL_MAJOR) return fail(TG_ERR_INVALID_ARGUMENT, "unknown layout %d", int(layout));
  if (batch < 0 || m < 0 || n < 0 || k < 0) return fail(TG_ERR_INVALID_ARGUMENT, "negative size");
  if (batch == 0 || k == 0) return TG_OK;
  const bool row = layout == TG_ROW_MAJOR;
  // Output dims in caller layout: grad_A is M x K, grad_B is K x N.
  const int64_t g_rows = want_a ? m : k, g_cols = want_a ? k : n;
  if (g_rows == 0 || g_cols == 0) return TG_OK;
  if (!grad) return fail(TG_ERR_INVALID_ARGUMENT, "gradient output is null");
  const bool empty_c = (m == 0 || n == 0);
  if (!empty_c && (!grad_c || !argmax)) return fail(TG_ERR_INVALID_ARGUMENT, "grad_c or argmax is null");
  if (semiring == TG_MAXMUL && !empty_c && !w) return fail(TG_ERR_INVALID_ARGUMENT, "MaxMul backward needs the partner matrix (%s)", want_a ? "B" : "A");
  const int64_t need_ldc = row ? n : m;
  const int64_t need_ldg = row ? g_cols : g_rows;
  if (!empty_c && ldc < std::max<int64_t>(1, need_ldc)) return fail(TG_ERR_DIMENSION_MISMATCH, "ldc=%lld < %lld", (long long)ldc, (long long)need_ldc);
  if (ldg < std::max<int64_t>(1, need_ldg)) return fail(TG_ERR_DIMENSION_MISMATCH, "gradient ld=%lld < %lld", (long long)ldg, (long long)need_ldg);
  if (semiring == TG_MAXMUL && !empty_c) {
    // partner: B (K x N) for grad_A, A (M x K) for grad_B, in caller layout
    const int64_t need_ldw = want_a ? (row ? n : k) : (row ? k : m);
    if (ldw < std::max<int64_t>(1, need_ldw)) return fail(TG_ERR_DIMENSION_MISMATCH, "partner ld=%lld < %lld", (long long)ldw, (long long)need_ldw);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  tg::HistArgs h;
  // Canonical (row-major) view: row-major grad_A = row histogram, grad_B =
  // column histogram; column-major swaps the two roles (C^T = B^T (x) A^T).
  const bool rows_kind = (want_a == row);
  h.rows = row ? m : n;
  h.cols = row ? n : m;
  h.k = k;
  h.gc = grad_c; h.ldc = ldc; h.sc = sc; h.arg = argmax;
  h.w = semiring == TG_MAXMUL ? w : nullptr; h.ldw = ldw; h.sw = sw;
  h.out = grad; h.ldo = ldg; h.so = sg;
  h.accumulate = accumulate;
  if (empty_c) {  // nothing scatters; overwrite means zero
    if (accumulate) return TG_OK;
    const int64_t orow = rows_kind ? h.rows : k, ocol = rows_kind ? k : h.cols;
    for (int64_t b0 = 0; b0 < batch; b0 += 65535) {
      const unsigned nb = unsigned(std::min<int64_t>(65535, batch - b0));
      if (dtype == TG_F32)
        tg::zero_matrix_kernel<float><<<dim3(256, nb), 256, 0, st>>>(static_cast<float*>(grad) + b0 * sg, orow, ocol, ldg, sg);
      else
        tg::zero_matrix_kernel<double><<<dim3(256, nb), 256, 0, st>>>(static_cast<double*>(grad) + b0 * sg, orow, ocol, ldg, sg);
      tg_status s = check_launch("zero_matrix_kernel launch");
      if (s != TG_OK) return s;
    }
    return TG_OK;
  }
  return dtype == TG_F32 ? hist_launch<float>(rows_kind, h, batch, st) : hist_launch<double>(rows_kind, h, batch, st);
}

}  // namespace tgi
