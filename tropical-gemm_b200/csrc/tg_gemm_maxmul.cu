// Kernel dispatch of the maxmul semiring (all dtypes); see tg_dispatch.cuh.
#include "tg_dispatch.cuh"

namespace tgi {
TG_INSTANTIATE_SEMIRING(tg::kMaxMul)
}  // namespace tgi
