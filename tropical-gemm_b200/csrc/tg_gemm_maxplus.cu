// Kernel dispatch of the maxplus semiring (all dtypes); see tg_dispatch.cuh.
#include "tg_dispatch.cuh"

namespace tgi {
TG_INSTANTIATE_SEMIRING(tg::kMaxPlus)
}  // namespace tgi
