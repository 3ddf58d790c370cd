// Kernel dispatch of the minplus semiring (all dtypes); see tg_dispatch.cuh.
#include "tg_dispatch.cuh"

namespace tgi {
TG_INSTANTIATE_SEMIRING(tg::kMinPlus)
}  // namespace tgi
