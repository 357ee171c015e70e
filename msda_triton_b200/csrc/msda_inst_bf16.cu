// Kernel instantiations for value dtype __nv_bfloat16, sampling dtype __nv_bfloat16.
#include "msda_launch.cuh"

namespace msda {
MSDA_INSTANTIATE_MODE(__nv_bfloat16, __nv_bfloat16, false)
}  // namespace msda
