// Kernel instantiations for value dtype __nv_bfloat16, sampling dtype float.
#include "msda_launch.cuh"

namespace msda {
MSDA_INSTANTIATE_MODE(__nv_bfloat16, float, false)
}  // namespace msda
