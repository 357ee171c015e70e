// Kernel instantiations for value dtype __nv_bfloat16, sampling dtype float.
#include "msda_binned_launch.cuh"
#include "msda_launch.cuh"

namespace msda {
MSDA_INSTANTIATE_MODE(__nv_bfloat16, float, false)
MSDA_INSTANTIATE_BINNED(__nv_bfloat16, float)
}  // namespace msda
