// Sorted-backward instantiations for value dtype __nv_bfloat16, sampling dtype float.
#include "msda_sorted_launch.cuh"

namespace msda {
MSDA_INSTANTIATE_SORTED(__nv_bfloat16, float)
}  // namespace msda
