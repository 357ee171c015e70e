// Sorted-backward instantiations for value dtype __nv_bfloat16, sampling dtype __nv_bfloat16.
#include "msda_sorted_launch.cuh"

namespace msda {
MSDA_INSTANTIATE_SORTED(__nv_bfloat16, __nv_bfloat16)
}  // namespace msda
