// Sorted-backward instantiations for value dtype __half, sampling dtype __half.
#include "msda_sorted_launch.cuh"

namespace msda {
MSDA_INSTANTIATE_SORTED(__half, __half)
}  // namespace msda
