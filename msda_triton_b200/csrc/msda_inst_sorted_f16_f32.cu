// Sorted-backward instantiations for value dtype __half, sampling dtype float.
#include "msda_sorted_launch.cuh"

namespace msda {
MSDA_INSTANTIATE_SORTED(__half, float)
}  // namespace msda
