// Sorted-backward instantiations for value dtype float, sampling dtype float.
#include "msda_sorted_launch.cuh"

namespace msda {
MSDA_INSTANTIATE_SORTED(float, float)
}  // namespace msda
