// Kernel instantiations for value dtype float, sampling dtype float.
#include "msda_binned_launch.cuh"
#include "msda_launch.cuh"

namespace msda {
MSDA_INSTANTIATE_MODE(float, float, false)
MSDA_INSTANTIATE_BINNED(float, float)
}  // namespace msda
