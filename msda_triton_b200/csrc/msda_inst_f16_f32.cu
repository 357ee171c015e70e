// Kernel instantiations for value dtype __half, sampling dtype float.
#include "msda_binned_launch.cuh"
#include "msda_launch.cuh"

namespace msda {
MSDA_INSTANTIATE_MODE(__half, float, false)
MSDA_INSTANTIATE_BINNED(__half, float)
}  // namespace msda
