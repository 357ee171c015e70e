// Kernel instantiations for value dtype __half, sampling dtype __half.
#include "msda_binned_launch.cuh"
#include "msda_launch.cuh"

namespace msda {
MSDA_INSTANTIATE_MODE(__half, __half, false)
MSDA_INSTANTIATE_BINNED(__half, __half)
}  // namespace msda
