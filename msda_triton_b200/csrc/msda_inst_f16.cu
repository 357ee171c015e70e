// Kernel instantiations for value dtype __half, sampling dtype __half.
#include "msda_binned_launch.cuh"
#include "msda_launch.cuh"

namespace msda {
MSDA_INSTANTIATE_PAIR(__half, __half)
MSDA_INSTANTIATE_BINNED(__half, __half)
}  // namespace msda
