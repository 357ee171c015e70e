// Kernel instantiations for value dtype __half, sampling dtype __half.
#include "msda_launch.cuh"

namespace msda {
MSDA_INSTANTIATE_MODE(__half, __half, false)
}  // namespace msda
