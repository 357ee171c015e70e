// Kernel instantiations for value dtype __half, sampling dtype float.
#include "msda_launch.cuh"

namespace msda {
MSDA_INSTANTIATE_MODE(__half, float, false)
}  // namespace msda
