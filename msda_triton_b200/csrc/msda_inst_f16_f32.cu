// Kernel instantiations for value dtype __half, sampling dtype float.
#include "msda_launch.cuh"

namespace msda {
MSDA_INSTANTIATE_PAIR(__half, float)
}  // namespace msda
