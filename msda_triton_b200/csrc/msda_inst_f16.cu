// Kernel instantiations for value dtype __half, sampling dtype __half.
#include "msda_launch.cuh"

namespace msda {
MSDA_INSTANTIATE_PAIR(__half, __half)
}  // namespace msda
