// Kernel instantiations for value dtype float, sampling dtype float.
#include "msda_launch.cuh"

namespace msda {
MSDA_INSTANTIATE_MODE(float, float, false)
}  // namespace msda
