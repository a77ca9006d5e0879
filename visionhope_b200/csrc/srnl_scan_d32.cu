// SRNL scan kernels instantiated for head_dim 32.
#include "srnl_scan_launch.cuh"

namespace vh {
VH_INSTANTIATE_SCAN(32)
}  // namespace vh
