// SRNL scan kernels instantiated for head_dim 64.
#include "srnl_scan_launch.cuh"

namespace vh {
VH_INSTANTIATE_SCAN(64)
}  // namespace vh
