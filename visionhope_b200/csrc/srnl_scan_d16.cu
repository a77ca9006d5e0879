// SRNL scan kernels instantiated for head_dim 16.
#include "srnl_scan_launch.cuh"

namespace vh {
VH_INSTANTIATE_SCAN(16)
}  // namespace vh
