// SRNL scan kernels instantiated for head_dim 8.
#include "srnl_scan_launch.cuh"

namespace vh {
VH_INSTANTIATE_SCAN(8)
}  // namespace vh
