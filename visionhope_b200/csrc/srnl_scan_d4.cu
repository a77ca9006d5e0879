// SRNL scan kernels instantiated for head_dim 4.
#include "srnl_scan_launch.cuh"

namespace vh {
VH_INSTANTIATE_SCAN(4)
}  // namespace vh
