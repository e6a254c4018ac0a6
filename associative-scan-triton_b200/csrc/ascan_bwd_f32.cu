// ascan_bwd_f32.cu -- compilation unit of the scan library: the fused backward scans (plain and persistent TMA, every tile width and slab variant) for float32.
// The kernels and launchers are defined in ascan_impl.cuh.
#include "ascan_impl.cuh"

namespace ascan {

ASCAN_DECL_BWD(float, int32_t)
ASCAN_DECL_BWD(float, int64_t)

ASCAN_UNIT_ERROR_ACCESSORS(bwd_f32)

}  // namespace ascan
