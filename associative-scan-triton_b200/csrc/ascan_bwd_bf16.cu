// ascan_bwd_bf16.cu -- compilation unit of the scan library: the fused backward scans for bfloat16.
// The kernels and launchers are defined in ascan_impl.cuh.
#include "ascan_impl.cuh"

namespace ascan {

ASCAN_DECL_BWD(__nv_bfloat16, int32_t)
ASCAN_DECL_BWD(__nv_bfloat16, int64_t)

ASCAN_UNIT_ERROR_ACCESSORS(bwd_bf16)

}  // namespace ascan
