// ascan_bwd_f16.cu -- compilation unit of the scan library: the fused backward scans for float16.
// The kernels and launchers are defined in ascan_impl.cuh.
#include "ascan_impl.cuh"

namespace ascan {

ASCAN_DECL_BWD(__half, int32_t)
ASCAN_DECL_BWD(__half, int64_t)

ASCAN_UNIT_ERROR_ACCESSORS(bwd_f16)

}  // namespace ascan
