// ascan_fwd_f16.cu -- compilation unit of the scan library: the forward scans for float16.
// The kernels and launchers are defined in ascan_impl.cuh.
#include "ascan_impl.cuh"

namespace ascan {

ASCAN_DECL_FWD(__half, int32_t)
ASCAN_DECL_FWD(__half, int64_t)

ASCAN_UNIT_ERROR_ACCESSORS(fwd_f16)

}  // namespace ascan
