// ascan_bidi.cu -- compilation unit of the scan library: the one-launch bidirectional pairs (forward and adjoint) for every dtype.
// The kernels and launchers are defined in ascan_impl.cuh.
#include "ascan_impl.cuh"

namespace ascan {

ASCAN_FOR_EACH_TYPE_PAIR(ASCAN_DECL_FWD_BIDI)
ASCAN_FOR_EACH_TYPE_PAIR(ASCAN_DECL_BWD_BIDI)

ASCAN_UNIT_ERROR_ACCESSORS(bidi)

}  // namespace ascan
