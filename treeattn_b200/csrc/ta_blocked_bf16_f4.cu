// Instantiations of the generalised-tree launchers for bf16 inputs, fanout 4.
#include "ta_blocked_impl.cuh"

namespace ta {
TA_BLK_EPLS(TA_BLK_INSTANTIATE, __nv_bfloat16, 4)
}  // namespace ta
