// Instantiations of the generalised-tree launchers for bf16 inputs, fanout 2.
#include "ta_blocked_impl.cuh"

namespace ta {
TA_BLK_EPLS(TA_BLK_INSTANTIATE, __nv_bfloat16, 2)
}  // namespace ta
