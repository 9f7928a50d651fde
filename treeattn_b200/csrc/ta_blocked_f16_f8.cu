// Instantiations of the generalised-tree launchers for f16 inputs, fanout 8.
#include "ta_blocked_impl.cuh"

namespace ta {
TA_BLK_EPLS(TA_BLK_INSTANTIATE, __half, 8)
}  // namespace ta
