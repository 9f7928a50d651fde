// Instantiations of the generalised-tree launchers for f32 inputs, fanout 8.
#include "ta_blocked_impl.cuh"

namespace ta {
TA_BLK_EPLS(TA_BLK_INSTANTIATE, float, 8)
}  // namespace ta
