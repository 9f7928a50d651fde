// Tensor-core leaf-block attention launchers of the generalised tree, f16 inputs.
#include "ta_blocked_impl.cuh"

namespace ta {
template void attn_fwd_mma<__half>(const BlkParams&, cudaStream_t);
template void attn_bwd_mma<__half>(const BlkParams&, cudaStream_t);
}  // namespace ta
