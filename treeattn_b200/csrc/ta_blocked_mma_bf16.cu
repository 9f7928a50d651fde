// Tensor-core leaf-block attention launchers of the generalised tree, bf16 inputs.
#include "ta_blocked_impl.cuh"

namespace ta {
template void attn_fwd_mma<__nv_bfloat16>(const BlkParams&, cudaStream_t);
template void attn_bwd_mma<__nv_bfloat16>(const BlkParams&, cudaStream_t);
}  // namespace ta
