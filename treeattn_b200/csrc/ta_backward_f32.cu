// f32 instantiation of the backward kernels (see ta_backward_kernels.cuh).
#include "ta_backward_kernels.cuh"

namespace ta {
template int run_backward_typed<float>(BwdParams&, cudaStream_t);
}  // namespace ta
