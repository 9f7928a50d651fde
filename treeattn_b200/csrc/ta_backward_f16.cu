// f16 instantiation of the backward kernels (see ta_backward_kernels.cuh).
#include "ta_backward_kernels.cuh"

namespace ta {
template int run_backward_typed<__half>(BwdParams&, cudaStream_t);
}  // namespace ta
