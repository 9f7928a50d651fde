// The reference's Gumbel stream, regenerated in-kernel (sm_100a).
//
// The reference draws Gumbel noise per tree depth with
//   torch.empty((L,B,H,S,2), dtype=float32, device=cuda).exponential_().log_().neg_()
// (_autograd.py:188-195; _tree_mha.py:109). torch's distribution kernel runs a grid-stride
// loop with 256-thread blocks and 4 uniforms per curand_uniform4 call, so element e of a
// draw of stride St is component (e/St)%4 of call (e/St)/4 of philox subsequence e%St,
// starting at the generator's (seed, offset). The exponential transform is
//   E = -log(u), with log(u) replaced by -eps/2 when u >= 1 - eps/2 (eps = FLT_EPSILON),
// and the Gumbel is G = -log(E). All logs are the accurate libm logf (torch's own kernels
// are not built with fast-math, so neither is this one).
#pragma once

#include <curand_kernel.h>
#include <float.h>

namespace ta {

// n / d for 32-bit n with a divisor fixed per launch (Granlund & Montgomery, PLDI 1994).
struct FastDiv {
  uint32_t d, m, s;
  __host__ void init(uint32_t div) {
    d = div;
    s = 0;
    while ((1ull << s) < div) ++s;
    m = (uint32_t)((((1ull << 32) * ((1ull << s) - div)) / div) + 1ull);
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    return (uint32_t)(((uint64_t)__umulhi(n, m) + n) >> s);
  }
};

// One uniform of torch's CUDA exponential_ draw: element `e` of a draw whose philox state
// starts at (seed, offset) with grid stride `stride`.
__device__ __forceinline__ float torch_uniform(uint64_t seed, uint64_t offset, uint32_t e,
                                               const FastDiv& stride) {
  const uint32_t bundle = stride.div(e);
  const uint32_t tid = e - bundle * stride.d;
  curandStatePhilox4_32_10_t st;
  // Position (offset/4 + bundle/4) of subsequence `tid`; offsets are multiples of 4, so the
  // state's first output is exactly the 4-vector that call bundle/4 of torch's loop returns.
  curand_init(seed, tid, offset + 4ull * (uint64_t)(bundle >> 2), &st);
  const float4 u4 = _curand_uniform4(st.output);
  const uint32_t c = bundle & 3u;
  return c == 0 ? u4.x : (c == 1 ? u4.y : (c == 2 ? u4.z : u4.w));
}

__device__ __forceinline__ float gumbel_from_uniform(float u) {
  const float half_eps = FLT_EPSILON * 0.5f;
  const float lg = (u >= 1.0f - half_eps) ? -half_eps : __logf(u);
  const float e = -1.0f / 1.0f * lg;
  return -logf(e);
}

__device__ __forceinline__ float torch_gumbel(uint64_t seed, uint64_t offset, uint32_t e,
                                              const FastDiv& stride) {
  return gumbel_from_uniform(torch_uniform(seed, offset, e, stride));
}

}  // namespace ta
