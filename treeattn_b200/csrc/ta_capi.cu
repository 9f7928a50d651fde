// Runtime helpers of the C ABI: per-thread error messages, version, RNG plan.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include "ta_common.cuh"

namespace ta {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(TA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return TA_OK;
}

}  // namespace ta

extern "C" const char* ta_last_error(void) { return ta::g_err; }

extern "C" int32_t ta_abi_version(void) { return TA_ABI_VERSION; }

// torch's calc_execution_policy for distribution kernels: 256-thread blocks, grid capped at
// SMs * (max threads per SM / 256), 4 philox outputs per thread per loop trip; the offset
// advances by 4 per trip (sample_non_causal_paths.cu:139-156 restates the same policy).
extern "C" int ta_philox_plan(int64_t numel, int32_t sm_count, int32_t max_threads_per_sm,
                              uint64_t* offset_step, int64_t* draw_stride) {
  if (numel <= 0 || sm_count <= 0 || max_threads_per_sm < 256 || !offset_step || !draw_stride)
    return ta::fail(TA_ERR_INVALID, "ta_philox_plan: invalid arguments");
  const uint64_t block = 256, unroll = 4;
  const uint64_t n = (uint64_t)numel;
  const uint64_t max_grid = (uint64_t)sm_count * (uint64_t)(max_threads_per_sm / 256);
  uint64_t grid = (n + block - 1) / block;
  if (grid > max_grid) grid = max_grid;
  *offset_step = ((n - 1) / (block * grid * unroll) + 1) * 4;
  *draw_stride = (int64_t)(block * grid);
  return TA_OK;
}

extern "C" int ta_device_rng_geometry(int32_t device, int32_t* sm_count,
                                      int32_t* max_threads_per_sm) {
  if (!sm_count || !max_threads_per_sm) return ta::fail(TA_ERR_INVALID, "NULL output");
  int a = 0, b = 0;
  cudaError_t e = cudaDeviceGetAttribute(&a, cudaDevAttrMultiProcessorCount, device);
  if (e == cudaSuccess)
    e = cudaDeviceGetAttribute(&b, cudaDevAttrMaxThreadsPerMultiProcessor, device);
  if (e != cudaSuccess) return ta::fail(TA_ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
  *sm_count = a;
  *max_threads_per_sm = b;
  return TA_OK;
}
