// Tree build that allocates nothing: ta_tree_build_noalloc.
//
// Some callers cannot hand the library a workspace: a host that has given all device
// memory to its own pool (a serving runtime that preallocates HBM at start-up), or a C/FFI
// caller with no device allocator of its own to call. This entry point runs the same
// kernels as ta_tree_build, with the pass-to-pass scratch in a fixed file-scope device
// array instead of a caller workspace, so it calls no cudaMalloc, cudaFree or other
// allocating routine.
//
// Limits and rules:
//  * The scratch holds TA_NOALLOC_SCRATCH_BYTES (8 MiB). Shapes whose scratch need
//    (ta_tree_build_workspace_size) is larger are rejected with TA_ERR_WORKSPACE before
//    anything is launched.
//  * Nothing in the scratch has to start at zero: every pass writes each entry it hands to
//    the next pass before that pass reads it.
//  * The first call on a device does set-up (cudaGetSymbolAddress with that device current,
//    which may load this file's module); make it before any stream capture.
//  * There is one scratch array per device: calls that overlap on the same device (two
//    streams, two host threads) race on it. Serialise them.

#include "ta_common.cuh"

#include <mutex>

namespace {

constexpr size_t kNoAllocScratch = TA_NOALLOC_SCRATCH_BYTES;
static_assert(kNoAllocScratch % 256 == 0, "scratch size must keep 256-byte alignment");

static __device__ __align__(256) unsigned char g_tree_scratch[kNoAllocScratch];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_setup_mu;

// Device address of this device's scratch; looked up once per device.
int scratch_for_current_device(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return ta::fail(TA_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return ta::fail(TA_ERR_UNSUPPORTED, "device ordinal %d beyond %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_tree_scratch);
    if (e != cudaSuccess || !p)
      return ta::fail(TA_ERR_CUDA, "cudaGetSymbolAddress(tree scratch) on device %d: %s", dev,
                      cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return TA_OK;
}

}  // namespace

extern "C" int ta_tree_build_noalloc(int32_t dtype, int64_t B, int64_t S, int64_t H, int64_t D,
                                     const void* k_leaf, ta_layout kl, void* k_int,
                                     ta_layout nl, ta_stream_t stream) {
  if (B > 0 && S > 0 && H > 0 && D > 0) {
    const size_t need = ta_tree_build_workspace_size(B, S, H, D, dtype);
    if (need > kNoAllocScratch)
      return ta::fail(TA_ERR_WORKSPACE,
                      "ta_tree_build_noalloc: this shape needs %zu bytes of scratch, more than "
                      "its fixed %zu; call ta_tree_build with a workspace instead",
                      need, kNoAllocScratch);
  }
  void* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  // ta_tree_build validates the remaining arguments.
  return ta_tree_build(dtype, B, S, H, D, k_leaf, kl, k_int, nl, scratch, kNoAllocScratch,
                       stream);
}
