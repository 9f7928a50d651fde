// Runtime helpers of the C ABI: per-thread error messages, version, RNG plan.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <map>
#include <mutex>
#include <string>
#include <vector>

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

// ---- per-launch profiling -------------------------------------------------------------
struct ProfRecord {
  const char* name;
  cudaEvent_t start, stop;
};
static std::mutex g_prof_mu;
static bool g_prof_on = false;
static std::vector<ProfRecord> g_prof;
static std::vector<cudaEvent_t> g_prof_pool;

static cudaEvent_t prof_event() {
  if (!g_prof_pool.empty()) {
    cudaEvent_t e = g_prof_pool.back();
    g_prof_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

ProfScope::ProfScope(const char* name, cudaStream_t st) : slot(-1), stream(st) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  if (!g_prof_on) return;
  ProfRecord r{name, prof_event(), prof_event()};
  cudaEventRecord(r.start, st);
  slot = (int)g_prof.size();
  g_prof.push_back(r);
}

ProfScope::~ProfScope() {
  if (slot < 0) return;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  cudaEventRecord(g_prof[slot].stop, stream);
}

}  // namespace ta

extern "C" int ta_profile_enable(int32_t on) {
  std::lock_guard<std::mutex> lk(ta::g_prof_mu);
  ta::g_prof_on = on != 0;
  return TA_OK;
}

// Waits for every recorded launch, writes "name count total_ms" lines (sorted by name) and
// clears the records. Returns the bytes needed (excluding the terminator); truncates to len.
extern "C" int64_t ta_profile_collect(char* buf, size_t len) {
  std::lock_guard<std::mutex> lk(ta::g_prof_mu);
  std::map<std::string, std::pair<int64_t, double>> agg;
  for (auto& r : ta::g_prof) {
    float ms = 0.0f;
    if (cudaEventSynchronize(r.stop) == cudaSuccess) cudaEventElapsedTime(&ms, r.start, r.stop);
    auto& a = agg[r.name];
    a.first += 1;
    a.second += ms;
    ta::g_prof_pool.push_back(r.start);
    ta::g_prof_pool.push_back(r.stop);
  }
  ta::g_prof.clear();
  std::string out;
  char line[256];
  for (auto& kv : agg) {
    snprintf(line, sizeof(line), "%s %lld %.6f\n", kv.first.c_str(), (long long)kv.second.first,
             kv.second.second);
    out += line;
  }
  if (buf && len) {
    const size_t n = out.size() < len - 1 ? out.size() : len - 1;
    memcpy(buf, out.data(), n);
    buf[n] = 0;
  }
  return (int64_t)out.size();
}

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
