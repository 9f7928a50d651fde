// Fused deterministic backward: host entry point and the per-head path sort.
// The typed kernels live in ta_backward_kernels.cuh (instantiated per dtype in
// ta_backward_{f32,f16,bf16}.cu so the heavy templates compile in parallel).

#include "ta_backward_kernels.cuh"

namespace ta {

template <typename T> int run_backward_typed(BwdParams& p, cudaStream_t st);
extern template int run_backward_typed<float>(BwdParams&, cudaStream_t);
extern template int run_backward_typed<__half>(BwdParams&, cudaStream_t);
extern template int run_backward_typed<__nv_bfloat16>(BwdParams&, cudaStream_t);

// ---------------------------------------------------------------------------------------
// 2. segmented stable LSD radix sort of (key, value) records, one segment per head
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kSortThreads) sort_hist_kernel(const BwdParams p, int src, int shift) {
  __shared__ uint32_t cnt[kRadix];
  const int seg = blockIdx.x / p.tiles_per_seg;
  const int tile = blockIdx.x - seg * p.tiles_per_seg;
  for (int i = threadIdx.x; i < kRadix; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  const int64_t base = (int64_t)seg * p.P + (int64_t)tile * kSortTile;
  const int64_t end = min((int64_t)(tile + 1) * kSortTile, p.P) - (int64_t)tile * kSortTile;
  for (int i = threadIdx.x; i < end; i += blockDim.x)
    atomicAdd(&cnt[(p.keys[src][base + i] >> shift) & (kRadix - 1)], 1u);
  __syncthreads();
  for (int d = threadIdx.x; d < kRadix; d += blockDim.x)
    p.hist[((int64_t)seg * kRadix + d) * p.tiles_per_seg + tile] = cnt[d];
}

// exclusive scan of one segment's histogram in (digit, tile) order
__global__ void __launch_bounds__(1024) sort_scan_kernel(const BwdParams p) {
  __shared__ uint32_t warp_tot[32];
  __shared__ uint32_t carry;
  const int seg = blockIdx.x;
  uint32_t* hh = p.hist + (int64_t)seg * kRadix * p.tiles_per_seg;
  const int64_t n = (int64_t)kRadix * p.tiles_per_seg;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t base = 0; base < n; base += blockDim.x) {
    const int64_t i = base + threadIdx.x;
    const uint32_t v = i < n ? hh[i] : 0u;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    if (warp == 0) {
      uint32_t t = lane < (int)(blockDim.x >> 5) ? warp_tot[lane] : 0u;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t += y;
      }
      warp_tot[lane] = t;  // inclusive
    }
    __syncthreads();
    const uint32_t before = carry + (warp > 0 ? warp_tot[warp - 1] : 0u) + x - v;
    if (i < n) hh[i] = before;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = before + v;
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kSortThreads) sort_scatter_kernel(const BwdParams p, int src, int shift) {
  constexpr int kWarps = kSortThreads / 32;
  constexpr int kPerWarp = kSortTile / kWarps;  // 256 records
  __shared__ uint32_t wcnt[kWarps][kRadix];
  const int seg = blockIdx.x / p.tiles_per_seg;
  const int tile = blockIdx.x - seg * p.tiles_per_seg;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < kWarps * kRadix; i += blockDim.x) (&wcnt[0][0])[i] = 0;
  __syncthreads();
  const int64_t tbase = (int64_t)tile * kSortTile;
  const int64_t base = (int64_t)seg * p.P + tbase;
  const int64_t nvalid = min((int64_t)kSortTile, p.P - tbase);
  // per-warp digit counts
  uint32_t key[kPerWarp / 32], val[kPerWarp / 32];
  int dig[kPerWarp / 32];
#pragma unroll
  for (int r = 0; r < kPerWarp / 32; ++r) {
    const int64_t i = (int64_t)warp * kPerWarp + r * 32 + lane;
    if (i < nvalid) {
      key[r] = p.keys[src][base + i];
      val[r] = p.vals[src][base + i];
      dig[r] = (key[r] >> shift) & (kRadix - 1);
      atomicAdd(&wcnt[warp][dig[r]], 1u);
    } else {
      dig[r] = kRadix;  // sentinel: not written
    }
  }
  __syncthreads();
  // exclusive scan over warps per digit, plus the global (digit, tile) offset
  for (int d = threadIdx.x; d < kRadix; d += blockDim.x) {
    uint32_t run = p.hist[((int64_t)seg * kRadix + d) * p.tiles_per_seg + tile];
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const uint32_t c = wcnt[w][d];
      wcnt[w][d] = run;
      run += c;
    }
  }
  __syncthreads();
  const unsigned lt_mask = (1u << lane) - 1u;
  uint32_t* dk = p.keys[src ^ 1] + (int64_t)seg * p.P;
  uint32_t* dv = p.vals[src ^ 1] + (int64_t)seg * p.P;
#pragma unroll
  for (int r = 0; r < kPerWarp / 32; ++r) {
    const unsigned same = __match_any_sync(0xffffffffu, dig[r]);
    const int leader = __ffs(same) - 1;
    if (dig[r] < kRadix) {
      const uint32_t pos = wcnt[warp][dig[r]] + __popc(same & lt_mask);
      dk[pos] = key[r];
      dv[pos] = val[r];
    }
    __syncwarp();
    if (lane == leader && dig[r] < kRadix) wcnt[warp][dig[r]] += __popc(same);
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------
struct BwdLayout {
  size_t keys[2], vals[2], dlp, hist, partial, flags, total;
};

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

namespace {
int32_t g_node_range_chunks = 0;  // 0: chunks per node-pass range follow from the shape
}

extern "C" int32_t ta_backward_set_node_range(int32_t chunks) {
  const int32_t old = g_node_range_chunks;
  g_node_range_chunks = chunks < 0 ? 0 : chunks;
  return old;
}

static int chunk_of(const ta_shape* s) {
  return use_mma_node_pass(s->dtype, s->head_dim, floor_log2(s->num_leaves)) ? kChunkMma : kChunk;
}

static BwdLayout bwd_layout(const ta_shape* s) {
  BwdLayout w{};
  const int64_t HB = s->batch * s->num_heads;
  const int64_t P = s->num_queries * s->num_samples;
  const int ln = floor_log2(s->num_leaves);
  const int64_t tiles = (P + kSortTile - 1) / kSortTile;
  const int64_t chunks = HB * ((P + chunk_of(s) - 1) / chunk_of(s));
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += align256(bytes); return o; };
  w.keys[0] = take(HB * P * 4);
  w.keys[1] = take(HB * P * 4);
  w.vals[0] = take(HB * P * 4);
  w.vals[1] = take(HB * P * 4);
  w.dlp = take(HB * P * 4);
  w.hist = take(HB * kRadix * tiles * 4);
  w.partial = take(chunks * (ln + 1) * 2 * s->head_dim * 4);
  w.flags = take(chunks * (ln + 1) * 2);
  w.total = off;
  return w;
}


bool backward_fork_handles(cudaStream_t& side, cudaEvent_t& fork, cudaEvent_t& join,
                           cudaStream_t st) {
  struct Handles {
    cudaStream_t side = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
  };
  constexpr int kMaxDevices = 64;
  thread_local Handles h[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return false;
  }
  int sdev = dev;  // fork only when the caller's stream is on the current device
  if (cudaStreamGetDevice(st, &sdev) != cudaSuccess || sdev != dev) {
    cudaGetLastError();
    return false;
  }
  Handles& x = h[dev];
  if (x.side == nullptr) {
    if (cudaStreamCreateWithFlags(&x.side, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&x.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&x.join, cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      x = Handles{};
      return false;
    }
  }
  side = x.side;
  fork = x.fork;
  join = x.join;
  return true;
}

int run_sort(BwdParams& p, cudaStream_t st) {
  const int passes = (p.log_n + kRadixBits - 1) / kRadixBits;
  const unsigned tiles = (unsigned)(p.B * p.H * p.tiles_per_seg);
  int src = 0;
  for (int ps = 0; ps < passes; ++ps) {
    {
      TA_PROFILE("sort_hist", st);
      sort_hist_kernel<<<tiles, kSortThreads, 0, st>>>(p, src, ps * kRadixBits);
    }
    {
      TA_PROFILE("sort_scan", st);
      sort_scan_kernel<<<p.B * p.H, 1024, 0, st>>>(p);
    }
    {
      TA_PROFILE("sort_scatter", st);
      sort_scatter_kernel<<<tiles, kSortThreads, 0, st>>>(p, src, ps * kRadixBits);
    }
    src ^= 1;
  }
  p.sorted_buf = src;
  return check_launch("backward path sort");
}

}  // namespace ta

using namespace ta;

extern "C" size_t ta_backward_workspace_size(const ta_shape* shape) {
  if (check_shape(shape, true) != TA_OK) return 0;
  return bwd_layout(shape).total;
}

// Shared setup of ta_backward / ta_backward_coef.
static int bwd_setup(const ta_shape* shape, const void* q, ta_layout ql, const void* k,
                     ta_layout kl, const void* gout, ta_layout gl, void* dq, ta_layout dql,
                     void* dk, ta_layout dkl, int32_t dk_dtype, void* dv, ta_layout dvl,
                     int32_t dv_dtype, void* ws, size_t ws_bytes, BwdParams& p) {
  int rc = check_shape(shape, true);
  if (rc) return rc;
  const int es = dtype_size(shape->dtype);
  if (dk_dtype != TA_F32 && dk_dtype != shape->dtype)
    return fail(TA_ERR_INVALID, "dk_dtype must be TA_F32 or the input dtype");
  if (dv_dtype != TA_F32 && dv_dtype != shape->dtype)
    return fail(TA_ERR_INVALID, "dv_dtype must be TA_F32 or the input dtype");
  if ((rc = check_view("q", q, ql, es, false)) || (rc = check_view("k_int", k, kl, es, false)) ||
      (rc = check_view("grad_out", gout, gl, es, false)) ||
      (rc = check_view("dq", dq, dql, es, false)) ||
      (rc = check_view("dk", dk, dkl, dtype_size(dk_dtype), false)) ||
      (rc = check_view("dv", dv, dvl, dtype_size(dv_dtype), false)))
    return rc;
  if (shape->num_queries * shape->num_samples >= (1ll << 31))
    return fail(TA_ERR_UNSUPPORTED, "L * S must be < 2^31");
  const BwdLayout w = bwd_layout(shape);
  if (ws == nullptr || ws_bytes < w.total)
    return fail(TA_ERR_WORKSPACE, "backward workspace too small (%zu < %zu)", ws_bytes, w.total);
  p = BwdParams{};
  p.q = (const char*)q; p.k = (const char*)k; p.dout = (const char*)gout;
  p.dq = (char*)dq; p.dk = (char*)dk; p.dv = (char*)dv;
  p.qs = ql.seq; p.qb = ql.batch; p.qh = ql.head;
  p.ks = kl.seq; p.kb = kl.batch; p.kh = kl.head;
  p.gs = gl.seq; p.gb = gl.batch; p.gh = gl.head;
  p.dqs = dql.seq; p.dqb = dql.batch; p.dqh = dql.head;
  p.dks = dkl.seq; p.dkb = dkl.batch; p.dkh = dkl.head;
  p.dvs = dvl.seq; p.dvb = dvl.batch; p.dvh = dvl.head;
  char* base = (char*)ws;
  p.keys[0] = (uint32_t*)(base + w.keys[0]); p.keys[1] = (uint32_t*)(base + w.keys[1]);
  p.vals[0] = (uint32_t*)(base + w.vals[0]); p.vals[1] = (uint32_t*)(base + w.vals[1]);
  p.dlp = (float*)(base + w.dlp); p.hist = (uint32_t*)(base + w.hist);
  p.partial = (float*)(base + w.partial); p.flags = (uint8_t*)(base + w.flags);
  p.B = (int32_t)shape->batch; p.L = (int32_t)shape->num_queries; p.H = (int32_t)shape->num_heads;
  p.S = (int32_t)shape->num_samples; p.N = (int32_t)shape->num_leaves;
  p.D = (int32_t)shape->head_dim; p.log_n = floor_log2(shape->num_leaves);
  p.nchunks = (int32_t)(shape->head_dim * es / 16);
  p.sig_stride = (p.log_n + 3) & ~3;
  p.top_levels = smem_tree_levels(p.log_n, p.nchunks * 16, kTreeSmemBudget);
  p.dk_f32 = dk_dtype == TA_F32 ? 1 : 0;
  p.dv_f32 = dv_dtype == TA_F32 ? 1 : 0;
  p.P = shape->num_queries * shape->num_samples;
  p.tiles_per_seg = (int32_t)((p.P + kSortTile - 1) / kSortTile);
  p.chunk = chunk_of(shape);
  p.chunks_per_seg = (int32_t)((p.P + p.chunk - 1) / p.chunk);
  p.max_logit = shape->max_logit;
  p.node_range_chunks = g_node_range_chunks;
  p.qtable_levels = 0;
  if (shape->dtype == TA_BF16 && p.nchunks % 2 == 0 && p.nchunks <= 16 && p.log_n >= 4) {
    const int tl = p.log_n < kQTableLevels ? p.log_n : kQTableLevels;
    if ((size_t)kBwdGroups * p.S * 4 + qtable_smem(tl, p.nchunks * 16, p.nchunks * 8) <= 200 * 1024) {
      p.qtable_levels = tl;
      p.top_levels = 0;
    }
  }
  if (p.log_n > 30) return fail(TA_ERR_UNSUPPORTED, "tree too deep");
  return TA_OK;
}

static int bwd_run(const ta_shape* shape, BwdParams& p, cudaStream_t st) {
  switch (shape->dtype) {
    case TA_F32: return run_backward_typed<float>(p, st);
    case TA_F16: return run_backward_typed<__half>(p, st);
    default: return run_backward_typed<__nv_bfloat16>(p, st);
  }
}

extern "C" int ta_backward(const ta_shape* shape, const void* q, ta_layout ql, const void* k,
                           ta_layout kl, const void* v, ta_layout vl, const void* gout,
                           ta_layout gl, const int32_t* leaf, const float* weights,
                           const float* branch_prob, void* dq, ta_layout dql, void* dk,
                           ta_layout dkl, int32_t dk_dtype, void* dv, ta_layout dvl,
                           int32_t dv_dtype, void* ws, size_t ws_bytes, ta_stream_t stream) {
  BwdParams p;
  int rc = bwd_setup(shape, q, ql, k, kl, gout, gl, dq, dql, dk, dkl, dk_dtype, dv, dvl,
                     dv_dtype, ws, ws_bytes, p);
  if (rc) return rc;
  if ((rc = check_view("v", v, vl, dtype_size(shape->dtype), false))) return rc;
  if (!leaf || !weights || !branch_prob)
    return fail(TA_ERR_INVALID, "leaf, weights and branch_prob must not be NULL");
  p.v = (const char*)v; p.vs = vl.seq; p.vb = vl.batch; p.vh = vl.head;
  p.leaf = leaf; p.weights = weights; p.sig = branch_prob;
  return bwd_run(shape, p, (cudaStream_t)stream);
}

extern "C" int ta_backward_coef(const ta_shape* shape, const void* q, ta_layout ql,
                                const void* k, ta_layout kl, const void* gout, ta_layout gl,
                                const float* coef, const float* value_weight,
                                const uint32_t* keys, const uint32_t* vals, void* dq,
                                ta_layout dql, void* dk, ta_layout dkl, int32_t dk_dtype,
                                void* dv, ta_layout dvl, int32_t dv_dtype, void* ws,
                                size_t ws_bytes, ta_stream_t stream) {
  BwdParams p;
  int rc = bwd_setup(shape, q, ql, k, kl, gout, gl, dq, dql, dk, dkl, dk_dtype, dv, dvl,
                     dv_dtype, ws, ws_bytes, p);
  if (rc) return rc;
  if (!coef || !value_weight || !keys || !vals)
    return fail(TA_ERR_INVALID, "coef, value_weight, keys and vals must not be NULL");
  cudaStream_t st = (cudaStream_t)stream;
  const size_t n = (size_t)(shape->batch * shape->num_heads) * (size_t)p.P;
  cudaMemcpyAsync(p.keys[0], keys, n * 4, cudaMemcpyDeviceToDevice, st);
  cudaMemcpyAsync(p.vals[0], vals, n * 4, cudaMemcpyDeviceToDevice, st);
  cudaMemcpyAsync(p.dlp, value_weight, n * 4, cudaMemcpyDeviceToDevice, st);
  if ((rc = check_launch("backward inputs"))) return rc;
  p.sig = coef;
  p.coef_mode = 1;
  return bwd_run(shape, p, st);
}
