// Generalised tree attention (fanout, leaf blocks): C-ABI entry points, summary build and
// noise dump. Kernels and launchers: ta_blocked_impl.cuh; per-(dtype, fanout) instantiations:
// ta_blocked_<dtype>_f<fanout>.cu; tensor-core leaf-block kernels: ta_blocked_mma_<dtype>.cu.

#include <atomic>
#include <mutex>

#include "ta_blocked_impl.cuh"

namespace ta {

__global__ void __launch_bounds__(256) blk_summary_up_kernel(const BlkParams p, int d) {
  // level d from level d + 1: mean of the f children's summaries
  int64_t rows = 1;
  for (int t = 0; t < d; ++t) rows *= p.f;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t per_head = rows * p.D;
  if (i >= per_head * p.B * p.H) return;
  const int bh = (int)(i / per_head);
  const int64_t r = i - (int64_t)bh * per_head;
  const int64_t j = r / p.D;
  const int c = (int)(r - j * p.D);
  const float* src = p.summ + ((int64_t)bh * p.R + p.lvl_off[d + 1] + j * p.f) * p.D + c;
  float acc = 0.0f;
  for (int t = 0; t < p.f; ++t) acc += src[(int64_t)t * p.D];
  p.summ[((int64_t)bh * p.R + p.lvl_off[d] + j) * p.D + c] = acc / (float)p.f;
}

__global__ void __launch_bounds__(256) blk_gumbel_kernel(const BlkParams p, float* out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)p.Dp * p.L * p.B * p.H * p.S * p.f;
  if (i >= total) return;
  int64_t t = i;
  const int ci = (int)(t % p.f); t /= p.f;
  const int s = (int)(t % p.S); t /= p.S;
  const int h = (int)(t % p.H); t /= p.H;
  const int b = (int)(t % p.B); t /= p.B;
  const int l = (int)(t % p.L);
  const int d = (int)(t / p.L);
  out[i] = blk_gumbel(p, b, h, l, d, s, ci);
}

template <typename T>
static int blk_build_typed(BlkParams& p, cudaStream_t st) {
  const int64_t HB = (int64_t)p.B * p.H;
  {
    TA_PROFILE("blocked_summary", st);
    const int64_t n = HB * p.nb * p.D;
    if (p.Dp > 0) blk_summary_leaf_kernel<T><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(p);
    int64_t rows = p.nb;
    for (int d = p.Dp - 1; d >= 1; --d) {
      rows /= p.f;
      const int64_t m = HB * rows * p.D;
      blk_summary_up_kernel<<<(unsigned)((m + 255) / 256), 256, 0, st>>>(p, d);
    }
  }
  return check_launch("blocked summaries");
}

// (dtype, head_dim, fanout) -> the instantiation of FN for it
#define TA_BLK_DISPATCH_F(FN, T, EPL, ...)                           \
  switch (p.f) {                                                     \
    case 2: return FN<T, EPL, 2>(__VA_ARGS__);                       \
    case 4: return FN<T, EPL, 4>(__VA_ARGS__);                       \
    case 8: return FN<T, EPL, 8>(__VA_ARGS__);                       \
    default: return FN<T, EPL, 16>(__VA_ARGS__);                     \
  }
#define TA_BLK_DISPATCH_D(FN, T, ...)                                \
  switch (p.D) {                                                     \
    case 32: TA_BLK_DISPATCH_F(FN, T, 1, __VA_ARGS__)                \
    case 64: TA_BLK_DISPATCH_F(FN, T, 2, __VA_ARGS__)                \
    case 96: TA_BLK_DISPATCH_F(FN, T, 3, __VA_ARGS__)                \
    case 128: TA_BLK_DISPATCH_F(FN, T, 4, __VA_ARGS__)               \
    default: TA_BLK_DISPATCH_F(FN, T, 8, __VA_ARGS__)                \
  }
#define TA_BLK_DISPATCH(FN, ...)                                     \
  switch (p.dtype) {                                                 \
    case TA_F32: TA_BLK_DISPATCH_D(FN, float, __VA_ARGS__)           \
    case TA_F16: TA_BLK_DISPATCH_D(FN, __half, __VA_ARGS__)          \
    default: TA_BLK_DISPATCH_D(FN, __nv_bfloat16, __VA_ARGS__)       \
  }

}  // namespace ta

using namespace ta;

extern "C" int64_t ta_blocked_summary_rows(int64_t num_leaves, int32_t fanout, int32_t leaf_block) {
  int Dp; int64_t nb, R, off[kBlkMaxLevels + 1];
  if (blk_geometry(num_leaves, fanout, leaf_block, &Dp, &nb, &R, off) != TA_OK) return -1;
  return R;
}

extern "C" int ta_blocked_build(const ta_shape* shape, const ta_blocked* cfg, const void* k,
                                ta_layout kl, float* summaries, ta_stream_t stream) {
  BlkParams p;
  int rc = blk_setup(shape, cfg, p);
  if (rc) return rc;
  if ((rc = blk_views(shape, p, nullptr, {}, k, kl, nullptr, {}))) return rc;
  if (p.R > 0 && !summaries) return fail(TA_ERR_INVALID, "summaries is NULL");
  p.summ = summaries;
  if (p.Dp == 0) return TA_OK;
  cudaStream_t st = (cudaStream_t)stream;
  switch (p.dtype) {
    case TA_F32: return blk_build_typed<float>(p, st);
    case TA_F16: return blk_build_typed<__half>(p, st);
    default: return blk_build_typed<__nv_bfloat16>(p, st);
  }
}

static int blk_noise(BlkParams& p, const ta_rng* rng, const float* gumbels) {
  p.gumbels = gumbels;
  if (gumbels) return TA_OK;
  if (!rng) return fail(TA_ERR_INVALID, "rng is NULL and no gumbels were given");
  if (rng->offset & 3) return fail(TA_ERR_INVALID, "rng offset must be a multiple of 4");
  p.seed = rng->seed;
  p.offset = rng->offset;
  return TA_OK;
}

extern "C" int ta_blocked_gumbel_fill(const ta_shape* shape, const ta_blocked* cfg,
                                      const ta_rng* rng, float* out, ta_stream_t stream) {
  BlkParams p;
  int rc = blk_setup(shape, cfg, p);
  if (rc) return rc;
  if ((rc = blk_noise(p, rng, nullptr))) return rc;
  if (!out) return fail(TA_ERR_INVALID, "out is NULL");
  const int64_t n = (int64_t)p.Dp * p.L * p.B * p.H * p.S * p.f;
  if (n == 0) return TA_OK;
  blk_gumbel_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(p, out);
  return check_launch("blocked gumbel fill");
}

namespace {
// leaf-block forward on tcgen05 (1) or mma.sync (0). mma.sync is the default: it measured
// faster (config 2: 1.32 vs 1.54 ms per forward, config 3: 7.0 vs 9.6 ms), the tcgen05 kernel
// serialising gather, MMA and epilogue per 128-pair tile at two CTAs per SM.
int g_use_tcgen05 = -1;  // -1: by shape (tcgen05 at leaf block 128), 0: mma.sync, 1: tcgen05
int g_use_tcgen05_bwd = 1;
std::atomic<uint64_t> g_tc_wait_ns{kTcWaitNs};
std::mutex g_tc_status_mu;
int32_t* g_tc_status = nullptr;  // mapped, portable pinned host word (process-wide, sticky)

// The status word the tcgen05 kernels write on an expired wait: host memory the GPU writes
// through its mapping, so the host reads it without a device synchronisation.
int32_t* tc_status_word() {
  std::lock_guard<std::mutex> lk(g_tc_status_mu);
  if (g_tc_status == nullptr) {
    void* h = nullptr;
    if (cudaHostAlloc(&h, 256, cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    *(volatile int32_t*)h = 0;
    g_tc_status = (int32_t*)h;
  }
  return g_tc_status;
}

int32_t take_tc_status() {
  if (g_tc_status == nullptr) return 0;
  return __atomic_exchange_n(g_tc_status, 0, __ATOMIC_SEQ_CST);
}

// An earlier tensor-core forward whose bounded wait expired left invalid results: report it
// from the next blocked call (the flag is cleared when reported).
int check_tc_status() {
  if (take_tc_status() != 0)
    return fail(TA_ERR_CUDA, "an earlier tcgen05 leaf-block kernel gave up on an expired "
                             "mbarrier wait; its results are invalid");
  return TA_OK;
}
}  // namespace

extern "C" int32_t ta_blocked_set_tcgen05(int32_t enable) {
  const int32_t old = g_use_tcgen05;
  g_use_tcgen05 = enable < 0 ? -1 : (enable ? 1 : 0);
  return old;
}

extern "C" int32_t ta_blocked_set_tcgen05_backward(int32_t enable) {
  const int32_t old = g_use_tcgen05_bwd;
  g_use_tcgen05_bwd = enable ? 1 : 0;
  return old;
}

extern "C" uint64_t ta_blocked_set_tc_wait_ns(uint64_t ns) {
  return g_tc_wait_ns.exchange(ns == 0 ? kTcWaitNs : ns);
}

extern "C" int32_t ta_blocked_status(int32_t clear) {
  if (g_tc_status == nullptr) return 0;
  if (clear) return take_tc_status();
  return *(volatile int32_t*)g_tc_status;
}

extern "C" int32_t ta_blocked_uses_tensor_cores(const ta_shape* shape, const ta_blocked* cfg,
                                               int32_t backward) {
  BlkParams p;
  if (blk_setup(shape, cfg, p) != TA_OK) return 0;
  return backward ? (blk_mma_bwd_ok(p) ? 1 : 0) : (blk_mma_fwd_ok(p) ? 1 : 0);
}

extern "C" size_t ta_blocked_forward_workspace_size(const ta_shape* shape, const ta_blocked* cfg) {
  BlkParams p;
  if (blk_setup(shape, cfg, p) != TA_OK) return 0;
  return blk_mma_fwd_ok(p) ? blk_fwd_ws(p).total : 0;
}

extern "C" int ta_blocked_forward(const ta_shape* shape, const ta_blocked* cfg, const void* q,
                                  ta_layout ql, const void* k, ta_layout kl, const void* v,
                                  ta_layout vl, const float* summaries, void* out, ta_layout ol,
                                  const ta_rng* rng, const float* gumbels, int32_t* block,
                                  float* weights, float* path_out, void* ws, size_t ws_bytes,
                                  ta_stream_t stream) {
  BlkParams p;
  int rc = check_tc_status();
  if (rc) return rc;
  if ((rc = blk_setup(shape, cfg, p))) return rc;
  if ((rc = blk_views(shape, p, q, ql, k, kl, v, vl))) return rc;
  if ((rc = check_view("out", out, ol, dtype_size(shape->dtype), false))) return rc;
  if (!block || !weights || (p.R > 0 && !summaries))
    return fail(TA_ERR_INVALID, "block, weights and summaries must not be NULL");
  if ((rc = blk_noise(p, rng, gumbels))) return rc;
  p.summ = const_cast<float*>(summaries);
  p.out = (char*)out; p.os = ol.seq; p.ob = ol.batch; p.oh = ol.head;
  p.blk = block; p.weights = weights;
  BwdParams sp{};
  if (path_out != nullptr) {
    if (!blk_mma_fwd_ok(p))
      return fail(TA_ERR_UNSUPPORTED, "path_out given but this shape has no tensor-core path "
                                      "(ta_blocked_uses_tensor_cores)");
    const BlkWs w = blk_fwd_ws(p);
    if (!ws || ws_bytes < w.total) return fail(TA_ERR_WORKSPACE, "blocked forward workspace too small");
    p.path_out = path_out;
    // measured per forward: tcgen05 2.71 vs mma.sync 3.61 ms at leaf block 128 (config 3),
    // 0.65 vs 0.55 ms at leaf block 64 (config 2)
    p.use_tcgen05 = g_use_tcgen05 < 0 ? (p.Lb == 128 ? 1 : 0) : g_use_tcgen05;
    if (p.use_tcgen05) {
      int32_t* word = tc_status_word();
      void* dword = nullptr;
      if (word == nullptr || cudaHostGetDevicePointer(&dword, word, 0) != cudaSuccess) {
        cudaGetLastError();
        return fail(TA_ERR_CUDA, "cannot map the tcgen05 status word");
      }
      p.status = (volatile int32_t*)dword;
      p.wait_ns = g_tc_wait_ns.load();
    }
    p.keys0 = (uint32_t*)((char*)ws + w.keys[0]);
    p.vals0 = (uint32_t*)((char*)ws + w.vals[0]);
    if (p.R > 0) p.summ_split = (uint16_t*)((char*)ws + w.split);
    p.ranges = (uint32_t*)((char*)ws + w.ranges);
    sp = blk_sort_params(p, (char*)ws, w.keys, w.vals, w.hist);
  }
  cudaStream_t st = (cudaStream_t)stream;
  TA_BLK_DISPATCH(blk_fwd_typed, p, sp, st)
  return TA_OK;
}

extern "C" size_t ta_blocked_backward_workspace_size(const ta_shape* shape, const ta_blocked* cfg) {
  BlkParams p;
  if (blk_setup(shape, cfg, p) != TA_OK) return 0;
  return blk_ws(p, blk_mma_bwd_ok(p)).total;
}

extern "C" int ta_blocked_backward(const ta_shape* shape, const ta_blocked* cfg, const void* q,
                                   ta_layout ql, const void* k, ta_layout kl, const void* v,
                                   ta_layout vl, const float* summaries, const void* grad_out,
                                   ta_layout gl, const int32_t* block, const float* weights,
                                   const float* path_out, void* dq, ta_layout dql, void* dk,
                                   ta_layout dkl, void* dv, ta_layout dvl, void* ws,
                                   size_t ws_bytes, ta_stream_t stream) {
  BlkParams p;
  int rc = check_tc_status();
  if (rc) return rc;
  if ((rc = blk_setup(shape, cfg, p))) return rc;
  if ((rc = blk_views(shape, p, q, ql, k, kl, v, vl))) return rc;
  const int es = dtype_size(shape->dtype);
  if ((rc = check_view("grad_out", grad_out, gl, es, false)) || (rc = check_view("dq", dq, dql, es, false)) ||
      (rc = check_view("dk", dk, dkl, es, false)) || (rc = check_view("dv", dv, dvl, es, false)))
    return rc;
  if (!block || !weights || (p.R > 0 && !summaries))
    return fail(TA_ERR_INVALID, "block, weights and summaries must not be NULL");
  const bool mma = path_out != nullptr && blk_mma_bwd_ok(p);
  if (!mma && (int64_t)p.Lb * p.D > kAccRegs * kBlockThreads)
    return fail(TA_ERR_UNSUPPORTED, "leaf_block * head_dim > %d", kAccRegs * kBlockThreads);
  if ((int64_t)p.Dp * p.f * p.D > kSumRegs * kBlockThreads)
    return fail(TA_ERR_UNSUPPORTED, "levels * fanout * head_dim > %d", kSumRegs * kBlockThreads);
  const BlkWs w = blk_ws(p, mma);
  if (!ws || ws_bytes < w.total) return fail(TA_ERR_WORKSPACE, "blocked backward workspace too small");
  char* base = (char*)ws;
  p.dout = (const char*)grad_out; p.gs = gl.seq; p.gb = gl.batch; p.gh = gl.head;
  p.summ = const_cast<float*>(summaries);
  p.blk = const_cast<int32_t*>(block); p.weights = const_cast<float*>(weights);
  p.dq = (char*)dq; p.dqs = dql.seq; p.dqb = dql.batch; p.dqh = dql.head;
  p.dk = (char*)dk; p.dks = dkl.seq; p.dkb = dkl.batch; p.dkh = dkl.head;
  p.dv = (char*)dv; p.dvs = dvl.seq; p.dvb = dvl.batch; p.dvh = dvl.head;
  if (mma) {
    p.path_out = const_cast<float*>(path_out);  // 16-bit rows, then the lse (see the header)
    p.delta = (float*)(base + w.delta); p.dq_tree = (float*)(base + w.dq_tree);
    p.dq_path = base + w.dq_path;
    p.ranges = (uint32_t*)(base + w.ranges);
    if (p.R > 0) p.summ_split = (uint16_t*)(base + w.split);
    p.use_tcgen05_bwd = g_use_tcgen05_bwd && blk_tc_bwd_shape(p.Lb, p.D);
    if (p.use_tcgen05_bwd) {
      int32_t* word = tc_status_word();
      void* dword = nullptr;
      if (word == nullptr || cudaHostGetDevicePointer(&dword, word, 0) != cudaSuccess) {
        cudaGetLastError();
        return fail(TA_ERR_CUDA, "cannot map the tcgen05 status word");
      }
      p.status = (volatile int32_t*)dword;
      p.wait_ns = g_tc_wait_ns.load();
    }
  } else {
    p.ds_rows = (float*)(base + w.ds); p.wp_rows = (float*)(base + w.wp);
  }
  p.dz_rows = (float*)(base + w.dz);
  p.keys0 = (uint32_t*)(base + w.keys[0]); p.vals0 = (uint32_t*)(base + w.vals[0]);
  p.dk_attn = (float*)(base + w.dk_attn); p.dc_part = (float*)(base + w.dc_part); p.dc = (float*)(base + w.dc);
  BwdParams sp = blk_sort_params(p, base, w.keys, w.vals, w.hist);
  cudaStream_t st = (cudaStream_t)stream;
  TA_BLK_DISPATCH(blk_bwd_typed, p, sp, st)
  return TA_OK;
}
