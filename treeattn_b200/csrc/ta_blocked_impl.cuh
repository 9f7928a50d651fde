// Generalised tree attention (fanout, leaf blocks): kernels and typed launchers, shared by
// ta_blocked.cu (entry points) and the per-(dtype, fanout) instantiation units
// ta_blocked_<dtype>_f<fanout>.cu, which split the compile across processes.
#pragma once

#include <atomic>
#include <type_traits>

// Generalised tree attention: fanout f, leaf blocks of Lb keys (sm_100a).
//
// No counterpart in the reference (its tree is binary with one key per leaf); at f = 2,
// Lb = 1 it reduces to the reference sampler on the tree-correct node layout (two children
// scored by softmax(q . c_L, q . c_R) = (logsigmoid, logsigmoid(-)) of q . (c_L - c_R), with
// c_L - c_R the Haar difference), and a one-key leaf block returns that key's value.
//
// Tree over nb = N / Lb = f^Dp leaf blocks. Node (d, j) covers blocks [j f^(Dp-d),
// (j+1) f^(Dp-d)); its summary c(d, j) = mean of its keys / 2 (float32, levels 1..Dp stored
// head-major [B*H][R][D]). A sampled path scores the f children of its node at every level
// (z_i = q . c_i; causal queries mask children whose first key is beyond the boundary),
// draws dir = argmax(log_softmax(z) + G) and accumulates lp; at its leaf block it attends
// softmax(scale q . K_blk^T) V_blk. out = sum_s softmax(lp)_s o_s.
//
// Noise: counter-based philox keyed by the GLOBAL (batch, head, query) -- subsequence
// (b * H + h) * L + l -- so sharded and sequence-parallel runs draw exactly what one
// unsharded call draws; element (level, sample, child) is offset + level*S*f + s*f + i.
//
// Forward: one warp per (query, b, h); each path's child scores are warp-reduced dots, its
// leaf block is scored with lanes over keys and summed into the output with lanes over d;
// paths are combined with an online softmax.
// Backward, deterministic (no float atomics): a per-query pass recomputes every path and
// writes dq plus per-path coefficient rows; paths are sorted by leaf block per head; one CTA
// per leaf block reduces dK/dV of its keys and the summary gradients of the levels above
// in sorted order; per-node and per-key passes finish dK.

#include "ta_backward_kernels.cuh"
#include "ta_blocked_mma.cuh"
#include "ta_blocked_tc.cuh"
#include "ta_blocked_tc_bwd.cuh"
#include "ta_rng.cuh"

namespace ta {

int run_sort(BwdParams& p, cudaStream_t st);

constexpr int kBlkWarps = 8;
constexpr int kMaxFanout = 16;
constexpr int kBlkMaxLevels = 16;
constexpr int kMaxKeyRegs = 8;     // Lb <= 256: keys per lane in the leaf-block pass
constexpr int kBlockThreads = 256;
constexpr int kAccRegs = 64;       // Lb * D / 256 per accumulator (dK, dV) in the block pass
constexpr int kSumRegs = 16;       // Dp * f * D / 256 summary-gradient partials per thread

struct BlkParams {
  const char* q; const char* k; const char* v; const char* dout;
  int64_t qs, qb, qh, ks, kb, kh, vs, vb, vh, gs, gb, gh;
  char* out; int64_t os, ob, oh;
  float* summ;                  // [B*H][R][D] float32
  int64_t lvl_off[kBlkMaxLevels + 1];  // row of node (d, 0) in a head's block, d = 1..Dp
  int64_t R;
  int32_t B, H, L, N, D, S, f, Lb, Dp, nb, causal;
  float scale;
  uint64_t seed, offset;
  const float* gumbels;         // optional [Dp][L][B][H][S][f]
  int64_t row0, row_total, batch0, batch_total, head0, head_total;
  int32_t* blk; float* weights; // [L][B][H][S]
  // backward
  char* dq; int64_t dqs, dqb, dqh;
  char* dk; int64_t dks, dkb, dkh;
  char* dv; int64_t dvs, dvb, dvh;
  float* ds_rows;   // [B*H][P][Lb]  scale * dS
  float* wp_rows;   // [B*H][P][Lb]  w_s * P
  float* dz_rows;   // [B*H][P][Dp*f]
  uint32_t* keys0; uint32_t* vals0;
  const uint32_t* skeys; const uint32_t* svals;
  float* dk_attn;   // [B*H][N][D]
  float* dc_part;   // [B*H][nb][Dp*f][D]
  float* dc;        // [B*H][R][D]
  int64_t P;        // L * S
  int32_t dtype;
  // tensor-core leaf-block path
  int32_t sample_only;   // forward: tree walk only (weights = softmax, sort records)
  int32_t summary_only;  // backward block pass: summary gradients only
  void* path_out;        // [B*H][P][D] w_s o_s in the input dtype, then [B*H][P] float lse
  float* delta;          // [B*H][P]
  float* dq_tree;        // [L][B][H][D] float32 tree part of dq
  void* dq_path;         // [B*H][P][D] input dtype
  volatile int32_t* status;  // tensor-core wait status word (mapped host memory)
  uint64_t wait_ns;          // bound of one tensor-core mbarrier wait
  int32_t use_tcgen05;   // leaf-block forward on tcgen05 (else mma.sync)
  int32_t use_tcgen05_bwd;  // leaf-block backward on tcgen05 where its shape allows
  uint32_t* ranges;          // [B*H][nb + 1] first sorted pair of each leaf block
  uint16_t* summ_split;      // [2][B*H][RP][D] summaries as 16-bit high / low parts (or null)
};

template <typename T, int EPL>
__device__ __forceinline__ void ld_slice(const char* row, int lane, float* f) {
  const T* r = reinterpret_cast<const T*>(row) + lane * EPL;
#pragma unroll
  for (int e = 0; e < EPL; ++e) f[e] = static_cast<float>(r[e]);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Gumbel of (level, sample, child) for the query's global (b, h, l).
__device__ __forceinline__ float blk_gumbel(const BlkParams& p, int b, int h, int l, int d, int s, int i) {
  if (p.gumbels != nullptr)
    return p.gumbels[((((int64_t)d * p.L + l) * p.B + b) * p.H + h) * (int64_t)p.S * p.f +
                     (int64_t)s * p.f + i];
  const uint64_t sub = ((uint64_t)(p.batch0 + b) * p.head_total + (uint64_t)(p.head0 + h)) *
                           (uint64_t)p.row_total + (uint64_t)(p.row0 + l);
  const uint64_t e = (uint64_t)d * p.S * p.f + (uint64_t)s * p.f + (uint64_t)i;
  curandStatePhilox4_32_10_t st;
  curand_init(p.seed, sub, p.offset + 4ull * (e >> 2), &st);
  const float4 u4 = _curand_uniform4(st.output);
  const uint32_t c = (uint32_t)(e & 3);
  const float u = c == 0 ? u4.x : c == 1 ? u4.y : c == 2 ? u4.z : u4.w;
  return gumbel_from_uniform(u);
}

__device__ __forceinline__ int64_t blk_boundary(const BlkParams& p, int l) {
  return (int64_t)(p.row0 + l) + p.N - p.row_total;  // bottom-right aligned
}




// Sum of 32 per-lane partial values v[0..31] over the warp such that lane t ends with the
// full sum of slot t: five exchange rounds of halving width (31 shuffles instead of 160).
__device__ __forceinline__ float warp_transpose_sum(float* v, int lane) {
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
    const bool hi = (lane & w) != 0;
#pragma unroll
    for (int t = 0; t < w; ++t) {
      const float send = hi ? v[t] : v[t + w];
      const float keep = hi ? v[t + w] : v[t];
      v[t] = keep + __shfl_xor_sync(0xffffffffu, send, w);
    }
  }
  return v[0];
}

template <int N>
__device__ __forceinline__ int64_t pick_i64(const int64_t* a, int idx) {
  int64_t r = 0;
#pragma unroll
  for (int i = 0; i < N; ++i) r = i == idx ? a[i] : r;
  return r;
}
template <int N>
__device__ __forceinline__ float pick_f(const float* a, int idx) {
  float r = 0.0f;
#pragma unroll
  for (int i = 0; i < N; ++i) r = i == idx ? a[i] : r;
  return r;
}

// Child logits of G = 32 / F paths at one level, slot t = s F + i (path s, child i) in lane
// t: the 32 dots are accumulated per lane over its d-slice and fan-in reduced together.
// Masked children (causal) come back as -inf.
template <int EPL, int F>
__device__ __forceinline__ float group_logit(const BlkParams& p, const float* qf, int bh, int d,
                                             const int64_t* j, int64_t cspan, int64_t bnd, int lane) {
  constexpr int G = 32 / F;
  const float* lvl = p.summ + ((int64_t)bh * p.R + p.lvl_off[d + 1]) * p.D + lane * EPL;
  float v[32];
#pragma unroll
  for (int s = 0; s < G; ++s)
#pragma unroll
    for (int i = 0; i < F; ++i) {
      const float* row = lvl + (j[s] * F + i) * p.D;
      float a = 0.0f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) a = fmaf(qf[e], row[e], a);
      v[s * F + i] = a;
    }
  float z = warp_transpose_sum(v, lane);
  const int64_t child = pick_i64<G>(j, lane / F) * F + (lane % F);
  if (p.causal && child * cspan > bnd) z = -INFINITY;
  return z;
}

// log_softmax over the F lanes of this lane's path (segments of F consecutive lanes).
template <int F>
__device__ __forceinline__ float segment_log_softmax(float z) {
  float m = z;
#pragma unroll
  for (int o = 1; o < F; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float e = expf(z - m);
#pragma unroll
  for (int o = 1; o < F; o <<= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
  return z - (m + logf(e));
}

// Walk paths s0 .. s0 + G - 1 of this warp's query down the tree: j[s] = leaf block, lp[s] =
// log-probability (paths >= S are walked but never used).
template <int EPL, int F>
__device__ __forceinline__ void walk_group(const BlkParams& p, const float* qf, int bh, int b, int h,
                                           int l, int64_t bnd, int s0, int lane, int64_t* j, float* lp) {
  constexpr int G = 32 / F;
#pragma unroll
  for (int s = 0; s < G; ++s) { j[s] = 0; lp[s] = 0.0f; }
  const int ms = lane / F, mi = lane % F;
  int64_t cspan = p.N;
  for (int d = 0; d < p.Dp; ++d) {
    cspan /= F;
    const float z = group_logit<EPL, F>(p, qf, bh, d, j, cspan, bnd, lane);
    const float lsm = segment_log_softmax<F>(z);
    float score = -INFINITY;
    if (s0 + ms < p.S && z > -INFINITY) score = lsm + blk_gumbel(p, b, h, l, d, s0 + ms, mi);
    int dir = mi;
#pragma unroll
    for (int o = 1; o < F; o <<= 1) {  // argmax in the segment, first maximum on ties
      const float so = __shfl_xor_sync(0xffffffffu, score, o);
      const int io = __shfl_xor_sync(0xffffffffu, dir, o);
      if (so > score || (so == score && io < dir)) { score = so; dir = io; }
    }
    const float take = __shfl_sync(0xffffffffu, lsm, (lane & ~(F - 1)) + dir);
#pragma unroll
    for (int s = 0; s < G; ++s) {
      const int ds = __shfl_sync(0xffffffffu, dir, s * F);
      lp[s] += __shfl_sync(0xffffffffu, take, s * F);
      j[s] = j[s] * F + ds;
    }
  }
}

// Scores of this warp's leaf block (lanes over keys, kk = lane + 32 m) and their softmax.
template <typename T>
__device__ __forceinline__ void block_probs(const BlkParams& p, const uint4* s_q, int bh, int64_t j,
                                            int64_t bnd, int lane, float* pr) {
  const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const int nch = p.D * (int)sizeof(T) / 16;
  float mx = -INFINITY;
#pragma unroll
  for (int m = 0; m < kMaxKeyRegs; ++m) {
    const int kk = lane + 32 * m;
    float a = -INFINITY;
    if (kk < p.Lb) {
      const int64_t key = j * p.Lb + kk;
      const char* krow = p.k + (key * p.ks + (int64_t)b * p.kb + (int64_t)h * p.kh) * sizeof(T);
      float acc = 0.0f;
      for (int c = 0; c < nch; ++c) acc = Dot<T>::chunk(s_q[c], ldg16(krow + c * 16), acc);
      a = (p.causal && key > bnd) ? -INFINITY : p.scale * acc;
    }
    pr[m] = a;
    mx = fmaxf(mx, a);
  }
  mx = warp_max(mx);
  float sum = 0.0f;
#pragma unroll
  for (int m = 0; m < kMaxKeyRegs; ++m) {
    pr[m] = lane + 32 * m < p.Lb ? expf(pr[m] - mx) : 0.0f;
    sum += pr[m];
  }
  sum = warp_sum(sum);
  const float inv = 1.0f / sum;
#pragma unroll
  for (int m = 0; m < kMaxKeyRegs; ++m) pr[m] *= inv;
}

// o[e] = sum_k P_k * row_k[lane * EPL + e] over the block's keys (lanes over d).
template <typename T, int EPL>
__device__ __forceinline__ void block_combine(const BlkParams& p, const char* base, int64_t rstride,
                                              const float* pr, int64_t j, int lane, float* o) {
#pragma unroll
  for (int e = 0; e < EPL; ++e) o[e] = 0.0f;
  for (int kk = 0; kk < p.Lb; ++kk) {
    float pk = 0.0f;
#pragma unroll
    for (int m = 0; m < kMaxKeyRegs; ++m)
      if (m == (kk >> 5)) pk = pr[m];
    pk = __shfl_sync(0xffffffffu, pk, kk & 31);
    float vf[EPL];
    ld_slice<T, EPL>(base + (j * p.Lb + kk) * rstride * (int64_t)sizeof(T), lane, vf);
#pragma unroll
    for (int e = 0; e < EPL; ++e) o[e] = fmaf(pk, vf[e], o[e]);
  }
}

// ---------------------------------------------------------------------------------------
// summaries
// ---------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) blk_summary_leaf_kernel(const BlkParams p) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t per_head = (int64_t)p.nb * p.D;
  if (i >= per_head * p.B * p.H) return;
  const int bh = (int)(i / per_head);
  const int64_t r = i - (int64_t)bh * per_head;
  const int64_t j = r / p.D;
  const int c = (int)(r - j * p.D);
  const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const T* kp = reinterpret_cast<const T*>(p.k) + (int64_t)b * p.kb + (int64_t)h * p.kh + c;
  float acc = 0.0f;
  for (int kk = 0; kk < p.Lb; ++kk) acc += static_cast<float>(kp[(j * p.Lb + kk) * p.ks]);
  p.summ[((int64_t)bh * p.R + p.lvl_off[p.Dp] + j) * p.D + c] = acc * (0.5f / (float)p.Lb);
}


// ---------------------------------------------------------------------------------------
// noise dump (the same draws the forward makes), [Dp][L][B][H][S][f]
// ---------------------------------------------------------------------------------------

// ---------------------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------------------
template <typename T, int EPL, int F>
__global__ void __launch_bounds__(kBlkWarps * 32) blk_fwd_kernel(const BlkParams p) {
  constexpr int G = 32 / F;
  extern __shared__ uint4 blk_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lt = (p.L + kBlkWarps - 1) / kBlkWarps;
  const int bh = blockIdx.x / lt;
  const int l = (blockIdx.x - bh * lt) * kBlkWarps + warp;
  if (l >= p.L) return;  // warps are independent: no block-wide barrier below
  const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const int nch = p.D * (int)sizeof(T) / 16;
  uint4* s_q = blk_smem + warp * nch;
  const char* qrow = p.q + ((int64_t)l * p.qs + (int64_t)b * p.qb + (int64_t)h * p.qh) * sizeof(T);
  for (int c = lane; c < nch; c += 32) s_q[c] = ldg16(qrow + c * 16);
  float qf[EPL];
  ld_slice<T, EPL>(qrow, lane, qf);
  __syncwarp();
  const int64_t bnd = blk_boundary(p, l);
  const int64_t o0 = (((int64_t)l * p.B + b) * p.H + h) * p.S;
  float m_run = -INFINITY, z_run = 0.0f, acc[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) acc[e] = 0.0f;
  for (int s0 = 0; s0 < p.S; s0 += G) {
    int64_t jg[G];
    float lpg[G];
    walk_group<EPL, F>(p, qf, bh, b, h, l, bnd, s0, lane, jg, lpg);
#pragma unroll
    for (int sg = 0; sg < G; ++sg) {
      const int s = s0 + sg;
      if (s >= p.S) break;
      const int64_t j = jg[sg];
      const float lp = lpg[sg];
      float o[EPL];
      if (!p.sample_only) {
        float pr[kMaxKeyRegs];
        block_probs<T>(p, s_q, bh, j, bnd, lane, pr);
        block_combine<T, EPL>(p, p.v + ((int64_t)b * p.vb + (int64_t)h * p.vh) * sizeof(T), p.vs, pr, j, lane, o);
      } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) o[e] = 0.0f;
      }
      // online softmax over the paths
      if (lp > m_run) {
        const float r = expf(m_run - lp);
        z_run *= r;
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[e] *= r;
        m_run = lp;
      }
      const float w = expf(lp - m_run);
      z_run += w;
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[e] = fmaf(w, o[e], acc[e]);
    }
    // this group's leaf blocks and log-probabilities (weights need the final max)
    if (lane < G && s0 + lane < p.S) {
      const int s = s0 + lane;
      const int64_t j = pick_i64<G>(jg, lane);
      p.blk[o0 + s] = (int32_t)j;
      p.weights[o0 + s] = pick_f<G>(lpg, lane);
      if (p.sample_only) {
        const int64_t prow = (int64_t)bh * p.P + (int64_t)l * p.S + s;
        p.keys0[prow] = (uint32_t)j;
        p.vals0[prow] = (uint32_t)((int64_t)l * p.S + s);
      }
    }
  }
  const float inv = 1.0f / z_run;
  if (!p.sample_only) {
    T* orow = reinterpret_cast<T*>(p.out + ((int64_t)l * p.os + (int64_t)b * p.ob + (int64_t)h * p.oh) * sizeof(T));
#pragma unroll
    for (int e = 0; e < EPL; ++e) orow[lane * EPL + e] = static_cast<T>(acc[e] * inv);
  }
  __syncwarp();
  // weights = softmax over the paths' log-probabilities (each lane rereads its own writes)
  for (int s = lane; s < p.S; s += 32) {
    const int64_t o_ = o0 + s;
    p.weights[o_] = expf(p.weights[o_] - m_run) * inv;
  }
}

// ---------------------------------------------------------------------------------------
// backward 1: per (query, b, h) -- dq, coefficient rows, sort records
// ---------------------------------------------------------------------------------------
template <typename T, int EPL, int F>
__global__ void __launch_bounds__(kBlkWarps * 32) blk_bwd_query_kernel(const BlkParams p) {
  extern __shared__ uint4 blk_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lt = (p.L + kBlkWarps - 1) / kBlkWarps;
  const int bh = blockIdx.x / lt;
  const int l = (blockIdx.x - bh * lt) * kBlkWarps + warp;
  if (l >= p.L) return;
  const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const int nch = p.D * (int)sizeof(T) / 16;
  const int wbytes = 2 * nch * 16 + ((p.S * 4 + 15) & ~15);
  uint4* s_q = reinterpret_cast<uint4*>(reinterpret_cast<char*>(blk_smem) + warp * wbytes);
  uint4* s_g = s_q + nch;
  float* s_gs = reinterpret_cast<float*>(s_g + nch);  // [S] g_s = dO . o_s
  const char* qrow = p.q + ((int64_t)l * p.qs + (int64_t)b * p.qb + (int64_t)h * p.qh) * sizeof(T);
  const char* grow = p.dout + ((int64_t)l * p.gs + (int64_t)b * p.gb + (int64_t)h * p.gh) * sizeof(T);
  for (int c = lane; c < nch; c += 32) {
    s_q[c] = ldg16(qrow + c * 16);
    s_g[c] = ldg16(grow + c * 16);
  }
  float qf[EPL], gf[EPL];
  ld_slice<T, EPL>(qrow, lane, qf);
  ld_slice<T, EPL>(grow, lane, gf);
  __syncwarp();
  const int64_t bnd = blk_boundary(p, l);
  const int64_t o0 = (((int64_t)l * p.B + b) * p.H + h) * p.S;
  const char* vbase = p.v + ((int64_t)b * p.vb + (int64_t)h * p.vh) * sizeof(T);
  const char* kbase = p.k + ((int64_t)b * p.kb + (int64_t)h * p.kh) * sizeof(T);
  // pass 1: g_s = dO . o_s (tensor-core path: delta_s = dO . (w_s o_s) from the forward's
  // per-path rows, dlp_s = delta_s - w_s sum_t delta_t)
  float wg = 0.0f;
  const bool mma = p.path_out != nullptr;
  for (int s = 0; mma && s < p.S; ++s) {
    const T* orow = reinterpret_cast<const T*>(p.path_out) + ((int64_t)bh * p.P + (int64_t)l * p.S + s) * p.D;
    float part = 0.0f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) part = fmaf(gf[e], static_cast<float>(orow[lane * EPL + e]), part);
    const float dl = warp_sum(part);
    if (lane == 0) {
      s_gs[s] = dl;
      p.delta[(int64_t)bh * p.P + (int64_t)l * p.S + s] = dl;
    }
    wg += dl;
  }
  for (int s = 0; !mma && s < p.S; ++s) {
    const int64_t j = p.blk[o0 + s];
    float pr[kMaxKeyRegs];
    block_probs<T>(p, s_q, bh, j, bnd, lane, pr);
    float o[EPL];
    block_combine<T, EPL>(p, vbase, p.vs, pr, j, lane, o);
    float part = 0.0f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) part = fmaf(gf[e], o[e], part);
    const float g = warp_sum(part);
    if (lane == 0) s_gs[s] = g;
    wg = fmaf(p.weights[o0 + s], g, wg);
  }
  __syncwarp();
  float dq[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) dq[e] = 0.0f;
  const int nchk = p.D * (int)sizeof(T) / 16;
  for (int s = 0; s < p.S; ++s) {
    const int64_t path = (int64_t)l * p.S + s;
    const int64_t prow = (int64_t)bh * p.P + path;
    const int64_t j = p.blk[o0 + s];
    const float w = p.weights[o0 + s];
    __syncwarp();
    const float g = s_gs[s];
    const float dlp = mma ? g - w * wg : w * (g - wg);
    if (!mma) {
    // leaf block: dS_k = P_k (w dO . v_k - w g), dq += scale sum_k dS_k k_k
    float pr[kMaxKeyRegs];
    block_probs<T>(p, s_q, bh, j, bnd, lane, pr);
    float dsr[kMaxKeyRegs];
#pragma unroll
    for (int m = 0; m < kMaxKeyRegs; ++m) {
      const int kk = lane + 32 * m;
      dsr[m] = 0.0f;
      if (kk < p.Lb) {
        const char* vrow = vbase + ((j * p.Lb + kk) * p.vs) * (int64_t)sizeof(T);
        float acc = 0.0f;
        for (int c = 0; c < nchk; ++c) acc = Dot<T>::chunk(s_g[c], ldg16(vrow + c * 16), acc);
        dsr[m] = pr[m] * (w * acc - w * g);
        p.ds_rows[prow * p.Lb + kk] = p.scale * dsr[m];
        p.wp_rows[prow * p.Lb + kk] = w * pr[m];
      }
    }
    for (int kk = 0; kk < p.Lb; ++kk) {
      float dsk = 0.0f;
#pragma unroll
      for (int m = 0; m < kMaxKeyRegs; ++m)
        if (m == (kk >> 5)) dsk = dsr[m];
      dsk = p.scale * __shfl_sync(0xffffffffu, dsk, kk & 31);
      float kf[EPL];
      ld_slice<T, EPL>(kbase + (j * p.Lb + kk) * p.ks * (int64_t)sizeof(T), lane, kf);
#pragma unroll
      for (int e = 0; e < EPL; ++e) dq[e] = fmaf(dsk, kf[e], dq[e]);
    }
    }  // !mma
    __syncwarp();  // every lane has read g_s before lane 0 overwrites it
    if (lane == 0) {
      s_gs[s] = dlp;  // g_s is no longer needed: keep dlp_s for the tree levels
      p.keys0[prow] = (uint32_t)j;
      p.vals0[prow] = (uint32_t)path;
    }
  }
  __syncwarp();
  // tree levels, G paths at a time: dz = dlp (onehot - softmax) over the unmasked children
  {
    constexpr int G = 32 / F;
    const int ms = lane / F, mi = lane % F;
    int64_t top = 1;
    for (int t = 0; t < p.Dp; ++t) top *= F;
    for (int s0 = 0; s0 < p.S; s0 += G) {
      int64_t blk[G], jj[G];
#pragma unroll
      for (int sg = 0; sg < G; ++sg) {
        blk[sg] = s0 + sg < p.S ? (int64_t)p.blk[o0 + s0 + sg] : 0;
        jj[sg] = 0;
      }
      const bool valid = s0 + ms < p.S;
      const float dlp = valid ? s_gs[s0 + ms] : 0.0f;
      const int64_t myblk = pick_i64<G>(blk, ms);
      int64_t pw = top, cspan = p.N;
      for (int d = 0; d < p.Dp; ++d) {
        pw /= F;
        cspan /= F;
        const float z = group_logit<EPL, F>(p, qf, bh, d, jj, cspan, bnd, lane);
        const float lsm = segment_log_softmax<F>(z);
        const int dir = (int)((myblk / pw) % F);
        const float sm = z > -INFINITY ? expf(lsm) : 0.0f;
        const float dz = valid ? dlp * ((mi == dir ? 1.0f : 0.0f) - sm) : 0.0f;
        if (valid)
          p.dz_rows[((int64_t)bh * p.P + (int64_t)l * p.S + s0 + ms) * p.Dp * F + d * F + mi] = dz;
        // dq += sum over the 32 slots of dz_slot * c_slot (this lane's d-slice)
        const float* lvl = p.summ + ((int64_t)bh * p.R + p.lvl_off[d + 1]) * p.D + lane * EPL;
#pragma unroll
        for (int sg = 0; sg < G; ++sg)
#pragma unroll
          for (int i = 0; i < F; ++i) {
            const float c = __shfl_sync(0xffffffffu, dz, sg * F + i);
            const float* row = lvl + (jj[sg] * F + i) * p.D;
#pragma unroll
            for (int e = 0; e < EPL; ++e) dq[e] = fmaf(c, row[e], dq[e]);
          }
#pragma unroll
        for (int sg = 0; sg < G; ++sg) jj[sg] = jj[sg] * F + (blk[sg] / pw) % F;
      }
    }
  }
  if (mma) {  // the leaf-block part of dq comes from the tensor-core pass
    float* dst = p.dq_tree + (((int64_t)l * p.B + b) * p.H + h) * p.D;
#pragma unroll
    for (int e = 0; e < EPL; ++e) dst[lane * EPL + e] = dq[e];
    return;
  }
  T* dqrow = reinterpret_cast<T*>(p.dq + ((int64_t)l * p.dqs + (int64_t)b * p.dqb + (int64_t)h * p.dqh) * sizeof(T));
#pragma unroll
  for (int e = 0; e < EPL; ++e) dqrow[lane * EPL + e] = static_cast<T>(dq[e]);
}

// ---------------------------------------------------------------------------------------
// backward 2: one CTA per (b, h, leaf block), its paths in sorted (= path index) order
// ---------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kBlockThreads) blk_bwd_block_kernel(const BlkParams p) {
  extern __shared__ float sb[];
  constexpr int kStage = 8;
  const int bh = blockIdx.x / p.nb;
  const int j = blockIdx.x - bh * p.nb;
  const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const int D = p.D, Lb = p.Lb, DF = p.Dp * p.f;
  float* s_q = sb;                      // [kStage][D]
  float* s_g = s_q + kStage * D;        // [kStage][D]
  float* s_ds = s_g + kStage * D;       // [kStage][Lb]
  float* s_wp = s_ds + kStage * Lb;     // [kStage][Lb]
  float* s_dz = s_wp + kStage * Lb;     // [kStage][DF]
  __shared__ int64_t range[2];
  const uint32_t* keys = p.skeys + (int64_t)bh * p.P;
  const uint32_t* vals = p.svals + (int64_t)bh * p.P;
  if (threadIdx.x < 2) {
    const uint32_t target = (uint32_t)j + threadIdx.x;
    int64_t lo = 0, hi = p.P;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if (keys[mid] < target) lo = mid + 1; else hi = mid;
    }
    range[threadIdx.x] = lo;
  }
  __syncthreads();
  const int64_t beg = range[0], end = range[1];
  const int nacc = (Lb * D + kBlockThreads - 1) / kBlockThreads;
  const int nsum = (DF * D + kBlockThreads - 1) / kBlockThreads;
  float adk[kAccRegs], adv[kAccRegs], asum[kSumRegs];
#pragma unroll
  for (int r = 0; r < kAccRegs; ++r) { adk[r] = 0.0f; adv[r] = 0.0f; }
#pragma unroll
  for (int r = 0; r < kSumRegs; ++r) asum[r] = 0.0f;
  for (int64_t c0 = beg; c0 < end; c0 += kStage) {
    const int ns = (int)min((int64_t)kStage, end - c0);
    __syncthreads();
    for (int i = threadIdx.x; i < ns * D; i += blockDim.x) {
      const int r = i / D, c = i - r * D;
      const int64_t path = vals[c0 + r];
      const int64_t l = path / p.S;
      s_q[r * D + c] = static_cast<float>(reinterpret_cast<const T*>(p.q)[l * p.qs + (int64_t)b * p.qb + (int64_t)h * p.qh + c]);
      s_g[r * D + c] = static_cast<float>(reinterpret_cast<const T*>(p.dout)[l * p.gs + (int64_t)b * p.gb + (int64_t)h * p.gh + c]);
    }
    for (int i = threadIdx.x; i < (p.summary_only ? 0 : ns * Lb); i += blockDim.x) {
      const int r = i / Lb, c = i - r * Lb;
      const int64_t prow = (int64_t)bh * p.P + vals[c0 + r];
      s_ds[r * Lb + c] = p.ds_rows[prow * Lb + c];
      s_wp[r * Lb + c] = p.wp_rows[prow * Lb + c];
    }
    for (int i = threadIdx.x; i < ns * DF; i += blockDim.x) {
      const int r = i / DF, c = i - r * DF;
      s_dz[r * DF + c] = p.dz_rows[((int64_t)bh * p.P + vals[c0 + r]) * DF + c];
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < kAccRegs; ++r) {
      if (r < nacc && !p.summary_only) {
        const int e = threadIdx.x + r * kBlockThreads;
        if (e < Lb * D) {
          const int kk = e / D, c = e - kk * D;
          float a = adk[r], v = adv[r];
          for (int t = 0; t < ns; ++t) {
            a = fmaf(s_ds[t * Lb + kk], s_q[t * D + c], a);
            v = fmaf(s_wp[t * Lb + kk], s_g[t * D + c], v);
          }
          adk[r] = a;
          adv[r] = v;
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kSumRegs; ++r) {
      if (r < nsum) {
        const int e = threadIdx.x + r * kBlockThreads;
        if (e < DF * D) {
          const int row = e / D, c = e - row * D;
          float a = asum[r];
          for (int t = 0; t < ns; ++t) a = fmaf(s_dz[t * DF + row], s_q[t * D + c], a);
          asum[r] = a;
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kAccRegs; ++r) {
    if (r < nacc && !p.summary_only) {
      const int e = threadIdx.x + r * kBlockThreads;
      if (e < Lb * D) {
        const int kk = e / D, c = e - kk * D;
        const int64_t key = (int64_t)j * Lb + kk;
        p.dk_attn[((int64_t)bh * p.N + key) * D + c] = adk[r];
        reinterpret_cast<T*>(p.dv)[key * p.dvs + (int64_t)b * p.dvb + (int64_t)h * p.dvh + c] = static_cast<T>(adv[r]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kSumRegs; ++r) {
    if (r < nsum) {
      const int e = threadIdx.x + r * kBlockThreads;
      if (e < DF * D) p.dc_part[(((int64_t)bh * p.nb + j) * DF) * D + e] = asum[r];
    }
  }
}

// backward 3: summary gradient of node (d+1, c) = sum over the leaf blocks under its parent
// of the blocks' partials, in block order
template <typename T>
__global__ void __launch_bounds__(256) blk_bwd_node_kernel(const BlkParams p, int d) {
  int64_t rows = p.f;
  for (int t = 0; t < d; ++t) rows *= p.f;  // f^(d+1) children at level d+1
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t per_head = rows * p.D;
  if (i >= per_head * p.B * p.H) return;
  const int bh = (int)(i / per_head);
  const int64_t r = i - (int64_t)bh * per_head;
  const int64_t cnode = r / p.D;
  const int c = (int)(r - cnode * p.D);
  const int64_t parent = cnode / p.f;
  const int ci = (int)(cnode - parent * p.f);
  const int64_t blocks = (int64_t)p.nb * p.f / rows;  // leaf blocks under the parent
  const int DF = p.Dp * p.f;
  const float* src = p.dc_part + ((int64_t)bh * p.nb + parent * blocks) * DF * p.D +
                     (int64_t)(d * p.f + ci) * p.D + c;
  float acc = 0.0f;
  for (int64_t t = 0; t < blocks; ++t) acc += src[t * DF * p.D];
  p.dc[((int64_t)bh * p.R + p.lvl_off[d + 1] + cnode) * p.D + c] = acc;
}

// backward 4: dk[key] = dK of the leaf-block attention + sum over levels of the summary
// gradient of the key's ancestor / (2 * keys under it)
template <typename T>
__global__ void __launch_bounds__(256) blk_bwd_key_kernel(const BlkParams p) {
  // one row (head, key) per D/4 threads, four channels per thread
  const int tpr = p.D >> 2, rpb = 256 / tpr;
  const int rl = threadIdx.x / tpr, c = (threadIdx.x - rl * tpr) * 4;
  if (rl >= rpb) return;
  const int64_t row = (int64_t)blockIdx.x * rpb + rl;
  if (row >= (int64_t)p.B * p.H * p.N) return;
  const int bh = (int)(row / p.N);
  const int64_t key = row - (int64_t)bh * p.N;
  const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
  float4 acc = *reinterpret_cast<const float4*>(p.dk_attn + row * p.D + c);
  // node of `key` at level d: key / (N / f^d), N and f powers of two
  const int ln = __ffsll(p.N) - 1, lf = __ffs(p.f) - 1;
  for (int d = 1; d <= p.Dp; ++d) {
    const int ls = ln - d * lf;
    const int64_t node = key >> ls;
    const float sc = 0.5f / (float)(1ll << ls);
    const float4 v = *reinterpret_cast<const float4*>(p.dc + ((int64_t)bh * p.R + p.lvl_off[d] + node) * p.D + c);
    acc.x = fmaf(v.x, sc, acc.x);
    acc.y = fmaf(v.y, sc, acc.y);
    acc.z = fmaf(v.z, sc, acc.z);
    acc.w = fmaf(v.w, sc, acc.w);
  }
  T* dst = reinterpret_cast<T*>(p.dk) + key * p.dks + (int64_t)b * p.dkb + (int64_t)h * p.dkh + c;
  dst[0] = static_cast<T>(acc.x);
  dst[1] = static_cast<T>(acc.y);
  dst[2] = static_cast<T>(acc.z);
  dst[3] = static_cast<T>(acc.w);
}

// ---------------------------------------------------------------------------------------
// table-lookup walk (tensor-core path): Z = Q_tile C^T for every summary row at once
// ---------------------------------------------------------------------------------------
constexpr int kWalkQ = 32;         // queries per CTA
constexpr int kWalkChunk = 128;    // summary rows per product chunk
constexpr int kWalkMaxRows = 1024; // summary rows the table holds (levels 1..Dp)
constexpr int kWalkRep = 4;         // consecutive query tiles of one head per sampler CTA
constexpr int kBwdWalkRep = 1;      // ... per backward-walk CTA (more tiles per CTA measured slower
                                    // at config 3: 3.39 -> 3.53 ms)

__host__ __device__ inline int walk_rows_pad(int64_t R) { return (int)((R + kWalkChunk - 1) / kWalkChunk) * kWalkChunk; }
__host__ __device__ inline size_t walk_smem(int64_t R, int D, int S) {
  return (size_t)kWalkQ * (walk_rows_pad(R) + 4) * 4    // Z table
         + (size_t)2 * kWalkChunk * (D + 8) * 2          // C chunk, bf16 high and low parts
         + (size_t)kWalkQ * (D + 8) * 2                  // Q tile
         + (size_t)kWalkQ * S * 4;                       // path log-probabilities
}

// The F Gumbels of (level d, path s): the same elements blk_gumbel draws, one philox per
// 4-vector they share.
template <int F>
__device__ __forceinline__ void blk_gumbels_of(const BlkParams& p, int b, int h, int l, int d, int s, float* g) {
  if (p.gumbels != nullptr) {
    const float* src = p.gumbels + ((((int64_t)d * p.L + l) * p.B + b) * p.H + h) * (int64_t)p.S * F +
                       (int64_t)s * F;
#pragma unroll
    for (int i = 0; i < F; ++i) g[i] = src[i];
    return;
  }
  const uint64_t sub = ((uint64_t)(p.batch0 + b) * p.head_total + (uint64_t)(p.head0 + h)) *
                           (uint64_t)p.row_total + (uint64_t)(p.row0 + l);
  const uint64_t e0 = ((uint64_t)d * p.S + (uint64_t)s) * F;
  float4 u4 = make_float4(0.f, 0.f, 0.f, 0.f);
  uint64_t vec = ~0ull;
#pragma unroll
  for (int i = 0; i < F; ++i) {
    const uint64_t e = e0 + i;
    if ((e >> 2) != vec) {
      vec = e >> 2;
      curandStatePhilox4_32_10_t st;
      curand_init(p.seed, sub, p.offset + 4ull * vec, &st);
      u4 = _curand_uniform4(st.output);
    }
    const uint32_t c = (uint32_t)(e & 3);
    g[i] = gumbel_from_uniform(c == 0 ? u4.x : c == 1 ? u4.y : c == 2 ? u4.z : u4.w);
  }
}

// Convert summary rows [r0, r0 + kWalkChunk) of head bh to bf16/fp16 high and low parts in
// shared memory ([row][d], padded rows; rows past R are zero).
template <typename T, int D>
__device__ __forceinline__ void walk_load_chunk(const BlkParams& p, int bh, int r0, uint16_t* s_chi,
                                                uint16_t* s_clo) {
  constexpr int LD = D + 8;
  if (p.summ_split != nullptr) {
    // the rows were split once per call (blk_split_summaries_kernel): 16-byte cp.async copies,
    // completed by the caller's cp_async_wait_0
    constexpr int CPR = D * 2 / 16;
    const int RP = walk_rows_pad(p.R);
    const int64_t half = (int64_t)p.B * p.H * RP * D;
    const uint16_t* hsrc = p.summ_split + ((int64_t)bh * RP + r0) * D;
    for (int i = threadIdx.x; i < kWalkChunk * CPR; i += blockDim.x) {
      const int r = i / CPR, c = i - r * CPR;
      cp_async16(s_chi + r * LD + c * 8, hsrc + (int64_t)r * D + c * 8);
      cp_async16(s_clo + r * LD + c * 8, hsrc + half + (int64_t)r * D + c * 8);
    }
    cp_async_commit();
    return;
  }
  const float* csrc = p.summ + (int64_t)bh * p.R * D;
  for (int i = threadIdx.x; i < kWalkChunk * D / 2; i += blockDim.x) {
    const int r = i / (D / 2), c = (i - r * (D / 2)) * 2;
    float2 v = make_float2(0.f, 0.f);
    if (r0 + r < p.R) v = *reinterpret_cast<const float2*>(csrc + (int64_t)(r0 + r) * D + c);
    const uint32_t hi = Mma<T>::pack(v.x, v.y);
    float2 hf;
    if constexpr (std::is_same<T, __half>::value) {
      hf = __half22float2(*reinterpret_cast<const __half2*>(&hi));
    } else {
      hf = make_float2(__uint_as_float(hi << 16), __uint_as_float(hi & 0xffff0000u));
    }
    *reinterpret_cast<uint32_t*>(s_chi + r * LD + c) = hi;
    *reinterpret_cast<uint32_t*>(s_clo + r * LD + c) = Mma<T>::pack(v.x - hf.x, v.y - hf.y);
  }
}

// summaries [B*H][R][D] float32 -> 16-bit high and low parts [2][B*H][RP][D] (rows >= R zero)
template <typename T>
__global__ void __launch_bounds__(256) blk_split_summaries_kernel(const BlkParams p) {
  const int RP = walk_rows_pad(p.R);
  const int64_t n = (int64_t)p.B * p.H * RP * p.D;
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 2;
  if (i >= n) return;
  const int64_t bh = i / ((int64_t)RP * p.D), rem = i - bh * RP * p.D;
  const int64_t r = rem / p.D, c = rem - r * p.D;
  float2 v = make_float2(0.f, 0.f);
  if (r < p.R) v = *reinterpret_cast<const float2*>(p.summ + (bh * p.R + r) * p.D + c);
  const uint32_t hi = Mma<T>::pack(v.x, v.y);
  float2 hf;
  if constexpr (std::is_same<T, __half>::value) {
    hf = __half22float2(*reinterpret_cast<const __half2*>(&hi));
  } else {
    hf = make_float2(__uint_as_float(hi << 16), __uint_as_float(hi & 0xffff0000u));
  }
  *reinterpret_cast<uint32_t*>(p.summ_split + i) = hi;
  *reinterpret_cast<uint32_t*>(p.summ_split + n + i) = Mma<T>::pack(v.x - hf.x, v.y - hf.y);
}

// Z[q][r] = q . c_r for the CTA's kWalkQ query rows (s_q, 16-bit) and every summary row, on
// the tensor cores with c split into high and low parts (a float32-accurate logit table).
// Waits for the caller's pending cp.async copies (the query rows).
template <typename T, int D>
__device__ __forceinline__ void walk_scores(const BlkParams& p, int bh, const uint16_t* s_q,
                                            uint16_t* s_chi, uint16_t* s_clo, float* s_z, int RP, int ZS,
                                            bool staged = false) {
  constexpr int LD = D + 8;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int m0 = (warp & 1) * 16, nb0 = (warp >> 1) * 32;  // warp: 16 queries x 32 rows of a chunk
  for (int r0 = 0; r0 < RP; r0 += kWalkChunk) {
    __syncthreads();  // the previous chunk's readers are done
    // (a single chunk staged for an earlier query tile of the same head is still in place)
    if (!(staged && RP == kWalkChunk)) walk_load_chunk<T, D>(p, bh, r0, s_chi, s_clo);
    cp_async_wait_0();
    __syncthreads();
    float acc[4][4];
#pragma unroll
    for (int t = 0; t < 4; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;
#pragma unroll
    for (int k0 = 0; k0 < D; k0 += 16) {
      uint32_t a[4];
      frag_a(a, s_q, LD, m0, k0, lane);
#pragma unroll
      for (int t = 0; t < 4; t += 2) {
        uint32_t bb[4];
        frag_b_nk(bb, s_chi, LD, nb0 + t * 8, k0, lane);
        Mma<T>::run(acc[t], a, bb);
        Mma<T>::run(acc[t + 1], a, bb + 2);
        frag_b_nk(bb, s_clo, LD, nb0 + t * 8, k0, lane);
        Mma<T>::run(acc[t], a, bb);
        Mma<T>::run(acc[t + 1], a, bb + 2);
      }
    }
    const int g = lane >> 2, tq = lane & 3;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int c = r0 + nb0 + t * 8 + tq * 2;
      *reinterpret_cast<float2*>(s_z + (m0 + g) * ZS + c) = make_float2(acc[t][0], acc[t][1]);
      *reinterpret_cast<float2*>(s_z + (m0 + g + 8) * ZS + c) = make_float2(acc[t][2], acc[t][3]);
    }
  }
}

template <typename T, int D, int F>
__global__ void __launch_bounds__(256) blk_walk_mma_kernel(const BlkParams p) {
  constexpr int LD = D + 8;
  extern __shared__ __align__(16) unsigned char smraw[];
  const int RP = walk_rows_pad(p.R);
  const int ZS = RP + 4;
  float* s_z = reinterpret_cast<float*>(smraw);                       // [kWalkQ][ZS]
  uint16_t* s_chi = reinterpret_cast<uint16_t*>(s_z + kWalkQ * ZS);   // [kWalkChunk][LD]
  uint16_t* s_clo = s_chi + kWalkChunk * LD;
  uint16_t* s_q = s_clo + kWalkChunk * LD;                            // [kWalkQ][LD]
  float* s_lp = reinterpret_cast<float*>(s_q + kWalkQ * LD);          // [kWalkQ][S]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int lt = (p.L + kWalkQ - 1) / kWalkQ;
  const int ltr = (lt + kWalkRep - 1) / kWalkRep;  // CTAs per head
  const int bh = blockIdx.x / ltr;
  const int tile0 = (blockIdx.x - bh * ltr) * kWalkRep;
  const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
  constexpr int CPR = D * 2 / 16;
  // consecutive query tiles of the head, the summary table staged once
  for (int rep = 0; rep < kWalkRep && tile0 + rep < lt; ++rep) {
  const int l0 = (tile0 + rep) * kWalkQ;
  if (rep > 0) __syncthreads();  // the previous tile's readers are done
  for (int i = tid; i < kWalkQ * CPR; i += blockDim.x) {
    const int r = i / CPR, c = i - r * CPR;
    if (l0 + r < p.L)
      cp_async16(s_q + r * LD + c * 8, p.q + ((int64_t)(l0 + r) * p.qs + (int64_t)b * p.qb + (int64_t)h * p.qh) * 2 + c * 16);
    else
      *reinterpret_cast<uint4*>(s_q + r * LD + c * 8) = make_uint4(0, 0, 0, 0);
  }
  cp_async_commit();
  walk_scores<T, D>(p, bh, s_q, s_chi, s_clo, s_z, RP, ZS, rep > 0);
  __syncthreads();
  // one thread per (query, path): the walk reads its children's logits from the table
  for (int i = tid; i < kWalkQ * p.S; i += blockDim.x) {
    const int qi = i / p.S, s = i - qi * p.S;
    const int l = l0 + qi;
    if (l >= p.L) continue;
    const float* zr = s_z + qi * ZS;
    const int64_t bnd = blk_boundary(p, l);
    int64_t j = 0, cspan = p.N;
    float lp = 0.0f;
    for (int d = 0; d < p.Dp; ++d) {
      cspan /= F;
      const float* zc = zr + p.lvl_off[d + 1] + j * F;
      float z[F], g[F];
      float m = -INFINITY;
#pragma unroll
      for (int c = 0; c < F; ++c) {
        z[c] = (p.causal && (j * F + c) * cspan > bnd) ? -INFINITY : zc[c];
        m = fmaxf(m, z[c]);
      }
      float se = 0.0f;
#pragma unroll
      for (int c = 0; c < F; ++c) se += expf(z[c] - m);
      const float lse = m + logf(se);
      blk_gumbels_of<F>(p, b, h, l, d, s, g);
      int dir = 0;
      float best = -INFINITY;
#pragma unroll
      for (int c = 0; c < F; ++c) {
        const float sc = z[c] > -INFINITY ? (z[c] - lse) + g[c] : -INFINITY;
        if (sc > best) { best = sc; dir = c; }
      }
      float take = 0.0f;
#pragma unroll
      for (int c = 0; c < F; ++c) take = c == dir ? z[c] - lse : take;
      lp += take;
      j = j * F + dir;
    }
    const int64_t o = (((int64_t)l * p.B + b) * p.H + h) * p.S + s;
    p.blk[o] = (int32_t)j;
    s_lp[qi * p.S + s] = lp;
    const int64_t prow = (int64_t)bh * p.P + (int64_t)l * p.S + s;
    p.keys0[prow] = (uint32_t)j;
    p.vals0[prow] = (uint32_t)((int64_t)l * p.S + s);
  }
  __syncthreads();
  // path weights: softmax of each query's path log-probabilities, in path order
  for (int qi = tid; qi < kWalkQ; qi += blockDim.x) {
    const int l = l0 + qi;
    if (l >= p.L) continue;
    float m = -INFINITY;
    for (int s = 0; s < p.S; ++s) m = fmaxf(m, s_lp[qi * p.S + s]);
    float z = 0.0f;
    for (int s = 0; s < p.S; ++s) z += expf(s_lp[qi * p.S + s] - m);
    const float inv = 1.0f / z;
    const int64_t o = (((int64_t)l * p.B + b) * p.H + h) * p.S;
    for (int s = 0; s < p.S; ++s) p.weights[o + s] = expf(s_lp[qi * p.S + s] - m) * inv;
  }
  }  // query tiles
}

// Backward of the tree levels as table lookups (tensor-core path), per 32 queries of a head:
// Z = Q C^T again; per (query, path) thread: delta_s = dO . (w_s o_s), dlp_s = delta_s -
// w_s sum_t delta_t, and per level the children's coefficients dz = dlp (onehot - softmax(z))
// (written per path for the summary gradients); per (query, level) thread: the query's
// coefficient row DZ (paths summed in order); then dq_tree = DZ C on the tensor cores with
// both operands split into high and low parts.
// The Q and dO tiles are dead once delta is formed, so they share one region with the per-path
// delta and dz: delta overlaps the Q tile only (Q is last read by the score product, while the
// delta pass still reads dO), dz follows it.
__host__ __device__ inline size_t bwd_walk_union(int D, int S, int DF) {
  const size_t tiles = (size_t)2 * kWalkQ * (D + 8) * 2;
  const size_t paths = (size_t)kWalkQ * S * 4 + (size_t)kWalkQ * S * DF * 4;
  return tiles > paths ? tiles : paths;
}
__host__ __device__ inline size_t bwd_walk_smem(int64_t R, int D, int S, int DF) {
  return (size_t)kWalkQ * (walk_rows_pad(R) + 4) * 4    // Z table, then DZ
         + (size_t)2 * kWalkChunk * (D + 8) * 2          // C chunk high / low
         + bwd_walk_union(D, S, DF);                     // Q, dO tiles | delta, dz per path
}

template <typename T, int D, int F>
__global__ void __launch_bounds__(256) blk_bwd_walk_mma_kernel(const BlkParams p) {
  constexpr int LD = D + 8;
  extern __shared__ __align__(16) unsigned char smraw[];
  const int RP = walk_rows_pad(p.R);
  const int ZS = RP + 4;
  const int DF = p.Dp * F;
  float* s_z = reinterpret_cast<float*>(smraw);                       // [kWalkQ][ZS]
  uint16_t* s_chi = reinterpret_cast<uint16_t*>(s_z + kWalkQ * ZS);   // [kWalkChunk][LD]
  uint16_t* s_clo = s_chi + kWalkChunk * LD;
  uint16_t* s_q = s_clo + kWalkChunk * LD;                            // [kWalkQ][LD]
  uint16_t* s_g = s_q + kWalkQ * LD;                                  // [kWalkQ][LD]
  float* s_dl = reinterpret_cast<float*>(s_q);                        // [kWalkQ][S] (over Q)
  float* s_dzp = s_dl + kWalkQ * p.S;                                 // [kWalkQ][S][DF]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int lt = (p.L + kWalkQ - 1) / kWalkQ;
  const int ltr = (lt + kBwdWalkRep - 1) / kBwdWalkRep;  // CTAs per head
  const int bh = blockIdx.x / ltr;
  const int tile0 = (blockIdx.x - bh * ltr) * kBwdWalkRep;
  const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
  constexpr int CPR = D * 2 / 16;
  // consecutive query tiles of the head, the summary table staged once
  for (int rep = 0; rep < kBwdWalkRep && tile0 + rep < lt; ++rep) {
  const int l0 = (tile0 + rep) * kWalkQ;
  if (rep > 0) __syncthreads();  // the previous tile's readers are done
  for (int i = tid; i < kWalkQ * CPR; i += blockDim.x) {
    const int r = i / CPR, c = i - r * CPR;
    if (l0 + r < p.L) {
      const int64_t l = l0 + r;
      cp_async16(s_q + r * LD + c * 8, p.q + (l * p.qs + (int64_t)b * p.qb + (int64_t)h * p.qh) * 2 + c * 16);
      cp_async16(s_g + r * LD + c * 8, p.dout + (l * p.gs + (int64_t)b * p.gb + (int64_t)h * p.gh) * 2 + c * 16);
    } else {
      *reinterpret_cast<uint4*>(s_q + r * LD + c * 8) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(s_g + r * LD + c * 8) = make_uint4(0, 0, 0, 0);
    }
  }
  cp_async_commit();
  walk_scores<T, D>(p, bh, s_q, s_chi, s_clo, s_z, RP, ZS, rep > 0);
  __syncthreads();
  // delta_s = dO_q . (w_s o_s)
  for (int i = tid; i < kWalkQ * p.S; i += blockDim.x) {
    const int qi = i / p.S, sp = i - qi * p.S;
    const int64_t l = l0 + qi;
    if (l >= p.L) continue;
    const int64_t prow = (int64_t)bh * p.P + l * p.S + sp;
    const uint2* orow = reinterpret_cast<const uint2*>(reinterpret_cast<const T*>(p.path_out) + prow * D);
    const uint16_t* grow = s_g + qi * LD;
    float dl = 0.0f;
#pragma unroll 4
    for (int c = 0; c < D / 4; ++c) {
      const uint2 o = orow[c];
      dl = fmaf(raw_to_float<T>(grow[4 * c]), raw_to_float<T>((uint16_t)(o.x & 0xFFFFu)), dl);
      dl = fmaf(raw_to_float<T>(grow[4 * c + 1]), raw_to_float<T>((uint16_t)(o.x >> 16)), dl);
      dl = fmaf(raw_to_float<T>(grow[4 * c + 2]), raw_to_float<T>((uint16_t)(o.y & 0xFFFFu)), dl);
      dl = fmaf(raw_to_float<T>(grow[4 * c + 3]), raw_to_float<T>((uint16_t)(o.y >> 16)), dl);
    }
    s_dl[qi * p.S + sp] = dl;
    p.delta[prow] = dl;
  }
  __syncthreads();
  // dlp and the per-level children's coefficients of every path
  float dlp_mine[4];
  int n_mine = 0;
  for (int i = tid; i < kWalkQ * p.S; i += blockDim.x, ++n_mine) {
    const int qi = i / p.S, sp = i - qi * p.S;
    const int64_t l = l0 + qi;
    float tot = 0.0f;
    for (int t = 0; t < p.S; ++t) tot += s_dl[qi * p.S + t];
    float dlp = 0.0f;
    if (l < p.L) {
      const int64_t o = ((l * p.B + b) * p.H + h) * p.S + sp;
      dlp = s_dl[qi * p.S + sp] - p.weights[o] * tot;
    }
    if (n_mine < 4) dlp_mine[n_mine] = dlp;
  }
  __syncthreads();  // every thread has read delta before dlp overwrites it
  n_mine = 0;
  for (int i = tid; i < kWalkQ * p.S; i += blockDim.x, ++n_mine) {
    const int qi = i / p.S, sp = i - qi * p.S;
    const int64_t l = l0 + qi;
    float* dzp = s_dzp + (int64_t)(qi * p.S + sp) * DF;
    if (l >= p.L) {
      for (int e = 0; e < DF; ++e) dzp[e] = 0.0f;
      continue;
    }
    float dlp = 0.0f;
#pragma unroll
    for (int u = 0; u < 4; ++u) dlp = u == n_mine ? dlp_mine[u] : dlp;
    const int64_t prow = (int64_t)bh * p.P + l * p.S + sp;
    const int64_t o = ((l * p.B + b) * p.H + h) * p.S + sp;
    const int64_t blk = p.blk[o];
    const int64_t bnd = blk_boundary(p, (int)l);
    const float* zr = s_z + qi * ZS;
    int64_t pw = 1;
    for (int t = 0; t < p.Dp; ++t) pw *= F;
    int64_t j = 0, cspan = p.N;
    for (int d = 0; d < p.Dp; ++d) {
      pw /= F;
      cspan /= F;
      const int dir = (int)((blk / pw) % F);
      const float* zc = zr + p.lvl_off[d + 1] + j * F;
      float z[F], m = -INFINITY;
#pragma unroll
      for (int c = 0; c < F; ++c) {
        z[c] = (p.causal && (j * F + c) * cspan > bnd) ? -INFINITY : zc[c];
        m = fmaxf(m, z[c]);
      }
      float se = 0.0f;
#pragma unroll
      for (int c = 0; c < F; ++c) se += expf(z[c] - m);
      const float lse = m + logf(se);
#pragma unroll
      for (int c = 0; c < F; ++c) {
        const float sm = z[c] > -INFINITY ? expf(z[c] - lse) : 0.0f;
        const float dz = dlp * ((c == dir ? 1.0f : 0.0f) - sm);
        dzp[d * F + c] = dz;
        p.dz_rows[prow * DF + d * F + c] = dz;
      }
      j = j * F + dir;
    }
    p.keys0[prow] = (uint32_t)blk;
    p.vals0[prow] = (uint32_t)(l * p.S + sp);
  }
  __syncthreads();
  // DZ: the table region becomes the coefficient rows, summed over paths in order
  for (int i = tid; i < kWalkQ * ZS; i += blockDim.x) s_z[i] = 0.0f;
  __syncthreads();
  for (int i = tid; i < kWalkQ * p.Dp; i += blockDim.x) {
    const int qi = i / p.Dp, d = i - qi * p.Dp;
    const int64_t l = l0 + qi;
    if (l >= p.L) continue;
    int64_t pw = 1;
    for (int t = 0; t < p.Dp - d; ++t) pw *= F;  // blocks under a level-d node
    float* dzr = s_z + qi * ZS + p.lvl_off[d + 1];
    const int64_t o = ((l * p.B + b) * p.H + h) * p.S;
    for (int sp = 0; sp < p.S; ++sp) {
      const int64_t jd = p.blk[o + sp] / pw;  // the path's node at level d
      const float* dzp = s_dzp + (int64_t)(qi * p.S + sp) * DF + d * F;
#pragma unroll
      for (int c = 0; c < F; ++c) dzr[jd * F + c] += dzp[c];
    }
  }
  // dq_tree = DZ C: warp w owns queries [16 (w & 1), +16) x columns [(w >> 1) D / 4, +D / 4)
  constexpr int NTW = D / 32;
  const int m0 = (warp & 1) * 16, n0 = (warp >> 1) * (D / 4);
  const int g = lane >> 2, tq = lane & 3;
  float acc[NTW][4];
#pragma unroll
  for (int t = 0; t < NTW; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;
  for (int r0 = 0; r0 < RP; r0 += kWalkChunk) {
    __syncthreads();  // DZ complete / previous chunk consumed
    // (a single chunk is still in shared memory from the score pass)
    if (RP > kWalkChunk) {
      walk_load_chunk<T, D>(p, bh, r0, s_chi, s_clo);
      cp_async_wait_0();
    }
    __syncthreads();
#pragma unroll 2
    for (int k0 = 0; k0 < kWalkChunk; k0 += 16) {
      uint32_t ahi[4], alo[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int row = m0 + g + (u & 1) * 8;
        const int col = r0 + k0 + tq * 2 + (u >> 1) * 8;
        const float2 v = *reinterpret_cast<const float2*>(s_z + row * ZS + col);
        ahi[u] = Mma<T>::pack(v.x, v.y);
        float2 hf;
        if constexpr (std::is_same<T, __half>::value) {
          hf = __half22float2(*reinterpret_cast<const __half2*>(&ahi[u]));
        } else {
          hf = make_float2(__uint_as_float(ahi[u] << 16), __uint_as_float(ahi[u] & 0xffff0000u));
        }
        alo[u] = Mma<T>::pack(v.x - hf.x, v.y - hf.y);
      }
#pragma unroll
      for (int t = 0; t < NTW; t += 2) {
        uint32_t bh_[4], bl_[4];
        frag_b_kn(bh_, s_chi, LD, n0 + t * 8, k0, lane);
        frag_b_kn(bl_, s_clo, LD, n0 + t * 8, k0, lane);
        Mma<T>::run(acc[t], ahi, bh_);
        Mma<T>::run(acc[t + 1], ahi, bh_ + 2);
        Mma<T>::run(acc[t], ahi, bl_);
        Mma<T>::run(acc[t + 1], ahi, bl_ + 2);
        Mma<T>::run(acc[t], alo, bh_);
        Mma<T>::run(acc[t + 1], alo, bh_ + 2);
      }
    }
  }
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int64_t l = l0 + m0 + g + u * 8;
    if (l >= p.L) continue;
    float* dst = p.dq_tree + ((l * p.B + b) * p.H + h) * D + n0;
#pragma unroll
    for (int t = 0; t < NTW; ++t)
      *reinterpret_cast<float2*>(dst + t * 8 + tq * 2) = make_float2(acc[t][2 * u], acc[t][2 * u + 1]);
  }
  }  // query tiles
}

// out[l,b,h] = sum_s path_out[b*H+h][l*S+s] in path order (tensor-core forward); with
// `base` (dq), base[l,b,h] + sum_s. One row (l, b, h) per D/4 threads, four channels each.
template <typename T>
__device__ __forceinline__ void blk_combine_rows(const BlkParams& p, const void* paths_,
                                                 const float* base, char* dst, int64_t ss,
                                                 int64_t sb, int64_t sh) {
  const T* paths = reinterpret_cast<const T*>(paths_);  // per-path rows in the input dtype
  const int tpr = p.D >> 2, rpb = 256 / tpr;
  const int rl = threadIdx.x / tpr, c = (threadIdx.x - rl * tpr) * 4;
  if (rl >= rpb) return;
  const int64_t row = (int64_t)blockIdx.x * rpb + rl;  // (l, b, h)
  if (row >= (int64_t)p.L * p.B * p.H) return;
  const int h = (int)(row % p.H);
  const int64_t lb = row / p.H;
  const int b = (int)(lb % p.B);
  const int64_t l = lb / p.B;
  float4 acc = base ? *reinterpret_cast<const float4*>(base + row * p.D + c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  const T* src = paths + (((int64_t)b * p.H + h) * p.P + l * p.S) * p.D + c;
  if constexpr (sizeof(T) == 2) {  // (the tensor-core paths, the only users, are 16-bit)
    for (int s = 0; s < p.S; ++s) {
      const uint2 v = *reinterpret_cast<const uint2*>(src + (int64_t)s * p.D);
      acc.x += raw_to_float<T>((uint16_t)(v.x & 0xFFFFu));
      acc.y += raw_to_float<T>((uint16_t)(v.x >> 16));
      acc.z += raw_to_float<T>((uint16_t)(v.y & 0xFFFFu));
      acc.w += raw_to_float<T>((uint16_t)(v.y >> 16));
    }
  }
  T* o = reinterpret_cast<T*>(dst) + l * ss + (int64_t)b * sb + (int64_t)h * sh + c;
  o[0] = static_cast<T>(acc.x);
  o[1] = static_cast<T>(acc.y);
  o[2] = static_cast<T>(acc.z);
  o[3] = static_cast<T>(acc.w);
}

template <typename T>
__global__ void __launch_bounds__(256) blk_combine_out_kernel(const BlkParams p) {
  blk_combine_rows<T>(p, p.path_out, nullptr, p.out, p.os, p.ob, p.oh);
}

// dq = tree part + sum_s leaf-block part of path s, in path order
template <typename T>
__global__ void __launch_bounds__(256) blk_combine_dq_kernel(const BlkParams p) {
  blk_combine_rows<T>(p, p.dq_path, p.dq_tree, p.dq, p.dqs, p.dqb, p.dqh);
}

// grid of the row kernels above: `rows` rows of D channels
inline unsigned blk_row_grid(int64_t rows, int D) {
  const int rpb = 256 / (D >> 2);
  return (unsigned)((rows + rpb - 1) / rpb);
}

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------
static int blk_geometry(int64_t N, int32_t f, int32_t Lb, int* Dp, int64_t* nb, int64_t* R,
                        int64_t* off) {
  if (f < 2 || f > kMaxFanout || (f & (f - 1))) return fail(TA_ERR_UNSUPPORTED, "fanout must be a power of two in [2, 16]");
  if (Lb < 1 || Lb > 256 || (Lb & (Lb - 1))) return fail(TA_ERR_UNSUPPORTED, "leaf_block must be a power of two in [1, 256]");
  if (N % Lb) return fail(TA_ERR_INVALID, "num_leaves must be a multiple of leaf_block");
  const int64_t n = N / Lb;
  int d = 0;
  int64_t pw = 1;
  while (pw < n) { pw *= f; ++d; }
  if (pw != n) return fail(TA_ERR_INVALID, "num_leaves / leaf_block = %lld is not a power of the fanout %d", (long long)n, f);
  if (d > kBlkMaxLevels) return fail(TA_ERR_UNSUPPORTED, "tree deeper than %d levels", kBlkMaxLevels);
  *Dp = d;
  *nb = n;
  int64_t rows = 0, width = 1;
  off[0] = 0;
  for (int t = 1; t <= d; ++t) {
    width *= f;
    off[t] = rows;
    rows += width;
  }
  *R = rows;
  return TA_OK;
}

static int blk_setup(const ta_shape* s, const ta_blocked* cfg, BlkParams& p) {
  int rc = check_shape(s, false);
  if (rc) return rc;
  if (!cfg) return fail(TA_ERR_INVALID, "blocked config is NULL");
  const int64_t D = s->head_dim;
  if (D % 32 || D > 256 || D == 160 || D == 192 || D == 224)
    return fail(TA_ERR_UNSUPPORTED, "blocked mode needs head_dim in {32, 64, 96, 128, 256}");
  p = BlkParams{};
  int64_t nb = 0;
  if ((rc = blk_geometry(s->num_leaves, cfg->fanout, cfg->leaf_block, &p.Dp, &nb, &p.R, p.lvl_off)))
    return rc;
  if (cfg->row_total < s->num_queries || cfg->row0 < 0 || cfg->row0 + s->num_queries > cfg->row_total ||
      cfg->batch_total < s->batch || cfg->batch0 < 0 || cfg->batch0 + s->batch > cfg->batch_total ||
      cfg->head_total < s->num_heads || cfg->head0 < 0 || cfg->head0 + s->num_heads > cfg->head_total)
    return fail(TA_ERR_INVALID, "blocked config: query/batch/head block outside its totals");
  if (cfg->causal && cfg->row_total > s->num_leaves)
    return fail(TA_ERR_INVALID, "causal blocked attention needs num_queries <= num_leaves");
  if (!(cfg->softmax_scale > 0.0f)) return fail(TA_ERR_INVALID, "softmax_scale must be > 0");
  p.B = (int32_t)s->batch; p.H = (int32_t)s->num_heads; p.L = (int32_t)s->num_queries;
  p.N = (int32_t)s->num_leaves; p.D = (int32_t)D; p.S = (int32_t)s->num_samples;
  p.f = cfg->fanout; p.Lb = cfg->leaf_block; p.nb = (int32_t)nb; p.causal = cfg->causal ? 1 : 0;
  p.scale = cfg->softmax_scale;
  p.row0 = cfg->row0; p.row_total = cfg->row_total;
  p.batch0 = cfg->batch0; p.batch_total = cfg->batch_total;
  p.head0 = cfg->head0; p.head_total = cfg->head_total;
  p.P = (int64_t)p.L * p.S;
  p.dtype = s->dtype;
  return TA_OK;
}

static int blk_views(const ta_shape* s, BlkParams& p, const void* q, ta_layout ql, const void* k,
                     ta_layout kl, const void* v, ta_layout vl) {
  const int es = dtype_size(s->dtype);
  int rc;
  if ((q && (rc = check_view("q", q, ql, es, false))) || (rc = check_view("k", k, kl, es, false)) ||
      (v && (rc = check_view("v", v, vl, es, false))))
    return rc;
  p.q = (const char*)q; p.qs = ql.seq; p.qb = ql.batch; p.qh = ql.head;
  p.k = (const char*)k; p.ks = kl.seq; p.kb = kl.batch; p.kh = kl.head;
  p.v = (const char*)v; p.vs = vl.seq; p.vb = vl.batch; p.vh = vl.head;
  return TA_OK;
}


static bool blk_mma_fwd_ok(const BlkParams& p) {
  return p.dtype != TA_F32 && (p.D == 64 || p.D == 128) &&
         (p.Lb == 16 || p.Lb == 32 || p.Lb == 64 || p.Lb == 128);
}
static bool blk_mma_bwd_ok(const BlkParams& p) {
  return blk_mma_fwd_ok(p) && p.Lb >= 32 && p.Lb * p.D <= 8192 && p.Dp * p.f <= kDFMax;
}

static BwdParams blk_sort_params(const BlkParams& p, char* base, const size_t* keys,
                                 const size_t* vals, size_t hist) {
  BwdParams sp{};
  sp.keys[0] = (uint32_t*)(base + keys[0]); sp.keys[1] = (uint32_t*)(base + keys[1]);
  sp.vals[0] = (uint32_t*)(base + vals[0]); sp.vals[1] = (uint32_t*)(base + vals[1]);
  sp.hist = (uint32_t*)(base + hist);
  sp.B = p.B; sp.H = p.H; sp.P = p.P;
  sp.tiles_per_seg = (int32_t)((p.P + kSortTile - 1) / kSortTile);
  int bits = 0;
  while ((1ll << bits) < p.nb) ++bits;
  sp.log_n = bits > 0 ? bits : 1;
  return sp;
}

static BlkMmaParams blk_mma_params(const BlkParams& p) {
  BlkMmaParams m{};
  m.q = p.q; m.k = p.k; m.v = p.v; m.dout = p.dout;
  m.qs = p.qs; m.qb = p.qb; m.qh = p.qh; m.ks = p.ks; m.kb = p.kb; m.kh = p.kh;
  m.vs = p.vs; m.vb = p.vb; m.vh = p.vh; m.gs = p.gs; m.gb = p.gb; m.gh = p.gh;
  m.skeys = p.skeys; m.svals = p.svals; m.weights = p.weights; m.path_out = p.path_out;
  m.ranges = p.ranges;
  // the per-pair log-sum-exp follows the [B*H][P][D] rows in the same buffer
  m.lse = p.path_out != nullptr
              ? reinterpret_cast<float*>(static_cast<char*>(p.path_out) + (int64_t)p.B * p.H * p.P * p.D * 2)
              : nullptr;
  m.delta = p.delta; m.dq_path = p.dq_path; m.dk_attn = p.dk_attn;
  m.dz_rows = p.dz_rows; m.dc_part = p.dc_part; m.DF = p.Dp * p.f;
  m.dv = p.dv; m.dvs = p.dvs; m.dvb = p.dvb; m.dvh = p.dvh;
  m.B = p.B; m.H = p.H; m.L = p.L; m.N = p.N; m.S = p.S; m.nb = p.nb; m.causal = p.causal;
  m.P = p.P; m.row0 = p.row0; m.row_total = p.row_total; m.scale = p.scale;
  m.status = p.status;
  m.wait_ns = p.wait_ns;
  return m;
}

template <typename T, int LB, int D>
static void launch_attn_fwd_mma(const BlkMmaParams& m, unsigned grid, cudaStream_t st) {
  constexpr size_t smem = blk_mma_fwd_smem<LB, D>();
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(blk_attn_fwd_mma_kernel<T, LB, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  blk_attn_fwd_mma_kernel<T, LB, D><<<grid, 128, smem, st>>>(m);
}

template <typename T, int LB, int D>
static void launch_attn_bwd_mma(const BlkMmaParams& m, unsigned grid, cudaStream_t st) {
  if constexpr ((LB / 16) * (8 / (LB / 16)) == 8 && (D / (8 / (LB / 16))) % 16 == 0) {
    constexpr size_t smem = blk_mma_bwd_smem<LB, D>();
    cudaFuncSetAttribute(blk_attn_bwd_mma_kernel<T, LB, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    blk_attn_bwd_mma_kernel<T, LB, D><<<grid, 256, smem, st>>>(m);
  }
}

template <typename T, int LB, int D>
static bool launch_attn_bwd_tc(const BlkMmaParams& m, unsigned grid, cudaStream_t st) {
  if constexpr (BlkTcBwdGeom<LB, D>::OK) {
    using G = BlkTcBwdGeom<LB, D>;
    const size_t smem = G::smem(m.DF <= 16 ? 16 : 32);
    if (smem > (size_t)227 * 1024) return false;
    static std::atomic<uint32_t> set_on{0};  // devices whose function attribute is set
    int dev = 0;
    cudaGetDevice(&dev);
    const uint32_t bit = 1u << (dev & 31);
    if (!(set_on.load() & bit)) {
      cudaFuncSetAttribute(blk_attn_bwd_tc_kernel<T, LB, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           227 * 1024);
      set_on.fetch_or(bit);
    }
    blk_attn_bwd_tc_kernel<T, LB, D><<<grid, kTcBwdThreads, smem, st>>>(m);
    return true;
  }
  return false;
}

// the tcgen05 backward covers (leaf block, head_dim) = (128, 64) and (64, 128)
inline bool blk_tc_bwd_shape(int Lb, int D) {
  return (Lb == 128 && D == 64) || (Lb == 64 && D == 128);
}

template <typename T, int LB, int D>
static void launch_attn_fwd_tc(const BlkMmaParams& m, unsigned grid, cudaStream_t st) {
  if constexpr (BlkTcFwdGeom<LB, D>::OK) {
    constexpr size_t smem = BlkTcFwdGeom<LB, D>::SMEM;
    static std::atomic<uint32_t> set_on{0};  // devices whose function attribute is set
    int dev = 0;
    cudaGetDevice(&dev);
    const uint32_t bit = 1u << (dev & 31);
    if (!(set_on.load() & bit)) {
      cudaFuncSetAttribute(blk_attn_fwd_tc_kernel<T, LB, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      set_on.fetch_or(bit);
    }
    blk_attn_fwd_tc_kernel<T, LB, D><<<grid, 256, smem, st>>>(m);
  }
}

template <typename T>
void attn_fwd_mma(const BlkParams& p, cudaStream_t st) {
  const BlkMmaParams m = blk_mma_params(p);
  const unsigned grid = (unsigned)((int64_t)p.B * p.H * p.nb);
  if (p.use_tcgen05 && p.status != nullptr && p.ranges != nullptr) {
    TA_PROFILE("blocked_attn_tc", st);
    const int64_t HB = (int64_t)p.B * p.H;
    const int64_t nr = HB * (p.P + 1);
    blk_block_ranges_kernel<<<(unsigned)((nr + 255) / 256), 256, 0, st>>>(p.skeys, p.P, p.nb, HB, p.ranges);
    if (p.D == 64) {
      switch (p.Lb) {
        case 16: launch_attn_fwd_tc<T, 16, 64>(m, grid, st); break;
        case 32: launch_attn_fwd_tc<T, 32, 64>(m, grid, st); break;
        case 64: launch_attn_fwd_tc<T, 64, 64>(m, grid, st); break;
        default: launch_attn_fwd_tc<T, 128, 64>(m, grid, st); break;
      }
    } else {
      switch (p.Lb) {
        case 16: launch_attn_fwd_tc<T, 16, 128>(m, grid, st); break;
        case 32: launch_attn_fwd_tc<T, 32, 128>(m, grid, st); break;
        case 64: launch_attn_fwd_tc<T, 64, 128>(m, grid, st); break;
        default: launch_attn_fwd_tc<T, 128, 128>(m, grid, st); break;
      }
    }
    return;
  }
  TA_PROFILE("blocked_attn_mma", st);
  if (p.D == 64) {
    switch (p.Lb) {
      case 16: launch_attn_fwd_mma<T, 16, 64>(m, grid, st); break;
      case 32: launch_attn_fwd_mma<T, 32, 64>(m, grid, st); break;
      case 64: launch_attn_fwd_mma<T, 64, 64>(m, grid, st); break;
      default: launch_attn_fwd_mma<T, 128, 64>(m, grid, st); break;
    }
  } else {
    switch (p.Lb) {
      case 16: launch_attn_fwd_mma<T, 16, 128>(m, grid, st); break;
      case 32: launch_attn_fwd_mma<T, 32, 128>(m, grid, st); break;
      case 64: launch_attn_fwd_mma<T, 64, 128>(m, grid, st); break;
      default: launch_attn_fwd_mma<T, 128, 128>(m, grid, st); break;
    }
  }
}

template <typename T>
void attn_bwd_mma(const BlkParams& p, cudaStream_t st) {
  const BlkMmaParams m = blk_mma_params(p);
  const unsigned grid = (unsigned)((int64_t)p.B * p.H * p.nb);
  if (p.use_tcgen05_bwd && p.status != nullptr && p.ranges != nullptr && blk_tc_bwd_shape(p.Lb, p.D) &&
      p.Dp * p.f <= kDFMax) {
    TA_PROFILE("blocked_attn_bwd_tc", st);
    const int64_t HB = (int64_t)p.B * p.H;
    const int64_t nr = HB * (p.P + 1);
    blk_block_ranges_kernel<<<(unsigned)((nr + 255) / 256), 256, 0, st>>>(p.skeys, p.P, p.nb, HB, p.ranges);
    const bool ran = p.D == 64 ? launch_attn_bwd_tc<T, 128, 64>(m, grid, st)
                               : launch_attn_bwd_tc<T, 64, 128>(m, grid, st);
    if (ran) return;
  }
  TA_PROFILE("blocked_attn_bwd_mma", st);
  if (p.D == 64) {
    switch (p.Lb) {
      case 32: launch_attn_bwd_mma<T, 32, 64>(m, grid, st); break;
      case 64: launch_attn_bwd_mma<T, 64, 64>(m, grid, st); break;
      default: launch_attn_bwd_mma<T, 128, 64>(m, grid, st); break;
    }
  } else {
    switch (p.Lb) {
      case 32: launch_attn_bwd_mma<T, 32, 128>(m, grid, st); break;
      default: launch_attn_bwd_mma<T, 64, 128>(m, grid, st); break;
    }
  }
}

template <typename T, int EPL, int F>
int blk_fwd_typed(BlkParams& p, BwdParams& sp, cudaStream_t st) {
  const int lt = (p.L + kBlkWarps - 1) / kBlkWarps;
  const size_t smem = (size_t)kBlkWarps * p.D * sizeof(T);
  const unsigned grid = (unsigned)(lt * p.B * p.H);
  auto launch = [&]() { blk_fwd_kernel<T, EPL, F><<<grid, kBlkWarps * 32, smem, st>>>(p); };
  if (p.path_out == nullptr) {
    TA_PROFILE("blocked_fwd", st);
    launch();
    return check_launch("blocked forward");
  }
  if constexpr (sizeof(T) == 2) {
    p.sample_only = 1;
    {
      TA_PROFILE("blocked_sample", st);
      if constexpr (EPL == 2 || EPL == 4) {
        if (p.R <= kWalkMaxRows) {
          constexpr int D = 32 * EPL;
          const size_t wsm = walk_smem(p.R, D, p.S);
          cudaFuncSetAttribute(blk_walk_mma_kernel<T, D, F>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wsm);
          if (p.summ_split != nullptr) {
            const int64_t ns = (int64_t)p.B * p.H * walk_rows_pad(p.R) * D / 2;
            blk_split_summaries_kernel<T><<<(unsigned)((ns + 255) / 256), 256, 0, st>>>(p);
          }
          const unsigned wg = (unsigned)(((p.L + kWalkQ * kWalkRep - 1) / (kWalkQ * kWalkRep)) * (int64_t)p.B * p.H);
          blk_walk_mma_kernel<T, D, F><<<wg, 256, wsm, st>>>(p);
        } else {
          launch();
        }
      } else {
        launch();
      }
    }
    int rc = check_launch("blocked sampler");
    if (rc) return rc;
    if ((rc = run_sort(sp, st))) return rc;
    p.skeys = sp.keys[sp.sorted_buf];
    p.svals = sp.vals[sp.sorted_buf];
    attn_fwd_mma<T>(p, st);
    if ((rc = check_launch("blocked leaf-block attention"))) return rc;
    {
      TA_PROFILE("blocked_combine", st);
      blk_combine_out_kernel<T><<<blk_row_grid((int64_t)p.L * p.B * p.H, p.D), 256, 0, st>>>(p);
    }
    return check_launch("blocked combine");
  }
  return fail(TA_ERR_UNSUPPORTED, "tensor-core blocked forward needs 16-bit inputs");
}

template <typename T, int EPL, int F>
int blk_bwd_typed(BlkParams& p, BwdParams& sp, cudaStream_t st) {
  const int lt = (p.L + kBlkWarps - 1) / kBlkWarps;
  const size_t wbytes = 2 * (size_t)p.D * sizeof(T) + (((size_t)p.S * 4 + 15) & ~(size_t)15);
  const bool mma = p.path_out != nullptr;
  {
    TA_PROFILE("blocked_bwd_query", st);
    bool done = false;
    if constexpr (sizeof(T) == 2 && (EPL == 2 || EPL == 4)) {
      constexpr int D = 32 * EPL;
      const size_t wsm = bwd_walk_smem(p.R, D, p.S, p.Dp * F);
      if (mma && wsm <= 220 * 1024 && p.S * kWalkQ <= 4 * 256 && p.Dp * F <= kDFMax) {
        cudaFuncSetAttribute(blk_bwd_walk_mma_kernel<T, D, F>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wsm);
        if (p.summ_split != nullptr) {
          const int64_t ns = (int64_t)p.B * p.H * walk_rows_pad(p.R) * D / 2;
          blk_split_summaries_kernel<T><<<(unsigned)((ns + 255) / 256), 256, 0, st>>>(p);
        }
        const unsigned wg = (unsigned)(((p.L + kWalkQ * kBwdWalkRep - 1) / (kWalkQ * kBwdWalkRep)) * (int64_t)p.B * p.H);
        blk_bwd_walk_mma_kernel<T, D, F><<<wg, 256, wsm, st>>>(p);
        done = true;
      }
    }
    if (!done) {
      const unsigned grid = (unsigned)(lt * p.B * p.H);
      const size_t sm = kBlkWarps * wbytes;
      blk_bwd_query_kernel<T, EPL, F><<<grid, kBlkWarps * 32, sm, st>>>(p);
    }
  }
  int rc = check_launch("blocked backward (queries)");
  if (rc) return rc;
  if ((rc = run_sort(sp, st))) return rc;
  p.skeys = sp.keys[sp.sorted_buf];
  p.svals = sp.vals[sp.sorted_buf];
  if (mma) {
    if constexpr (sizeof(T) == 2) attn_bwd_mma<T>(p, st);
    if ((rc = check_launch("blocked leaf-block attention backward"))) return rc;
  }
  const int DF = p.Dp * p.f;
  const size_t bsmem = (size_t)8 * (2 * p.D + 2 * p.Lb + DF) * 4;
  if (!mma) {
    TA_PROFILE("blocked_bwd_block", st);
    if (bsmem > 48 * 1024)
      cudaFuncSetAttribute(blk_bwd_block_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bsmem);
    blk_bwd_block_kernel<T><<<(unsigned)((int64_t)p.B * p.H * p.nb), kBlockThreads, bsmem, st>>>(p);
  }
  if ((rc = check_launch("blocked backward (blocks)"))) return rc;
  {
    TA_PROFILE("blocked_bwd_nodes", st);
    int64_t rows = 1;
    for (int d = 0; d < p.Dp; ++d) {
      rows *= p.f;
      const int64_t m = (int64_t)p.B * p.H * rows * p.D;
      blk_bwd_node_kernel<T><<<(unsigned)((m + 255) / 256), 256, 0, st>>>(p, d);
    }
  }
  {
    TA_PROFILE("blocked_bwd_keys", st);
    blk_bwd_key_kernel<T><<<blk_row_grid((int64_t)p.B * p.H * p.N, p.D), 256, 0, st>>>(p);
  }
  if (mma) {
    TA_PROFILE("blocked_combine", st);
    blk_combine_dq_kernel<T><<<blk_row_grid((int64_t)p.L * p.B * p.H, p.D), 256, 0, st>>>(p);
  }
  return check_launch("blocked backward (keys)");
}

struct BlkWs {
  size_t keys[2], vals[2], hist, ds, wp, dz, dk_attn, dc_part, dc, delta, dq_tree, dq_path, ranges, split, total;
};

// Backward workspace; `mma` = tensor-core leaf-block path (no per-path dS / wP rows, but
// delta, the tree part of dq and per-path dq rows).
static BlkWs blk_ws(const BlkParams& p, bool mma) {
  BlkWs w{};
  const int64_t HB = (int64_t)p.B * p.H;
  const int64_t tiles = (p.P + kSortTile - 1) / kSortTile;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += (bytes + 255) & ~(size_t)255; return o; };
  w.keys[0] = take(HB * p.P * 4); w.keys[1] = take(HB * p.P * 4);
  w.vals[0] = take(HB * p.P * 4); w.vals[1] = take(HB * p.P * 4);
  w.hist = take(HB * kRadix * tiles * 4);
  if (!mma) {
    w.ds = take(HB * p.P * p.Lb * 4);
    w.wp = take(HB * p.P * p.Lb * 4);
  } else {
    w.delta = take(HB * p.P * 4);
    w.dq_tree = take(HB * p.L * p.D * 4);
    w.dq_path = take(HB * p.P * p.D * 2);  // 16-bit rows (the tensor-core paths are 16-bit)
    w.ranges = take(HB * (p.nb + 1) * 4);
    w.split = take((size_t)2 * HB * walk_rows_pad(p.R > 0 ? p.R : 1) * p.D * 2);
  }
  w.dz = take(HB * p.P * (p.Dp * p.f > 0 ? p.Dp * p.f : 1) * 4);
  w.dk_attn = take(HB * p.N * p.D * 4);
  w.dc_part = take(HB * p.nb * (p.Dp * p.f > 0 ? p.Dp * p.f : 1) * p.D * 4);
  w.dc = take(HB * (p.R > 0 ? p.R : 1) * p.D * 4);
  w.total = off;
  return w;
}

// Forward workspace (tensor-core path): the sort of the (query, path) pairs by leaf block.
static BlkWs blk_fwd_ws(const BlkParams& p) {
  BlkWs w{};
  const int64_t HB = (int64_t)p.B * p.H;
  const int64_t tiles = (p.P + kSortTile - 1) / kSortTile;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += (bytes + 255) & ~(size_t)255; return o; };
  w.keys[0] = take(HB * p.P * 4); w.keys[1] = take(HB * p.P * 4);
  w.vals[0] = take(HB * p.P * 4); w.vals[1] = take(HB * p.P * 4);
  w.hist = take(HB * kRadix * tiles * 4);
  w.split = take((size_t)2 * HB * walk_rows_pad(p.R > 0 ? p.R : 1) * p.D * 2);
  w.ranges = take(HB * (p.nb + 1) * 4);
  w.total = off;
  return w;
}


#define TA_BLK_EPLS(X, T, F) X(T, 1, F) X(T, 2, F) X(T, 3, F) X(T, 4, F) X(T, 8, F)
#define TA_BLK_EXTERN(T, EPL, F)                                                        \
  extern template int blk_fwd_typed<T, EPL, F>(BlkParams&, BwdParams&, cudaStream_t);   \
  extern template int blk_bwd_typed<T, EPL, F>(BlkParams&, BwdParams&, cudaStream_t);
#define TA_BLK_INSTANTIATE(T, EPL, F)                                                   \
  template int blk_fwd_typed<T, EPL, F>(BlkParams&, BwdParams&, cudaStream_t);          \
  template int blk_bwd_typed<T, EPL, F>(BlkParams&, BwdParams&, cudaStream_t);
#define TA_BLK_ALL_F(X, T) TA_BLK_EPLS(X, T, 2) TA_BLK_EPLS(X, T, 4) TA_BLK_EPLS(X, T, 8) TA_BLK_EPLS(X, T, 16)
TA_BLK_ALL_F(TA_BLK_EXTERN, float)
TA_BLK_ALL_F(TA_BLK_EXTERN, __half)
TA_BLK_ALL_F(TA_BLK_EXTERN, __nv_bfloat16)
extern template void attn_fwd_mma<__half>(const BlkParams&, cudaStream_t);
extern template void attn_fwd_mma<__nv_bfloat16>(const BlkParams&, cudaStream_t);
extern template void attn_bwd_mma<__half>(const BlkParams&, cudaStream_t);
extern template void attn_bwd_mma<__nv_bfloat16>(const BlkParams&, cudaStream_t);

}  // namespace ta
