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

// Child logits of node (d, j) for this warp's query: z[i] on every lane, -inf if masked.
template <int EPL>
__device__ __forceinline__ void child_logits(const BlkParams& p, const float* qf, int bh, int d,
                                             int64_t j, int64_t bnd, int lane, float* z) {
  const float* base = p.summ + ((int64_t)bh * p.R + p.lvl_off[d + 1] + j * p.f) * p.D;
  for (int i = 0; i < p.f; ++i) {
    float acc = 0.0f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc = fmaf(qf[e], base[(int64_t)i * p.D + lane * EPL + e], acc);
    z[i] = warp_sum(acc);
  }
  if (p.causal) {
    // keys under child (d+1, f j + i) start at (f j + i) * N / f^(d+1)
    int64_t pw = 1;
    for (int t = 0; t <= d; ++t) pw *= p.f;
    const int64_t cspan = (int64_t)p.N / pw;
    for (int i = 0; i < p.f; ++i)
      if ((j * p.f + i) * cspan > bnd) z[i] = -INFINITY;
  }
}

__device__ __forceinline__ void log_softmax_f(const float* z, int f, float* lsm) {
  float m = -INFINITY;
  for (int i = 0; i < f; ++i) m = fmaxf(m, z[i]);
  float s = 0.0f;
  for (int i = 0; i < f; ++i) s += expf(z[i] - m);
  const float lse = m + logf(s);
  for (int i = 0; i < f; ++i) lsm[i] = z[i] - lse;
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

// ---------------------------------------------------------------------------------------
// noise dump (the same draws the forward makes), [Dp][L][B][H][S][f]
// ---------------------------------------------------------------------------------------
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

// ---------------------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------------------
template <typename T, int EPL>
__global__ void __launch_bounds__(kBlkWarps * 32) blk_fwd_kernel(const BlkParams p) {
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
  float m_run = -INFINITY, z_run = 0.0f, acc[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) acc[e] = 0.0f;
  float my_lp = 0.0f;
  int my_blk = 0;
  for (int s = 0; s < p.S; ++s) {
    int64_t j = 0;
    float lp = 0.0f;
    for (int d = 0; d < p.Dp; ++d) {
      float z[kMaxFanout], lsm[kMaxFanout];
      child_logits<EPL>(p, qf, bh, d, j, bnd, lane, z);
      log_softmax_f(z, p.f, lsm);
      float score = -INFINITY;
      if (lane < p.f && z[lane] > -INFINITY) {
        float zl = -INFINITY;
        for (int i = 0; i < p.f; ++i) if (i == lane) zl = lsm[i];
        score = zl + blk_gumbel(p, b, h, l, d, s, lane);
      }
      int dir = lane;
      // argmax over the f lanes, first maximum on ties
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float so = __shfl_xor_sync(0xffffffffu, score, o);
        const int io = __shfl_xor_sync(0xffffffffu, dir, o);
        if (so > score || (so == score && io < dir)) { score = so; dir = io; }
      }
      float take = 0.0f;
      for (int i = 0; i < p.f; ++i) if (i == dir) take = lsm[i];
      lp += take;
      j = j * p.f + dir;
    }
    float pr[kMaxKeyRegs];
    block_probs<T>(p, s_q, bh, j, bnd, lane, pr);
    float o[EPL];
    block_combine<T, EPL>(p, p.v + ((int64_t)b * p.vb + (int64_t)h * p.vh) * sizeof(T), p.vs, pr, j, lane, o);
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
    if (lane == (s & 31)) { my_lp = lp; my_blk = (int)j; }
    if ((s & 31) == 31 || s == p.S - 1) {
      // flush this group of up to 32 paths' outputs; weights need the final max, so store lp
      const int s0 = s & ~31;
      if (lane <= (s & 31)) {
        const int64_t o_ = (((int64_t)l * p.B + b) * p.H + h) * p.S + s0 + lane;
        p.blk[o_] = my_blk;
        p.weights[o_] = my_lp;
      }
    }
  }
  const float inv = 1.0f / z_run;
  T* orow = reinterpret_cast<T*>(p.out + ((int64_t)l * p.os + (int64_t)b * p.ob + (int64_t)h * p.oh) * sizeof(T));
#pragma unroll
  for (int e = 0; e < EPL; ++e) orow[lane * EPL + e] = static_cast<T>(acc[e] * inv);
  __syncwarp();
  // weights = softmax over the paths' log-probabilities
  for (int s = lane; s < p.S; s += 32) {
    const int64_t o_ = (((int64_t)l * p.B + b) * p.H + h) * p.S + s;
    p.weights[o_] = expf(p.weights[o_] - m_run) * inv;
  }
}

// ---------------------------------------------------------------------------------------
// backward 1: per (query, b, h) -- dq, coefficient rows, sort records
// ---------------------------------------------------------------------------------------
template <typename T, int EPL>
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
  // pass 1: g_s = dO . o_s
  float wg = 0.0f;
  for (int s = 0; s < p.S; ++s) {
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
    const float dlp = w * (g - wg);
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
    // tree levels: dz_i = dlp (onehot_i - softmax_i) over the unmasked children
    int64_t pw = 1;
    for (int t = 0; t < p.Dp; ++t) pw *= p.f;
    int64_t jj = 0;
    for (int d = 0; d < p.Dp; ++d) {
      pw /= p.f;
      const int dir = (int)((j / pw) % p.f);
      float z[kMaxFanout], lsm[kMaxFanout];
      child_logits<EPL>(p, qf, bh, d, jj, bnd, lane, z);
      log_softmax_f(z, p.f, lsm);
      const float* cbase = p.summ + ((int64_t)bh * p.R + p.lvl_off[d + 1] + jj * p.f) * p.D;
      for (int i = 0; i < p.f; ++i) {
        const float sm = z[i] > -INFINITY ? expf(lsm[i]) : 0.0f;
        const float dz = dlp * ((i == dir ? 1.0f : 0.0f) - sm);
#pragma unroll
        for (int e = 0; e < EPL; ++e) dq[e] = fmaf(dz, cbase[(int64_t)i * p.D + lane * EPL + e], dq[e]);
        if (lane == 0) p.dz_rows[prow * p.Dp * p.f + d * p.f + i] = dz;
      }
      jj = jj * p.f + dir;
    }
    if (lane == 0) {
      p.keys0[prow] = (uint32_t)j;
      p.vals0[prow] = (uint32_t)path;
    }
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
    for (int i = threadIdx.x; i < ns * Lb; i += blockDim.x) {
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
      if (r < nacc) {
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
    if (r < nacc) {
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
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t per_head = (int64_t)p.N * p.D;
  if (i >= per_head * p.B * p.H) return;
  const int bh = (int)(i / per_head);
  const int64_t r = i - (int64_t)bh * per_head;
  const int64_t key = r / p.D;
  const int c = (int)(r - key * p.D);
  const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
  float acc = p.dk_attn[((int64_t)bh * p.N + key) * p.D + c];
  int64_t span = p.N;
  for (int d = 1; d <= p.Dp; ++d) {
    span /= p.f;
    const int64_t node = key / span;
    acc = fmaf(p.dc[((int64_t)bh * p.R + p.lvl_off[d] + node) * p.D + c], 0.5f / (float)span, acc);
  }
  reinterpret_cast<T*>(p.dk)[key * p.dks + (int64_t)b * p.dkb + (int64_t)h * p.dkh + c] = static_cast<T>(acc);
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

template <typename T, int EPL>
static int blk_fwd_typed(BlkParams& p, cudaStream_t st) {
  const int lt = (p.L + kBlkWarps - 1) / kBlkWarps;
  const size_t smem = (size_t)kBlkWarps * p.D * sizeof(T);
  TA_PROFILE("blocked_fwd", st);
  blk_fwd_kernel<T, EPL><<<(unsigned)(lt * p.B * p.H), kBlkWarps * 32, smem, st>>>(p);
  return check_launch("blocked forward");
}

template <typename T, int EPL>
static int blk_bwd_typed(BlkParams& p, BwdParams& sp, cudaStream_t st) {
  const int lt = (p.L + kBlkWarps - 1) / kBlkWarps;
  const size_t wbytes = 2 * (size_t)p.D * sizeof(T) + (((size_t)p.S * 4 + 15) & ~(size_t)15);
  {
    TA_PROFILE("blocked_bwd_query", st);
    blk_bwd_query_kernel<T, EPL><<<(unsigned)(lt * p.B * p.H), kBlkWarps * 32, kBlkWarps * wbytes, st>>>(p);
  }
  int rc = check_launch("blocked backward (queries)");
  if (rc) return rc;
  if ((rc = run_sort(sp, st))) return rc;
  p.skeys = sp.keys[sp.sorted_buf];
  p.svals = sp.vals[sp.sorted_buf];
  const int DF = p.Dp * p.f;
  const size_t bsmem = (size_t)8 * (2 * p.D + 2 * p.Lb + DF) * 4;
  {
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
      blk_bwd_node_kernel<<<(unsigned)((m + 255) / 256), 256, 0, st>>>(p, d);
    }
  }
  {
    TA_PROFILE("blocked_bwd_keys", st);
    const int64_t m = (int64_t)p.B * p.H * p.N * p.D;
    blk_bwd_key_kernel<T><<<(unsigned)((m + 255) / 256), 256, 0, st>>>(p);
  }
  return check_launch("blocked backward (keys)");
}

#define TA_BLK_DISPATCH(FN, ...)                                                    \
  switch (p.dtype) {                                                                \
    case TA_F32:                                                                    \
      switch (p.D) {                                                                \
        case 32: return FN<float, 1>(__VA_ARGS__);                                  \
        case 64: return FN<float, 2>(__VA_ARGS__);                                  \
        case 96: return FN<float, 3>(__VA_ARGS__);                                  \
        case 128: return FN<float, 4>(__VA_ARGS__);                                 \
        default: return FN<float, 8>(__VA_ARGS__);                                  \
      }                                                                             \
    case TA_F16:                                                                    \
      switch (p.D) {                                                                \
        case 32: return FN<__half, 1>(__VA_ARGS__);                                 \
        case 64: return FN<__half, 2>(__VA_ARGS__);                                 \
        case 96: return FN<__half, 3>(__VA_ARGS__);                                 \
        case 128: return FN<__half, 4>(__VA_ARGS__);                                \
        default: return FN<__half, 8>(__VA_ARGS__);                                 \
      }                                                                             \
    default:                                                                        \
      switch (p.D) {                                                                \
        case 32: return FN<__nv_bfloat16, 1>(__VA_ARGS__);                          \
        case 64: return FN<__nv_bfloat16, 2>(__VA_ARGS__);                          \
        case 96: return FN<__nv_bfloat16, 3>(__VA_ARGS__);                          \
        case 128: return FN<__nv_bfloat16, 4>(__VA_ARGS__);                         \
        default: return FN<__nv_bfloat16, 8>(__VA_ARGS__);                          \
      }                                                                             \
  }

struct BlkWs {
  size_t keys[2], vals[2], hist, ds, wp, dz, dk_attn, dc_part, dc, total;
};

static BlkWs blk_ws(const BlkParams& p) {
  BlkWs w{};
  const int64_t HB = (int64_t)p.B * p.H;
  const int64_t tiles = (p.P + kSortTile - 1) / kSortTile;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += (bytes + 255) & ~(size_t)255; return o; };
  w.keys[0] = take(HB * p.P * 4); w.keys[1] = take(HB * p.P * 4);
  w.vals[0] = take(HB * p.P * 4); w.vals[1] = take(HB * p.P * 4);
  w.hist = take(HB * kRadix * tiles * 4);
  w.ds = take(HB * p.P * p.Lb * 4);
  w.wp = take(HB * p.P * p.Lb * 4);
  w.dz = take(HB * p.P * (p.Dp * p.f > 0 ? p.Dp * p.f : 1) * 4);
  w.dk_attn = take(HB * p.N * p.D * 4);
  w.dc_part = take(HB * p.nb * (p.Dp * p.f > 0 ? p.Dp * p.f : 1) * p.D * 4);
  w.dc = take(HB * (p.R > 0 ? p.R : 1) * p.D * 4);
  w.total = off;
  return w;
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

extern "C" int ta_blocked_forward(const ta_shape* shape, const ta_blocked* cfg, const void* q,
                                  ta_layout ql, const void* k, ta_layout kl, const void* v,
                                  ta_layout vl, const float* summaries, void* out, ta_layout ol,
                                  const ta_rng* rng, const float* gumbels, int32_t* block,
                                  float* weights, ta_stream_t stream) {
  BlkParams p;
  int rc = blk_setup(shape, cfg, p);
  if (rc) return rc;
  if ((rc = blk_views(shape, p, q, ql, k, kl, v, vl))) return rc;
  if ((rc = check_view("out", out, ol, dtype_size(shape->dtype), false))) return rc;
  if (!block || !weights || (p.R > 0 && !summaries))
    return fail(TA_ERR_INVALID, "block, weights and summaries must not be NULL");
  if ((rc = blk_noise(p, rng, gumbels))) return rc;
  p.summ = const_cast<float*>(summaries);
  p.out = (char*)out; p.os = ol.seq; p.ob = ol.batch; p.oh = ol.head;
  p.blk = block; p.weights = weights;
  cudaStream_t st = (cudaStream_t)stream;
  TA_BLK_DISPATCH(blk_fwd_typed, p, st)
  return TA_OK;
}

extern "C" size_t ta_blocked_backward_workspace_size(const ta_shape* shape, const ta_blocked* cfg) {
  BlkParams p;
  if (blk_setup(shape, cfg, p) != TA_OK) return 0;
  return blk_ws(p).total;
}

extern "C" int ta_blocked_backward(const ta_shape* shape, const ta_blocked* cfg, const void* q,
                                   ta_layout ql, const void* k, ta_layout kl, const void* v,
                                   ta_layout vl, const float* summaries, const void* grad_out,
                                   ta_layout gl, const int32_t* block, const float* weights,
                                   void* dq, ta_layout dql, void* dk, ta_layout dkl, void* dv,
                                   ta_layout dvl, void* ws, size_t ws_bytes, ta_stream_t stream) {
  BlkParams p;
  int rc = blk_setup(shape, cfg, p);
  if (rc) return rc;
  if ((rc = blk_views(shape, p, q, ql, k, kl, v, vl))) return rc;
  const int es = dtype_size(shape->dtype);
  if ((rc = check_view("grad_out", grad_out, gl, es, false)) || (rc = check_view("dq", dq, dql, es, false)) ||
      (rc = check_view("dk", dk, dkl, es, false)) || (rc = check_view("dv", dv, dvl, es, false)))
    return rc;
  if (!block || !weights || (p.R > 0 && !summaries))
    return fail(TA_ERR_INVALID, "block, weights and summaries must not be NULL");
  if ((int64_t)p.Lb * p.D > kAccRegs * kBlockThreads)
    return fail(TA_ERR_UNSUPPORTED, "leaf_block * head_dim > %d", kAccRegs * kBlockThreads);
  if ((int64_t)p.Dp * p.f * p.D > kSumRegs * kBlockThreads)
    return fail(TA_ERR_UNSUPPORTED, "levels * fanout * head_dim > %d", kSumRegs * kBlockThreads);
  const BlkWs w = blk_ws(p);
  if (!ws || ws_bytes < w.total) return fail(TA_ERR_WORKSPACE, "blocked backward workspace too small");
  char* base = (char*)ws;
  p.dout = (const char*)grad_out; p.gs = gl.seq; p.gb = gl.batch; p.gh = gl.head;
  p.summ = const_cast<float*>(summaries);
  p.blk = const_cast<int32_t*>(block); p.weights = const_cast<float*>(weights);
  p.dq = (char*)dq; p.dqs = dql.seq; p.dqb = dql.batch; p.dqh = dql.head;
  p.dk = (char*)dk; p.dks = dkl.seq; p.dkb = dkl.batch; p.dkh = dkl.head;
  p.dv = (char*)dv; p.dvs = dvl.seq; p.dvb = dvl.batch; p.dvh = dvl.head;
  p.ds_rows = (float*)(base + w.ds); p.wp_rows = (float*)(base + w.wp); p.dz_rows = (float*)(base + w.dz);
  p.keys0 = (uint32_t*)(base + w.keys[0]); p.vals0 = (uint32_t*)(base + w.vals[0]);
  p.dk_attn = (float*)(base + w.dk_attn); p.dc_part = (float*)(base + w.dc_part); p.dc = (float*)(base + w.dc);
  BwdParams sp{};
  sp.keys[0] = (uint32_t*)(base + w.keys[0]); sp.keys[1] = (uint32_t*)(base + w.keys[1]);
  sp.vals[0] = (uint32_t*)(base + w.vals[0]); sp.vals[1] = (uint32_t*)(base + w.vals[1]);
  sp.hist = (uint32_t*)(base + w.hist);
  sp.B = p.B; sp.H = p.H; sp.P = p.P;
  sp.tiles_per_seg = (int32_t)((p.P + kSortTile - 1) / kSortTile);
  int bits = 0;
  while ((1ll << bits) < p.nb) ++bits;
  sp.log_n = bits > 0 ? bits : 1;
  cudaStream_t st = (cudaStream_t)stream;
  TA_BLK_DISPATCH(blk_bwd_typed, p, sp, st)
  return TA_OK;
}
