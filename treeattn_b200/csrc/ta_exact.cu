// Exact (deterministic) tree attention over all leaves, sm_100a.
//
// Reference: _deterministic_attention (treeattn_torch/_tree_mha.py:271-321). For a query,
// log p(leaf) = sum over the leaf's path of logsigmoid(+-q . k[node]); non-causal weights are
// exp(log p) (they sum to one over a complete tree), causal weights mask leaves n > l + offset
// and softmax over the rest; out = sum_n w_n v_n.
//
// Forward: one CTA per (query, batch, head) computes every node logit (K dots), every leaf's
// weight and the weighted value sum. Backward: the same CTA layout forms two coefficient rows
// per query --
//   W[l][n] = w_n                                     (dV = W^T dO)
//   C[l][node] = sigmoid(-s) DL(left) - sigmoid(s) DL(right)   (dq = C K, dK = C^T Q)
// with dlp_n = w_n (g_n - sum_m w_m g_m) (causal) or w_n g_n (non-causal), g_n = dO . v_n, and
// DL(child) the sum of dlp over the child's leaves -- then three strided GEMMs with a fixed
// summation order produce the gradients (no atomics). Queries are processed in blocks so the
// per-query rows stay within the workspace.

#include <float.h>

#include "ta_common.cuh"

namespace ta {

constexpr int kExactThreads = 256;

struct ExactParams {
  const char* q; const char* k; const char* v; const char* dout;
  int64_t qs, qb, qh, ks, kb, kh, vs, vb, vh, gs, gb, gh;
  char* out; int64_t os, ob, oh;
  float* weights;          // optional (L, B, H, N)
  float* node_buf;         // [QB][B][H][K]: logits, then (backward) subtree sums -> C
  float* leaf_buf;         // [QB][B][H][N]: weights w
  float* dlp_buf;          // [QB][B][H][N]: backward dlp
  int32_t B, H, D, N, log_n, causal;
  int64_t l0, nq;          // query block [l0, l0 + nq)
  int64_t query_offset;    // causal boundary of query l is l + query_offset
  int32_t mode;            // 0: forward (out); 1: weights only; 2: backward coefficients
};

__device__ __forceinline__ float block_reduce_sum(float v, float* s_red) {
  // fixed-order reduction: warp butterflies, then warp sums in warp order
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) s_red[warp] = v;
  __syncthreads();
  float t = 0.0f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += s_red[w];
  return t;
}

__device__ __forceinline__ float block_reduce_max(float v, float* s_red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) s_red[warp] = v;
  __syncthreads();
  float t = -INFINITY;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t = fmaxf(t, s_red[w]);
  return t;
}

template <typename T>
__device__ __forceinline__ float row_dot(const float* a_smem, const char* row, int D) {
  using E = Elem<T>;
  float acc = 0.0f;
  for (int c = 0; c < D; c += E::EPC) {
    float f[E::EPC];
    E::unpack(ldg16(row + c * sizeof(T)), f);
#pragma unroll
    for (int e = 0; e < E::EPC; ++e) acc = fmaf(a_smem[c + e], f[e], acc);
  }
  return acc;
}

template <typename T>
__global__ void __launch_bounds__(kExactThreads) exact_kernel(const ExactParams p) {
  extern __shared__ float sm[];
  float* s_q = sm;                 // [D] query
  float* s_g = sm + p.D;           // [D] grad_out (backward)
  float* s_red = s_g + p.D;        // [32]
  float* s_col = s_red + 32;       // [kExactThreads] column partial sums
  const int64_t lb = blockIdx.x / (p.B * p.H);
  const int bh = (int)(blockIdx.x - lb * p.B * p.H);
  const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const int64_t l = p.l0 + lb;
  const int K = p.N - 1, N = p.N, ln = p.log_n, D = p.D;
  const int tid = threadIdx.x;
  float* sd = p.node_buf + (lb * p.B * p.H + bh) * (int64_t)K;
  float* w = p.leaf_buf + (lb * p.B * p.H + bh) * (int64_t)N;

  const char* qrow = p.q + (l * p.qs + (int64_t)b * p.qb + (int64_t)h * p.qh) * sizeof(T);
  for (int c = tid; c < D; c += blockDim.x) s_q[c] = static_cast<float>(reinterpret_cast<const T*>(qrow)[c]);
  if (p.mode == 2) {
    const char* grow = p.dout + (l * p.gs + (int64_t)b * p.gb + (int64_t)h * p.gh) * sizeof(T);
    for (int c = tid; c < D; c += blockDim.x) s_g[c] = static_cast<float>(reinterpret_cast<const T*>(grow)[c]);
  }
  __syncthreads();
  // node logits
  const char* kbase = p.k + ((int64_t)b * p.kb + (int64_t)h * p.kh) * sizeof(T);
  for (int n = tid; n < K; n += blockDim.x)
    sd[n] = row_dot<T>(s_q, kbase + (int64_t)n * p.ks * sizeof(T), D);
  __syncthreads();
  // leaf log-probabilities (path order: root first, as the reference accumulates)
  const int64_t limit = l + p.query_offset;
  auto leaf_lp = [&](int n) -> float {
    const uint32_t bits = (uint32_t)n;
    float lp = 0.0f;
    for (int d = 0; d < ln; ++d) {
      const int node = (1 << d) - 1 + (int)(bits >> (ln - d));
      float a, c;
      log_sigmoid_pair(sd[node], a, c);
      lp += ((bits >> (ln - 1 - d)) & 1u) ? c : a;
    }
    return lp;
  };
  float lse = 0.0f;
  if (p.causal) {
    float m = -INFINITY;
    for (int n = tid; n < N; n += blockDim.x)
      if (n <= limit) m = fmaxf(m, leaf_lp(n));
    m = block_reduce_max(m, s_red);
    float s = 0.0f;
    for (int n = tid; n < N; n += blockDim.x)
      if (n <= limit) s += expf(leaf_lp(n) - m);
    s = block_reduce_sum(s, s_red);
    lse = m + logf(s);
  }
  for (int n = tid; n < N; n += blockDim.x) {
    float wn;
    if (p.causal) wn = n <= limit ? expf(leaf_lp(n) - lse) : 0.0f;
    else wn = expf(leaf_lp(n));
    w[n] = wn;
    if (p.weights) p.weights[((l * p.B + b) * p.H + h) * (int64_t)N + n] = wn;
  }
  __syncthreads();
  const char* vbase = p.v + ((int64_t)b * p.vb + (int64_t)h * p.vh) * sizeof(T);
  if (p.mode == 1) return;
  if (p.mode == 0) {
    // out[c] = sum_n w_n v[n][c]: groups of D threads split the leaves, then a fixed-order sum
    const int groups = max(1, (int)blockDim.x / D);
    const int gidx = tid / D, c = tid - gidx * D;
    float acc = 0.0f;
    if (gidx < groups && c < D)
      for (int n = gidx; n < N; n += groups)
        acc = fmaf(w[n], static_cast<float>(reinterpret_cast<const T*>(vbase + (int64_t)n * p.vs * sizeof(T))[c]), acc);
    if (D > (int)blockDim.x) {  // wide rows: each thread loops over columns
      for (int cc = tid; cc < D; cc += blockDim.x) {
        float a2 = 0.0f;
        for (int n = 0; n < N; ++n)
          a2 = fmaf(w[n], static_cast<float>(reinterpret_cast<const T*>(vbase + (int64_t)n * p.vs * sizeof(T))[cc]), a2);
        reinterpret_cast<T*>(p.out + (l * p.os + (int64_t)b * p.ob + (int64_t)h * p.oh) * sizeof(T))[cc] = static_cast<T>(a2);
      }
      return;
    }
    s_col[tid] = acc;
    __syncthreads();
    if (tid < D) {
      float t = 0.0f;
      for (int g = 0; g < groups; ++g) t += s_col[g * D + tid];
      reinterpret_cast<T*>(p.out + (l * p.os + (int64_t)b * p.ob + (int64_t)h * p.oh) * sizeof(T))[tid] = static_cast<T>(t);
    }
    return;
  }
  // backward: dlp_n, subtree sums, node coefficients
  float* dl = p.dlp_buf + (lb * p.B * p.H + bh) * (int64_t)N;
  float wg = 0.0f;
  for (int n = tid; n < N; n += blockDim.x) {
    const float g = row_dot<T>(s_g, vbase + (int64_t)n * p.vs * sizeof(T), D);
    dl[n] = g;
    wg += w[n] * g;
  }
  if (p.causal) wg = block_reduce_sum(wg, s_red);
  __syncthreads();
  for (int n = tid; n < N; n += blockDim.x) dl[n] = p.causal ? w[n] * (dl[n] - wg) : w[n] * dl[n];
  __syncthreads();
  // bottom-up over levels: DL(node) = dlp summed over the node's leaves (stored over the
  // weights, which the dV product has already consumed), and the node's coefficient C
  // replaces its logit once both children's sums are known
  float* cb = p.node_buf + (lb * p.B * p.H + bh) * (int64_t)K;
  float* dlnode = w;  // K < N entries
  for (int d = ln - 1; d >= 0; --d) {
    const int first = (1 << d) - 1, cnt = 1 << d;
    for (int i = tid; i < cnt; i += blockDim.x) {
      const int node = first + i;
      float lsum, rsum;
      if (d == ln - 1) {
        lsum = dl[2 * i];
        rsum = dl[2 * i + 1];
      } else {
        lsum = dlnode[2 * node + 1];
        rsum = dlnode[2 * node + 2];
      }
      dlnode[node] = lsum + rsum;
      const float s = cb[node];
      // C = sigmoid(-s) DL(left) - sigmoid(s) DL(right)
      const float sl = 1.0f / (1.0f + expf(s)), sr = 1.0f / (1.0f + expf(-s));
      cb[node] = sl * lsum - sr * rsum;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------------------
// strided batched GEMM, fixed summation order: Y[m][n] (+)= sum_k A[m][k] * B[k][n]
// A float32, B in T, Y float32 or T. One batch per (b, h) of the query block.
// ---------------------------------------------------------------------------------------
struct GemmParams {
  const float* A; int64_t sAm, sAk, sAb, sAh;  // batch strides per b and per h
  const char* Bm; int64_t sBk, sBn, sBb, sBh;  // elements of T
  char* Y; int64_t sYm, sYn, sYb, sYh;         // elements of the output type
  int32_t M, Nn, Kd, H, accumulate, y_f32;
};

template <typename T>
__global__ void __launch_bounds__(256) gemm_kernel(const GemmParams g) {
  __shared__ float sA[16][65];
  __shared__ float sB[16][65];
  const int bh = blockIdx.z;
  const int b = bh / g.H, h = bh - (bh / g.H) * g.H;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const float* A = g.A + (int64_t)b * g.sAb + (int64_t)h * g.sAh;
  const T* Bm = reinterpret_cast<const T*>(g.Bm) + (int64_t)b * g.sBb + (int64_t)h * g.sBh;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < g.Kd; k0 += 16) {
    for (int i = threadIdx.x; i < 16 * 64; i += 256) {
      const int kk = i >> 6, mm = i & 63;
      const int m = m0 + mm, k = k0 + kk;
      sA[kk][mm] = (m < g.M && k < g.Kd) ? A[(int64_t)m * g.sAm + (int64_t)k * g.sAk] : 0.0f;
      const int n = n0 + mm;
      sB[kk][mm] = (n < g.Nn && k < g.Kd) ? static_cast<float>(Bm[(int64_t)k * g.sBk + (int64_t)n * g.sBn]) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], bb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = sA[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bb[j] = sB[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= g.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= g.Nn) continue;
      const int64_t off = (int64_t)b * g.sYb + (int64_t)h * g.sYh + (int64_t)m * g.sYm + (int64_t)n * g.sYn;
      if (g.y_f32) {
        float* y = reinterpret_cast<float*>(g.Y) + off;
        *y = g.accumulate ? *y + acc[i][j] : acc[i][j];
      } else {
        T* y = reinterpret_cast<T*>(g.Y) + off;
        *y = static_cast<T>(g.accumulate ? static_cast<float>(*y) + acc[i][j] : acc[i][j]);
      }
    }
  }
}

template <typename T>
static void launch_gemm(const GemmParams& g, int BH, cudaStream_t st) {
  const dim3 grid((unsigned)((g.Nn + 63) / 64), (unsigned)((g.M + 63) / 64), (unsigned)BH);
  TA_PROFILE("exact_gemm", st);
  gemm_kernel<T><<<grid, 256, 0, st>>>(g);
}

static int64_t exact_block(int64_t L, int64_t B, int64_t H, int64_t N) {
  const int64_t per_query = B * H * (3 * N) * 4;  // node logits/C, weights, dlp (K < N)
  const int64_t budget = (int64_t)512 << 20;
  int64_t qb = budget / per_query;
  if (qb < 1) qb = 1;
  return qb < L ? qb : L;
}

template <typename T>
static int run_exact(ExactParams p, int64_t L, cudaStream_t st, bool backward,
                     const GemmParams* proto, char* dq, ta_layout dql, char* dk, ta_layout dkl,
                     char* dv, ta_layout dvl, int32_t accumulate) {
  const int64_t qb = exact_block(L, p.B, p.H, p.N);
  const size_t smem = (size_t)(2 * p.D + 32 + kExactThreads) * 4;
  for (int64_t l0 = 0; l0 < L; l0 += qb) {
    p.l0 = l0;
    p.nq = qb < L - l0 ? qb : L - l0;
    p.mode = backward ? 1 : 0;
    {
      TA_PROFILE(backward ? "exact_bwd_weights" : "exact_fwd", st);
      exact_kernel<T><<<(unsigned)(p.nq * p.B * p.H), kExactThreads, smem, st>>>(p);
    }
    int rc = check_launch("exact attention");
    if (rc) return rc;
    if (!backward) continue;
    // leaf_buf now holds w; dV (+)= W^T dO for this block
    const int BH = p.B * p.H;
    GemmParams g{};
    g.A = p.leaf_buf; g.sAm = 1; g.sAk = (int64_t)BH * p.N; g.sAb = (int64_t)p.H * p.N; g.sAh = p.N;
    g.Bm = p.dout + (l0 * p.gs) * sizeof(T); g.sBk = p.gs; g.sBn = 1; g.sBb = p.gb; g.sBh = p.gh;
    g.Y = dv; g.sYm = dvl.seq; g.sYn = 1; g.sYb = dvl.batch; g.sYh = dvl.head;
    g.M = p.N; g.Nn = p.D; g.Kd = (int32_t)p.nq; g.H = p.H; g.y_f32 = 1;
    g.accumulate = (accumulate || l0 > 0) ? 1 : 0;
    launch_gemm<T>(g, BH, st);
    // coefficients C for the block
    p.mode = 2;
    {
      TA_PROFILE("exact_bwd_coef", st);
      exact_kernel<T><<<(unsigned)(p.nq * p.B * p.H), kExactThreads, smem, st>>>(p);
    }
    if ((rc = check_launch("exact attention backward"))) return rc;
    const int K = p.N - 1;
    // dq = C K   (rows of this block; written, not accumulated)
    g = GemmParams{};
    g.A = p.node_buf; g.sAm = (int64_t)BH * K; g.sAk = 1; g.sAb = (int64_t)p.H * K; g.sAh = K;
    g.Bm = p.k; g.sBk = p.ks; g.sBn = 1; g.sBb = p.kb; g.sBh = p.kh;
    g.Y = dq + (l0 * dql.seq) * sizeof(T); g.sYm = dql.seq; g.sYn = 1; g.sYb = dql.batch; g.sYh = dql.head;
    g.M = (int32_t)p.nq; g.Nn = p.D; g.Kd = K; g.H = p.H; g.y_f32 = 0; g.accumulate = 0;
    launch_gemm<T>(g, BH, st);
    // dK (+)= C^T Q
    g = GemmParams{};
    g.A = p.node_buf; g.sAm = 1; g.sAk = (int64_t)BH * K; g.sAb = (int64_t)p.H * K; g.sAh = K;
    g.Bm = p.q + (l0 * p.qs) * sizeof(T); g.sBk = p.qs; g.sBn = 1; g.sBb = p.qb; g.sBh = p.qh;
    g.Y = dk; g.sYm = dkl.seq; g.sYn = 1; g.sYb = dkl.batch; g.sYh = dkl.head;
    g.M = K; g.Nn = p.D; g.Kd = (int32_t)p.nq; g.H = p.H; g.y_f32 = 1;
    g.accumulate = (accumulate || l0 > 0) ? 1 : 0;
    launch_gemm<T>(g, BH, st);
    if ((rc = check_launch("exact attention gemm"))) return rc;
  }
  (void)proto;
  return TA_OK;
}

static int exact_checks(const ta_shape* s) {
  int rc = check_shape(s, true);
  if (rc) return rc;
  if (s->head_dim > 1024) return fail(TA_ERR_UNSUPPORTED, "head_dim > 1024");
  return TA_OK;
}

}  // namespace ta

using namespace ta;

extern "C" size_t ta_exact_workspace_size(const ta_shape* shape) {
  if (exact_checks(shape) != TA_OK) return 0;
  const int64_t qb = exact_block(shape->num_queries, shape->batch, shape->num_heads, shape->num_leaves);
  return (size_t)(qb * shape->batch * shape->num_heads * 3 * shape->num_leaves * 4) + 256;
}

static int exact_common(const ta_shape* shape, const void* q, ta_layout ql, const void* k,
                        ta_layout kl, const void* v, ta_layout vl, void* ws, size_t ws_bytes,
                        ExactParams& p) {
  int rc = exact_checks(shape);
  if (rc) return rc;
  const int es = dtype_size(shape->dtype);
  if ((rc = check_view("q", q, ql, es, false)) || (rc = check_view("k_int", k, kl, es, false)) ||
      (rc = check_view("v", v, vl, es, false)))
    return rc;
  if (!ws || ws_bytes < ta_exact_workspace_size(shape))
    return fail(TA_ERR_WORKSPACE, "exact attention workspace too small");
  p = ExactParams{};
  p.q = (const char*)q; p.k = (const char*)k; p.v = (const char*)v;
  p.qs = ql.seq; p.qb = ql.batch; p.qh = ql.head;
  p.ks = kl.seq; p.kb = kl.batch; p.kh = kl.head;
  p.vs = vl.seq; p.vb = vl.batch; p.vh = vl.head;
  p.B = (int32_t)shape->batch; p.H = (int32_t)shape->num_heads; p.D = (int32_t)shape->head_dim;
  p.N = (int32_t)shape->num_leaves; p.log_n = floor_log2(shape->num_leaves);
  const int64_t qb = exact_block(shape->num_queries, p.B, p.H, p.N);
  float* base = (float*)ws;
  p.node_buf = base;
  p.leaf_buf = base + qb * p.B * p.H * (int64_t)p.N;
  p.dlp_buf = p.leaf_buf + qb * p.B * p.H * (int64_t)p.N;
  return TA_OK;
}

extern "C" int ta_exact_forward(const ta_shape* shape, int32_t causal, int64_t query_offset,
                                const void* q, ta_layout ql, const void* k, ta_layout kl,
                                const void* v, ta_layout vl, void* out, ta_layout ol,
                                float* weights, void* ws, size_t ws_bytes, ta_stream_t stream) {
  ExactParams p;
  int rc = exact_common(shape, q, ql, k, kl, v, vl, ws, ws_bytes, p);
  if (rc) return rc;
  if ((rc = check_view("out", out, ol, dtype_size(shape->dtype), false))) return rc;
  p.out = (char*)out; p.os = ol.seq; p.ob = ol.batch; p.oh = ol.head;
  p.weights = weights;
  p.causal = causal ? 1 : 0;
  p.query_offset = query_offset;
  cudaStream_t st = (cudaStream_t)stream;
  switch (shape->dtype) {
    case TA_F32: return run_exact<float>(p, shape->num_queries, st, false, nullptr, nullptr, {}, nullptr, {}, nullptr, {}, 0);
    case TA_F16: return run_exact<__half>(p, shape->num_queries, st, false, nullptr, nullptr, {}, nullptr, {}, nullptr, {}, 0);
    default: return run_exact<__nv_bfloat16>(p, shape->num_queries, st, false, nullptr, nullptr, {}, nullptr, {}, nullptr, {}, 0);
  }
}

extern "C" int ta_exact_backward(const ta_shape* shape, int32_t causal, int64_t query_offset,
                                 const void* q, ta_layout ql, const void* k, ta_layout kl,
                                 const void* v, ta_layout vl, const void* grad_out,
                                 ta_layout gl, void* dq, ta_layout dql, float* dk,
                                 ta_layout dkl, float* dv, ta_layout dvl, int32_t accumulate,
                                 void* ws, size_t ws_bytes, ta_stream_t stream) {
  ExactParams p;
  int rc = exact_common(shape, q, ql, k, kl, v, vl, ws, ws_bytes, p);
  if (rc) return rc;
  const int es = dtype_size(shape->dtype);
  if ((rc = check_view("grad_out", grad_out, gl, es, false)) || (rc = check_view("dq", dq, dql, es, false)) ||
      (rc = check_view("dk", dk, dkl, 4, false)) || (rc = check_view("dv", dv, dvl, 4, false)))
    return rc;
  p.dout = (const char*)grad_out; p.gs = gl.seq; p.gb = gl.batch; p.gh = gl.head;
  p.causal = causal ? 1 : 0;
  p.query_offset = query_offset;
  cudaStream_t st = (cudaStream_t)stream;
  switch (shape->dtype) {
    case TA_F32: return run_exact<float>(p, shape->num_queries, st, true, nullptr, (char*)dq, dql, (char*)dk, dkl, (char*)dv, dvl, accumulate);
    case TA_F16: return run_exact<__half>(p, shape->num_queries, st, true, nullptr, (char*)dq, dql, (char*)dk, dkl, (char*)dv, dvl, accumulate);
    default: return run_exact<__nv_bfloat16>(p, shape->num_queries, st, true, nullptr, (char*)dq, dql, (char*)dk, dkl, (char*)dv, dvl, accumulate);
  }
}
