// Causal stochastic tree attention: sampler with the reference's boundary correction, and
// the coefficients its backward needs (sm_100a).
//
// Reference: _sample_paths_causal (treeattn_torch/_tree_mha.py:125-268). For query t with
// boundary leaf t + offset:
//   pass 1: along the boundary path, M[d] = logsumexp(M[d+1] + lp_on, off_mass + lp_off) with
//           M[log2 N] = 0, the off-path child masked (-inf) when the boundary goes left and
//           counted as log(#leaves of the left subtree) when it goes right;
//   pass 2: sample S paths per (b, h) top-down. At level d, if EVERY sample of the query (all
//           b, h, s) sits on the boundary node, the two branch log-probabilities become
//           m_child + lp - M[d] (m_left/m_right as in pass 1); otherwise they are the raw
//           logsigmoids. One Gumbel draw of B*H*S*2 values per (query, level).
// The "every sample" predicate couples all (b, h) of a query, so one CTA owns one query and
// evaluates the predicate with a block-wide AND between levels.
//
// Backward (coefficient form): every path contributes gl_{p,d} = sgn sigmoid(-sgn s) dlp_p at
// each level (the raw logsigmoid part); the corrected levels add the gradient of the masses,
// which lands on the boundary path's nodes and is carried by one extra "boundary path" per
// (query, b, h) with per-level coefficients and no value weight. The generic sorted-path
// backward (ta_backward.cu, coefficient mode) then forms dq, dK and dV deterministically.

#include "ta_common.cuh"
#include "ta_rng.cuh"

namespace ta {

constexpr int kCausalThreads = 256;

struct CausalParams {
  const char* q; const char* k; const char* v; const char* dout;
  int64_t qs, qb, qh, ks, kb, kh, vs, vb, vh, gs, gb, gh;
  char* out; int64_t os, ob, oh;
  int32_t* leaf; float* weights; float* sig;  // sig: [b*H+h][t*S+s][sig_stride]
  int32_t* corrected;                          // [L]
  float* masses;                               // [L][B][H][log_n + 1]
  const float* gumbels;                        // optional [L][log_n][B][H][S][2]
  uint64_t seed, offset, offset_step;
  FastDiv stride;
  int32_t B, H, S, N, D, log_n, sig_stride;
  int64_t L, query_offset;
  // backward (coefficient form)
  float* coef;      // [b*H+h][t*(S+1)+s][sig_stride]
  float* dvw;       // [b*H+h][t*(S+1)+s]
  uint32_t* keys;   // [b*H+h][t*(S+1)+s]
  uint32_t* vals;
};

template <typename T>
__device__ __forceinline__ float dot_row(const char* a, const char* b, int D) {
  float acc = 0.0f;
  for (int c = 0; c < D; c += Elem<T>::EPC)
    acc = Dot<T>::chunk(ldg16(a + c * sizeof(T)), ldg16(b + c * sizeof(T)), acc);
  return acc;
}

__device__ __forceinline__ float log_pow2(int m) {  // log(2^m) correctly rounded to float
  return (float)((double)m * 0.69314718055994530942);
}

template <typename T>
__global__ void __launch_bounds__(kCausalThreads) causal_fwd_kernel(const CausalParams p) {
  extern __shared__ float sm[];
  const int64_t t = blockIdx.x;
  const int ln = p.log_n, S = p.S, BH = p.B * p.H;
  const int J = BH * S;
  const uint32_t K = (uint32_t)p.N - 1u;
  const int64_t boundary = t + p.query_offset;
  uint32_t* s_node = reinterpret_cast<uint32_t*>(sm);  // [J]
  float* s_lp = sm + J;                                // [J]
  const int tid = threadIdx.x;
  // boundary nodes of every level
  auto bnode = [&](int d) -> uint32_t { return (1u << d) - 1u + (uint32_t)(boundary >> (ln - d)); };
  auto bdir = [&](int d) -> int { return (int)((boundary >> (ln - 1 - d)) & 1); };
  float* M = p.masses + t * (int64_t)BH * (ln + 1);
  // pass 1: boundary masses per (b, h)
  for (int bh = tid; bh < BH; bh += blockDim.x) {
    const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
    const char* qrow = p.q + (t * p.qs + (int64_t)b * p.qb + (int64_t)h * p.qh) * sizeof(T);
    const char* kbase = p.k + ((int64_t)b * p.kb + (int64_t)h * p.kh) * sizeof(T);
    float* Mb = M + (int64_t)bh * (ln + 1);
    float m = 0.0f;
    Mb[ln] = 0.0f;
    for (int d = ln - 1; d >= 0; --d) {
      const float s = dot_row<T>(qrow, kbase + (int64_t)bnode(d) * p.ks * sizeof(T), p.D);
      float lpl, lpr;
      log_sigmoid_pair(s, lpl, lpr);
      float on, off, offm;
      if (bdir(d) == 0) { on = lpl; off = lpr; offm = -INFINITY; }
      else { on = lpr; off = lpl; offm = log_pow2(ln - 1 - d); }
      const float a = m + on, c = offm + off;
      const float mx = fmaxf(a, c);
      m = mx + logf(expf(a - mx) + expf(c - mx));
      Mb[d] = m;
    }
  }
  for (int j = tid; j < J; j += blockDim.x) {
    s_node[j] = 0u;
    s_lp[j] = 0.0f;
  }
  __syncthreads();
  // pass 2: sampling
  const int M_draw = J * 2;
  int on_path = 1;
  int corrected = 0;
  for (int d = 0; d < ln; ++d) {
    if (on_path) corrected = d + 1;
    const uint64_t off = p.offset + ((uint64_t)t * ln + d) * p.offset_step;
    int mine_on = 1;
    for (int j = tid; j < J; j += blockDim.x) {
      const int bh = j / S, s = j - bh * S;
      const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
      const uint32_t node = s_node[j];
      const char* qrow = p.q + (t * p.qs + (int64_t)b * p.qb + (int64_t)h * p.qh) * sizeof(T);
      const char* krow = p.k + ((int64_t)b * p.kb + (int64_t)h * p.kh + (int64_t)node * p.ks) * sizeof(T);
      const float x = dot_row<T>(qrow, krow, p.D);
      float lpl, lpr;
      log_sigmoid_pair(x, lpl, lpr);
      const float raw_l = lpl, raw_r = lpr;
      if (on_path) {
        const float* Mb = M + (int64_t)bh * (ln + 1);
        const float parent = Mb[d], child = Mb[d + 1];
        float ml, mr;
        if (bdir(d) == 0) { ml = child; mr = -INFINITY; }
        else { ml = log_pow2(ln - 1 - d); mr = child; }
        lpl = ml + lpl - parent;
        lpr = mr + lpr - parent;
      }
      float gl, gr;
      if (p.gumbels != nullptr) {
        const float* gp = p.gumbels + ((t * ln + d) * (int64_t)J + j) * 2;
        gl = gp[0];
        gr = gp[1];
      } else {
        gl = torch_gumbel(p.seed, off, 2u * (uint32_t)j, p.stride);
        gr = torch_gumbel(p.seed, off, 2u * (uint32_t)j + 1u, p.stride);
      }
      (void)M_draw;
      const int dir = (lpr + gr > lpl + gl) ? 1 : 0;
      s_lp[j] += dir ? lpr : lpl;
      const uint32_t nn = 2u * node + 1u + (uint32_t)dir;
      s_node[j] = nn;
      if (p.sig != nullptr) {
        const int64_t path = (int64_t)bh * p.L * S + t * S + s;
        p.sig[path * p.sig_stride + d] = expf(dir ? raw_l : raw_r);
      }
      if (d + 1 < ln && nn != bnode(d + 1)) mine_on = 0;
    }
    on_path = __syncthreads_and(on_path && mine_on);
  }
  if (tid == 0) p.corrected[t] = corrected;
  __syncthreads();
  // softmax over the S paths of each (b, h) and the value gather
  for (int bh = tid; bh < BH; bh += blockDim.x) {
    const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
    float m = -INFINITY;
    for (int s = 0; s < S; ++s) {
      const int64_t lf = (int64_t)s_node[bh * S + s] - K;
      if (lf >= 0 && lf < p.N) m = fmaxf(m, s_lp[bh * S + s]);
    }
    float sum = 0.0f;
    for (int s = 0; s < S; ++s) {
      const int64_t lf = (int64_t)s_node[bh * S + s] - K;
      if (lf >= 0 && lf < p.N) sum += expf(s_lp[bh * S + s] - m);
    }
    const float lse = m + logf(sum);
    for (int s = 0; s < S; ++s) {
      const int j = bh * S + s;
      const int64_t lf = (int64_t)s_node[j] - K;
      const float w = (lf >= 0 && lf < p.N) ? expf(s_lp[j] - lse) : 0.0f;
      const int64_t o = ((t * p.B + b) * p.H + h) * (int64_t)S + s;
      p.weights[o] = w;
      p.leaf[o] = (int32_t)lf;
      s_lp[j] = w;
    }
  }
  __syncthreads();
  const int Dc = p.D;
  for (int idx = tid; idx < BH * Dc; idx += blockDim.x) {
    const int bh = idx / Dc, c = idx - bh * Dc;
    const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
    float acc = 0.0f;
    for (int s = 0; s < S; ++s) {
      int64_t lf = (int64_t)s_node[bh * S + s] - K;
      lf = lf < 0 ? 0 : (lf >= p.N ? p.N - 1 : lf);
      const T* vrow = reinterpret_cast<const T*>(p.v + ((int64_t)b * p.vb + (int64_t)h * p.vh + lf * p.vs) * sizeof(T));
      acc = fmaf(s_lp[bh * S + s], static_cast<float>(vrow[c]), acc);
    }
    reinterpret_cast<T*>(p.out + (t * p.os + (int64_t)b * p.ob + (int64_t)h * p.oh) * sizeof(T))[c] = static_cast<T>(acc);
  }
}

// Backward coefficients of query t: real paths (gl = sgn sigmoid(-sgn s) dlp) and the boundary
// path (gradient of the corrected levels' masses), plus sort records.
template <typename T>
__global__ void __launch_bounds__(kCausalThreads) causal_coef_kernel(const CausalParams p) {
  const int64_t t = blockIdx.x;
  const int ln = p.log_n, S = p.S, BH = p.B * p.H, SP = S + 1;
  const uint32_t K = (uint32_t)p.N - 1u;
  const uint32_t base_node = (1u << ln) - 1u;
  const int64_t boundary = t + p.query_offset;
  const int corrected = p.corrected[t];
  auto bnode = [&](int d) -> uint32_t { return (1u << d) - 1u + (uint32_t)(boundary >> (ln - d)); };
  auto bdir = [&](int d) -> int { return (int)((boundary >> (ln - 1 - d)) & 1); };
  for (int bh = threadIdx.x; bh < BH; bh += blockDim.x) {
    const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
    const int64_t o0 = ((t * p.B + b) * p.H + h) * (int64_t)S;
    const char* grow = p.dout + (t * p.gs + (int64_t)b * p.gb + (int64_t)h * p.gh) * sizeof(T);
    const char* vbase = p.v + ((int64_t)b * p.vb + (int64_t)h * p.vh) * sizeof(T);
    // g_s, dlp_s
    float wg = 0.0f;
    float dsum = 0.0f;
    for (int s = 0; s < S; ++s) {
      int64_t lf = p.leaf[o0 + s];
      lf = lf < 0 ? 0 : (lf >= p.N ? p.N - 1 : lf);
      wg = fmaf(p.weights[o0 + s], dot_row<T>(grow, vbase + lf * p.vs * sizeof(T), p.D), wg);
    }
    const int64_t pbase = (int64_t)bh * p.L * SP + t * SP;
    float A[32];
    for (int d = 0; d < 32; ++d) A[d] = 0.0f;
    for (int s = 0; s < S; ++s) {
      int64_t lf = p.leaf[o0 + s];
      const int64_t lfc = lf < 0 ? 0 : (lf >= p.N ? p.N - 1 : lf);
      const float g = dot_row<T>(grow, vbase + lfc * p.vs * sizeof(T), p.D);
      const float w = p.weights[o0 + s];
      const float dl = w * (g - wg);
      dsum += dl;
      const uint32_t bits = (uint32_t)lf + K - base_node;
      const float* sg = p.sig + ((int64_t)bh * p.L * S + t * S + s) * p.sig_stride;
      float* co = p.coef + (pbase + s) * p.sig_stride;
      for (int d = 0; d < ln; ++d) {
        const int dir = (int)((bits >> (ln - 1 - d)) & 1u);
        co[d] = (dir ? -sg[d] : sg[d]) * dl;
        if (d < corrected && dir == bdir(d)) A[d] += dl;
      }
      p.dvw[pbase + s] = w;
      p.keys[pbase + s] = bits;
      p.vals[pbase + s] = (uint32_t)(t * SP + s);
    }
    // boundary path: gradient of the masses M[d] of the corrected levels
    const char* qrow = p.q + (t * p.qs + (int64_t)b * p.qb + (int64_t)h * p.qh) * sizeof(T);
    const char* kbase = p.k + ((int64_t)b * p.kb + (int64_t)h * p.kh) * sizeof(T);
    const float* Mb = p.masses + (t * (int64_t)BH + bh) * (ln + 1);
    float* cb = p.coef + (pbase + S) * p.sig_stride;
    float dM = 0.0f;  // gradient reaching M[d]
    for (int d = 0; d < ln; ++d) {
      if (d < corrected) dM -= dsum;
      const float s = dot_row<T>(qrow, kbase + (int64_t)bnode(d) * p.ks * sizeof(T), p.D);
      const float sig_m = 1.0f / (1.0f + expf(s));   // sigmoid(-s)
      const float sig_p = 1.0f / (1.0f + expf(-s));  // sigmoid(s)
      float lpl, lpr;
      log_sigmoid_pair(s, lpl, lpr);
      float pi, don, doff;
      if (bdir(d) == 0) {  // on = logsigmoid(s), off masked
        pi = 1.0f;
        don = sig_m;
        doff = 0.0f;
      } else {             // on = logsigmoid(-s), off = logsigmoid(s) with log(#leaves)
        pi = expf(Mb[d + 1] + lpr - Mb[d]);
        don = -sig_p;
        doff = sig_m;
      }
      cb[d] = dM * (pi * don + (1.0f - pi) * doff);
      dM = pi * dM + (d < corrected ? A[d] : 0.0f);
    }
    p.dvw[pbase + S] = 0.0f;
    p.keys[pbase + S] = (uint32_t)boundary;
    p.vals[pbase + S] = (uint32_t)(t * SP + S);
  }
}

}  // namespace ta

using namespace ta;

static int causal_views(const ta_shape* shape, const void* q, ta_layout ql, const void* k,
                        ta_layout kl, const void* v, ta_layout vl, CausalParams& p) {
  int rc = check_shape(shape, true);
  if (rc) return rc;
  const int es = dtype_size(shape->dtype);
  if ((rc = check_view("q", q, ql, es, false)) || (rc = check_view("k_int", k, kl, es, false)) ||
      (rc = check_view("v", v, vl, es, false)))
    return rc;
  if (floor_log2(shape->num_leaves) > 30) return fail(TA_ERR_UNSUPPORTED, "tree too deep");
  p = CausalParams{};
  p.q = (const char*)q; p.k = (const char*)k; p.v = (const char*)v;
  p.qs = ql.seq; p.qb = ql.batch; p.qh = ql.head;
  p.ks = kl.seq; p.kb = kl.batch; p.kh = kl.head;
  p.vs = vl.seq; p.vb = vl.batch; p.vh = vl.head;
  p.B = (int32_t)shape->batch; p.H = (int32_t)shape->num_heads; p.S = (int32_t)shape->num_samples;
  p.N = (int32_t)shape->num_leaves; p.D = (int32_t)shape->head_dim;
  p.log_n = floor_log2(shape->num_leaves); p.L = shape->num_queries;
  p.sig_stride = (p.log_n + 3) & ~3;
  return TA_OK;
}

extern "C" int ta_causal_forward(const ta_shape* shape, int64_t query_offset, const void* q,
                                 ta_layout ql, const void* k, ta_layout kl, const void* v,
                                 ta_layout vl, void* out, ta_layout ol, const ta_rng* rng,
                                 const float* gumbels, int32_t* leaf, float* weights,
                                 float* branch_prob, int32_t* corrected, float* masses,
                                 ta_stream_t stream) {
  CausalParams p;
  int rc = causal_views(shape, q, ql, k, kl, v, vl, p);
  if (rc) return rc;
  if ((rc = check_view("out", out, ol, dtype_size(shape->dtype), false))) return rc;
  if (!leaf || !weights || !corrected || !masses)
    return fail(TA_ERR_INVALID, "leaf, weights, corrected and masses must not be NULL");
  if (query_offset < 0 || query_offset + shape->num_queries > shape->num_leaves)
    return fail(TA_ERR_INVALID, "causal boundaries must lie within the leaves");
  p.out = (char*)out; p.os = ol.seq; p.ob = ol.batch; p.oh = ol.head;
  p.leaf = leaf; p.weights = weights; p.sig = branch_prob; p.corrected = corrected;
  p.masses = masses; p.gumbels = gumbels; p.query_offset = query_offset;
  if (gumbels == nullptr) {
    if (!rng || rng->draw_stride <= 0 || rng->draw_stride >= (1ll << 31) || (rng->offset & 3) ||
        (rng->offset_step & 3))
      return fail(TA_ERR_INVALID, "invalid rng");
    p.seed = rng->seed; p.offset = rng->offset; p.offset_step = rng->offset_step;
    p.stride.init((uint32_t)rng->draw_stride);
  } else {
    p.stride.init(1);
  }
  const int J = p.B * p.H * p.S;
  const size_t smem = (size_t)J * 8;
  if (smem > 200 * 1024) return fail(TA_ERR_UNSUPPORTED, "batch * heads * samples too large for one CTA");
  if (p.L == 0) return TA_OK;
  cudaStream_t st = (cudaStream_t)stream;
  switch (shape->dtype) {
#define TA_LAUNCH(TY)                                                                          \
  {                                                                                            \
    if (smem > 48 * 1024)                                                                      \
      cudaFuncSetAttribute(causal_fwd_kernel<TY>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                           (int)smem);                                                         \
    TA_PROFILE("causal_fwd", st);                                                              \
    causal_fwd_kernel<TY><<<(unsigned)p.L, kCausalThreads, smem, st>>>(p);                     \
  }
    case TA_F32: TA_LAUNCH(float) break;
    case TA_F16: TA_LAUNCH(__half) break;
    default: TA_LAUNCH(__nv_bfloat16) break;
#undef TA_LAUNCH
  }
  return check_launch("causal forward");
}

// The coefficient half of the causal backward: writes, for L*(S+1) paths per head (S sampled
// paths and one boundary path per query), the per-level coefficients, value weights and sort
// records consumed by ta_backward_coef.
extern "C" int ta_causal_coefficients(const ta_shape* shape, int64_t query_offset,
                                      const void* q, ta_layout ql, const void* k, ta_layout kl,
                                      const void* v, ta_layout vl, const void* grad_out,
                                      ta_layout gl, const int32_t* leaf, const float* weights,
                                      const float* branch_prob, const int32_t* corrected,
                                      const float* masses, float* coef, float* value_weight,
                                      uint32_t* keys, uint32_t* vals, ta_stream_t stream) {
  CausalParams p;
  int rc = causal_views(shape, q, ql, k, kl, v, vl, p);
  if (rc) return rc;
  if ((rc = check_view("grad_out", grad_out, gl, dtype_size(shape->dtype), false))) return rc;
  if (!leaf || !weights || !branch_prob || !corrected || !masses || !coef || !value_weight ||
      !keys || !vals)
    return fail(TA_ERR_INVALID, "NULL argument");
  p.dout = (const char*)grad_out; p.gs = gl.seq; p.gb = gl.batch; p.gh = gl.head;
  p.leaf = const_cast<int32_t*>(leaf); p.weights = const_cast<float*>(weights);
  p.sig = const_cast<float*>(branch_prob); p.corrected = const_cast<int32_t*>(corrected);
  p.masses = const_cast<float*>(masses); p.query_offset = query_offset;
  p.coef = coef; p.dvw = value_weight; p.keys = keys; p.vals = vals;
  if (p.L == 0) return TA_OK;
  cudaStream_t st = (cudaStream_t)stream;
  switch (shape->dtype) {
    case TA_F32: { TA_PROFILE("causal_coef", st); causal_coef_kernel<float><<<(unsigned)p.L, 64, 0, st>>>(p); } break;
    case TA_F16: { TA_PROFILE("causal_coef", st); causal_coef_kernel<__half><<<(unsigned)p.L, 64, 0, st>>>(p); } break;
    default: { TA_PROFILE("causal_coef", st); causal_coef_kernel<__nv_bfloat16><<<(unsigned)p.L, 64, 0, st>>>(p); } break;
  }
  return check_launch("causal coefficients");
}
