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
// The "every sample" predicate couples all (b, h) of a query, so one CTA per query evaluates
// it with a block-wide AND between levels (prefix kernel). While it holds, every sample of a
// (b, h) stands on the boundary node, so those levels need only the boundary logits of pass
// 1; once it fails it stays false, and the remaining levels of every path are independent
// raw-logsigmoid steps, run by the non-causal sampler's kernel (kCausalTail in
// ta_forward.cu) with its per-head shared-memory tree and four-lane dot products.
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

// Prefix kernel, one CTA per query. Pass 1 (one thread per (b, h)): the boundary logits
// s_b[d] and masses M[d], stored in masses[t][b][h] = (M[0..ln], s_b[0..ln-1]). Pass 2: while
// EVERY sample of the query sits on the boundary node, all samples of a (b, h) stand on the
// same node, whose logit is s_b[d]; the corrected decisions need no other dot product. The
// first level after which some sample has left the boundary path ends the prefix: each path's
// node and log-probability go to leaf / weights (the tail kernel continues from there),
// `corrected` = number of prefix levels.
template <typename T>
__global__ void __launch_bounds__(kCausalThreads) causal_prefix_kernel(const CausalParams p) {
  extern __shared__ float sm[];
  const int64_t t = blockIdx.x;
  const int ln = p.log_n, S = p.S, BH = p.B * p.H;
  const int J = BH * S;
  const int MS = 2 * ln + 1;
  const int64_t boundary = t + p.query_offset;
  float* s_ms = sm;                                             // [BH][MS]
  uint32_t* s_node = reinterpret_cast<uint32_t*>(s_ms + BH * MS); // [J]
  float* s_lp = reinterpret_cast<float*>(s_node + J);           // [J]
  const int tid = threadIdx.x;
  auto bnode = [&](int d) -> uint32_t { return (1u << d) - 1u + (uint32_t)(boundary >> (ln - d)); };
  auto bdir = [&](int d) -> int { return (int)((boundary >> (ln - 1 - d)) & 1); };
  float* Mg = p.masses + t * (int64_t)BH * MS;
  // boundary logits: all (b, h, level) dots in parallel
  for (int i = tid; i < BH * ln; i += blockDim.x) {
    const int bh = i / ln, d = i - bh * ln;
    const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
    const char* qrow = p.q + (t * p.qs + (int64_t)b * p.qb + (int64_t)h * p.qh) * sizeof(T);
    const char* krow = p.k + ((int64_t)b * p.kb + (int64_t)h * p.kh + (int64_t)bnode(d) * p.ks) * sizeof(T);
    s_ms[bh * MS + ln + 1 + d] = dot_row<T>(qrow, krow, p.D);
  }
  __syncthreads();
  // masses, bottom-up per (b, h)
  for (int bh = tid; bh < BH; bh += blockDim.x) {
    float* Mb = s_ms + bh * MS;
    float m = 0.0f;
    Mb[ln] = 0.0f;
    for (int d = ln - 1; d >= 0; --d) {
      float lpl, lpr;
      log_sigmoid_pair(Mb[ln + 1 + d], lpl, lpr);
      float on, off, offm;
      if (bdir(d) == 0) { on = lpl; off = lpr; offm = -INFINITY; }
      else { on = lpr; off = lpl; offm = log_pow2(ln - 1 - d); }
      const float a = m + on, c = offm + off;
      const float mx = fmaxf(a, c);
      m = mx + logf(expf(a - mx) + expf(c - mx));
      Mb[d] = m;
    }
  }
  __syncthreads();
  for (int i = tid; i < BH * MS; i += blockDim.x) Mg[i] = s_ms[i];
  for (int j = tid; j < J; j += blockDim.x) {
    s_node[j] = 0u;
    s_lp[j] = 0.0f;
  }
  __syncthreads();
  int d = 0;
  bool on_path = true;
  while (on_path && d < ln) {
    const uint64_t off = p.offset + ((uint64_t)t * ln + d) * p.offset_step;
    int mine_on = 1;
    for (int j = tid; j < J; j += blockDim.x) {
      const int bh = j / S, s = j - bh * S;
      const float* Mb = s_ms + bh * MS;
      const float x = Mb[ln + 1 + d];
      float raw_l, raw_r;
      log_sigmoid_pair(x, raw_l, raw_r);
      const float parent = Mb[d], child = Mb[d + 1];
      float ml, mr;
      if (bdir(d) == 0) { ml = child; mr = -INFINITY; }
      else { ml = log_pow2(ln - 1 - d); mr = child; }
      const float lpl = ml + raw_l - parent, lpr = mr + raw_r - parent;
      float gl, gr;
      if (p.gumbels != nullptr) {
        const float* gp = p.gumbels + ((t * ln + d) * (int64_t)J + j) * 2;
        gl = gp[0];
        gr = gp[1];
      } else {
        gl = torch_gumbel(p.seed, off, 2u * (uint32_t)j, p.stride);
        gr = torch_gumbel(p.seed, off, 2u * (uint32_t)j + 1u, p.stride);
      }
      const int dir = (lpr + gr > lpl + gl) ? 1 : 0;
      s_lp[j] += dir ? lpr : lpl;
      const uint32_t nn = 2u * s_node[j] + 1u + (uint32_t)dir;
      s_node[j] = nn;
      if (p.sig != nullptr) {
        const int64_t path = (int64_t)bh * p.L * S + t * S + s;
        p.sig[path * p.sig_stride + d] = expf(dir ? raw_l : raw_r);
      }
      if (d + 1 < ln && nn != bnode(d + 1)) mine_on = 0;
    }
    ++d;
    on_path = __syncthreads_and(mine_on) != 0;
  }
  if (tid == 0) p.corrected[t] = d;
  for (int j = tid; j < J; j += blockDim.x) {
    const int bh = j / S, s = j - bh * S;
    const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
    const int64_t o = ((t * p.B + b) * p.H + h) * (int64_t)S + s;
    p.leaf[o] = (int32_t)s_node[j];
    p.weights[o] = s_lp[j];
  }
}

// Backward coefficients of query t, one thread per path: real paths get
// gl = sgn sigmoid(-sgn s) dlp (s from the forward's branch probabilities), and one boundary
// path per (b, h) carries the gradient of the corrected levels' masses, from the boundary
// logits the prefix kernel stored. Writes the sort records of ta_backward_coef.
template <typename T>
__global__ void __launch_bounds__(kCausalThreads) causal_coef_kernel(const CausalParams p) {
  extern __shared__ float sm[];
  const int64_t t = blockIdx.x;
  const int ln = p.log_n, S = p.S, BH = p.B * p.H, SP = S + 1;
  const int J = BH * S;
  const int MS = 2 * ln + 1;
  const uint32_t K = (uint32_t)p.N - 1u;
  const uint32_t base_node = (1u << ln) - 1u;
  const int64_t boundary = t + p.query_offset;
  const int corrected = p.corrected[t];
  float* s_wg = sm;       // [J] w g
  float* s_dl = sm + J;   // [J] dlp
  const int tid = threadIdx.x;
  auto bdir = [&](int d) -> int { return (int)((boundary >> (ln - 1 - d)) & 1); };
  for (int j = tid; j < J; j += blockDim.x) {
    const int bh = j / S;
    const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
    const int64_t o = ((t * p.B + b) * p.H + h) * (int64_t)S + (j - bh * S);
    const char* grow = p.dout + (t * p.gs + (int64_t)b * p.gb + (int64_t)h * p.gh) * sizeof(T);
    int64_t lf = p.leaf[o];
    lf = lf < 0 ? 0 : (lf >= p.N ? p.N - 1 : lf);
    const char* vrow = p.v + ((int64_t)b * p.vb + (int64_t)h * p.vh + lf * p.vs) * sizeof(T);
    const float g = dot_row<T>(grow, vrow, p.D);
    s_dl[j] = g;
    s_wg[j] = p.weights[o] * g;
  }
  __syncthreads();
  for (int j = tid; j < J; j += blockDim.x) {
    const int bh = j / S, s = j - bh * S;
    const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
    const int64_t o = ((t * p.B + b) * p.H + h) * (int64_t)S + s;
    float wg = 0.0f;
    for (int u = 0; u < S; ++u) wg += s_wg[bh * S + u];  // same order for every path of bh
    const float w = p.weights[o];
    const float dl = w * (s_dl[j] - wg);
    const int64_t lf = p.leaf[o];
    const uint32_t bits = (uint32_t)lf + K - base_node;
    const int64_t pidx = (int64_t)bh * p.L * SP + t * SP + s;
    const float* sg = p.sig + ((int64_t)bh * p.L * S + t * S + s) * p.sig_stride;
    float* co = p.coef + pidx * p.sig_stride;
    for (int d4 = 0; d4 < ln; d4 += 4) {
      const float4 g4 = *reinterpret_cast<const float4*>(sg + d4);
      const float gv[4] = {g4.x, g4.y, g4.z, g4.w};
      float cv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = d4 + e;
        const int dir = d < ln ? (int)((bits >> (ln - 1 - d)) & 1u) : 0;
        cv[e] = d < ln ? (dir ? -gv[e] : gv[e]) * dl : 0.0f;
      }
      *reinterpret_cast<float4*>(co + d4) = make_float4(cv[0], cv[1], cv[2], cv[3]);
    }
    p.dvw[pidx] = w;
    p.keys[pidx] = bits;
    p.vals[pidx] = (uint32_t)(t * SP + s);
    s_dl[j] = dl;  // only this thread reads or writes entry j in this pass
  }
  __syncthreads();
  // boundary path of each (b, h): gradient of the masses M[d] of the corrected levels
  for (int bh = tid; bh < BH; bh += blockDim.x) {
    const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
    const float* Mb = p.masses + (t * (int64_t)BH + bh) * MS;
    const int64_t o0 = ((t * p.B + b) * p.H + h) * (int64_t)S;
    const int64_t pbase = (int64_t)bh * p.L * SP + t * SP;
    float dsum = 0.0f;
    for (int u = 0; u < S; ++u) dsum += s_dl[bh * S + u];
    float* cb = p.coef + (pbase + S) * p.sig_stride;
    float dM = 0.0f;  // gradient reaching M[d]
    for (int d = 0; d < ln; ++d) {
      if (d < corrected) dM -= dsum;
      float A = 0.0f;  // dlp of the samples that took the boundary branch at level d
      if (d < corrected)
        for (int u = 0; u < S; ++u) {
          const uint32_t bits = (uint32_t)p.leaf[o0 + u] + K - base_node;
          if ((int)((bits >> (ln - 1 - d)) & 1u) == bdir(d)) A += s_dl[bh * S + u];
        }
      const float s = Mb[ln + 1 + d];
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
      dM = pi * dM + A;
    }
    for (int d = ln; d < p.sig_stride; ++d) cb[d] = 0.0f;
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
  const size_t smem = (size_t)J * 8 + (size_t)p.B * p.H * (2 * p.log_n + 1) * 4;
  if (smem > 200 * 1024) return fail(TA_ERR_UNSUPPORTED, "batch * heads * samples too large for one CTA");
  if (branch_prob && ((uintptr_t)branch_prob & 15))
    return fail(TA_ERR_INVALID, "branch_prob must be 16-byte aligned");
  if (p.L == 0) return TA_OK;
  cudaStream_t st = (cudaStream_t)stream;
  switch (shape->dtype) {
#define TA_LAUNCH(TY)                                                                             \
  {                                                                                               \
    if (smem > 48 * 1024)                                                                         \
      cudaFuncSetAttribute(causal_prefix_kernel<TY>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                           (int)smem);                                                            \
    TA_PROFILE("causal_prefix", st);                                                              \
    causal_prefix_kernel<TY><<<(unsigned)p.L, kCausalThreads, smem, st>>>(p);                     \
  }
    case TA_F32: TA_LAUNCH(float) break;
    case TA_F16: TA_LAUNCH(__half) break;
    default: TA_LAUNCH(__nv_bfloat16) break;
#undef TA_LAUNCH
  }
  if ((rc = check_launch("causal forward prefix"))) return rc;
  return causal_tail(shape, q, ql, k, kl, v, vl, out, ol, gumbels ? nullptr : rng, gumbels,
                     corrected, leaf, weights, branch_prob, st);
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
  const size_t smem = (size_t)p.B * p.H * p.S * 8;
  if (smem > 200 * 1024) return fail(TA_ERR_UNSUPPORTED, "batch * heads * samples too large for one CTA");
  if (((uintptr_t)branch_prob & 15) || ((uintptr_t)coef & 15))
    return fail(TA_ERR_INVALID, "branch_prob and coef must be 16-byte aligned");
  switch (shape->dtype) {
#define TA_LAUNCH(TY)                                                                           \
  {                                                                                             \
    if (smem > 48 * 1024)                                                                       \
      cudaFuncSetAttribute(causal_coef_kernel<TY>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                           (int)smem);                                                          \
    TA_PROFILE("causal_coef", st);                                                              \
    causal_coef_kernel<TY><<<(unsigned)p.L, kCausalThreads, smem, st>>>(p);                     \
  }
    case TA_F32: TA_LAUNCH(float) break;
    case TA_F16: TA_LAUNCH(__half) break;
    default: TA_LAUNCH(__nv_bfloat16) break;
#undef TA_LAUNCH
  }
  return check_launch("causal coefficients");
}
