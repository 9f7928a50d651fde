// Fused stochastic tree-attention forward for sm_100a.
//
// Work decomposition: one 4-lane group per (query, batch, head); a CTA of 256 threads owns
// 64 consecutive queries of one (batch, head), so concurrently resident CTAs walk the same
// head's tree and its rows stay hot in L2. Each lane holds a quarter of q (in 16-byte
// chunks, interleaved so the group reads 64 contiguous bytes per load), the group walks
// four sampled paths at once (four independent row gathers in flight per depth), and lane
// t draws the Gumbel pair of the t-th path of the four.
//
// Per depth (reference: _tree_mha.py:99-119, _autograd.py:187-217,
// sample_non_causal_paths.cu:54-128):
//   s = clamp(q . k[node], +-max_logit)            (float32 accumulation)
//   lp = (logsigmoid(s), logsigmoid(-s))
//   dir = 1 iff lp_R + G_R > lp_L + G_L             (argmax, ties to the left)
//   acc += lp[dir]; node = 2 node + 1 + dir
// then w = exp(lp - logsumexp(lp)) over the S paths of a query (_autograd.py:495-498) and
// out = sum_s w_s v[leaf_s] (weighted_value_sum.cu:8-47) -- all in one launch.

#include <stdio.h>

#include <atomic>
#include <type_traits>

#include "ta_common.cuh"
#include "ta_rng.cuh"

namespace ta {

constexpr int kFwdThreads = 256;
constexpr int kFwdGroups = kFwdThreads / 4;  // queries per CTA

// kCausalTail: the causal sampler's levels after its corrected prefix (ta_causal.cu), each
// path starting from the node and log-probability the prefix kernel left in leaf / weights,
// one torch draw of B*H*S*2 per (query, level), no logit clamp; outputs as kFull.
enum FwdMode { kFull = 0, kSampleOnly = 1, kReplay = 2, kReplaySoftmax = 3, kCausalTail = 4 };

struct FwdParams {
  const char* q;
  const char* k;
  const char* v;
  char* out;
  int64_t qs, qb, qh;  // element strides (seq, batch, head)
  int64_t ks, kb, kh;
  int64_t vs, vb, vh;
  int64_t os, ob, oh;
  int32_t* leaf;
  float* weights;   // kFull / kReplaySoftmax: weights; kSampleOnly / kReplay: log-probs
  uint8_t* packed;  // written (kFull, kSampleOnly) or read (kReplay*)
  float* sig;       // optional per (path, depth) σ(-sgn s) for the backward
  int64_t P;        // paths per head (L * S)
  int32_t sig_stride;
  const float* gumbels;
  uint64_t seed, offset, offset_step;
  FastDiv stride;
  int32_t B, L, H, S, N, log_n, nchunks, pbytes;
  float max_logit;
  int32_t mode;
  int32_t top_levels;  // tree levels staged in shared memory
  const int32_t* corrected;  // kCausalTail: levels the prefix kernel already sampled, per query
};

// After the walk: the paths' log-probabilities and leaves of this group's query sit in
// s_lp / s_leaf. Writes weights (softmax over the paths, or the raw log-probabilities in the
// sample-only modes), leaves, packed direction bits and out = sum_s w_s v[leaf_s].
template <typename T, int CPL>
__device__ __forceinline__ void fwd_finish(const FwdParams& p, bool active, int l, int b, int h,
                                           int t4, unsigned gmask, float* s_lp,
                                           const int32_t* s_leaf, uint32_t j0, bool replay,
                                           bool value_sum = true) {
  using E = Elem<T>;
  constexpr int EPC = E::EPC;
  constexpr int NE = CPL * EPC;
  const uint32_t K = (uint32_t)p.N - 1u;
  __syncwarp(gmask);
  if (!active) return;  // past the last tensor-core product: idle groups stop here
  if (p.mode == kSampleOnly || p.mode == kReplay) {
    for (int s = t4; s < p.S; s += 4) {
      p.weights[j0 + s] = s_lp[s];
      p.leaf[j0 + s] = s_leaf[s];
    }
  } else {
    // softmax over the S paths: lp - logsumexp(lp), exp
    float m = -INFINITY;
    for (int s = t4; s < p.S; s += 4) m = fmaxf(m, s_lp[s]);
    m = fmaxf(m, __shfl_xor_sync(gmask, m, 1, 4));
    m = fmaxf(m, __shfl_xor_sync(gmask, m, 2, 4));
    float sum = 0.0f;
    for (int s = 0; s < p.S; ++s) sum += expf(s_lp[s] - m);  // same order on every lane
    const float lse = m + logf(sum);
    __syncwarp(gmask);
    for (int s = t4; s < p.S; s += 4) {
      const float w = expf(s_lp[s] - lse);
      s_lp[s] = w;
      if (p.weights) p.weights[j0 + s] = w;
      if (p.leaf) p.leaf[j0 + s] = s_leaf[s];
    }
    __syncwarp(gmask);
  }
  if (p.packed != nullptr && !replay) {
    const int64_t base_node = ((int64_t)1 << p.log_n) - 1;
    for (int s = t4; s < p.S; s += 4) {
      const uint32_t bits = (uint32_t)((int64_t)s_leaf[s] + K - base_node);
      for (int pb = 0; pb < p.pbytes; ++pb) {
        uint32_t byte = 0;
        for (int d = pb * 8; d < min(p.log_n, pb * 8 + 8); ++d)
          byte |= ((bits >> (p.log_n - 1 - d)) & 1u) << (d & 7);
        p.packed[(int64_t)(j0 + s) * p.pbytes + pb] = (uint8_t)byte;
      }
    }
  }
  if ((p.mode != kFull && p.mode != kCausalTail) || !value_sum) return;

  // out[l,b,h] = sum_s w_s v[leaf_s]
  float acc[NE];
#pragma unroll
  for (int e = 0; e < NE; ++e) acc[e] = 0.0f;
  const char* vbase = p.v + ((int64_t)b * p.vb + (int64_t)h * p.vh) * sizeof(T);
  const uint32_t vstride = (uint32_t)(p.vs * (int64_t)sizeof(T));
  // rows are fetched four paths at a time (all loads in flight together), then summed in
  // path order
  for (int s0 = 0; s0 < p.S; s0 += 4) {
    uint4 vr[4][CPL];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int s = s0 + t < p.S ? s0 + t : p.S - 1;
      int32_t lf = s_leaf[s];
      lf = lf < 0 ? 0 : (lf >= p.N ? p.N - 1 : lf);
      const char* vrow = vbase + (uint64_t)(uint32_t)lf * vstride;
#pragma unroll
      for (int i = 0; i < CPL; ++i) {
        const int c = i * 4 + t4;
        vr[t][i] = c < p.nchunks ? ldg16(vrow + c * 16) : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      if (s0 + t >= p.S) break;
      const float w = s_lp[s0 + t];
#pragma unroll
      for (int i = 0; i < CPL; ++i) {
        float vf[EPC];
        E::unpack(vr[t][i], vf);
#pragma unroll
        for (int e = 0; e < EPC; ++e) acc[i * EPC + e] = fmaf(w, vf[e], acc[i * EPC + e]);
      }
    }
  }
  char* orow = p.out + ((int64_t)l * p.os + (int64_t)b * p.ob + (int64_t)h * p.oh) * sizeof(T);
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = i * 4 + t4;
    if (c < p.nchunks) st16(orow + c * 16, E::pack(acc + i * EPC));
  }
}

// MMA: the per-level dot products of the four paths in flight run as m16n8k16 tensor-core
// products over the warp's eight queries (mma_path_dots); 16-bit inputs with head_dim a
// multiple of 32 and non-causal modes only (every lane of a warp walks the same levels).
template <typename T, int CPL, bool MMA>
__global__ void __launch_bounds__(kFwdThreads) fwd_kernel(const FwdParams p) {
  extern __shared__ float smem[];

  const int ltiles = (p.L + kFwdGroups - 1) / kFwdGroups;
  const int bh = blockIdx.x / ltiles;
  const int lt = blockIdx.x - bh * ltiles;
  const int b = bh / p.H;
  const int h = bh - b * p.H;
  const int g = threadIdx.x >> 2;
  const int t4 = threadIdx.x & 3;
  const bool active = lt * kFwdGroups + g < p.L;
  // the tensor-core dot needs every lane of the warp: an idle group walks the last query
  // and stores nothing
  const int l = active ? lt * kFwdGroups + g : p.L - 1;
  const unsigned gmask = 0xFu << (threadIdx.x & 28);
  const int row_bytes = p.nchunks * 16;
  const int top_rows = (1 << p.top_levels) - 1;
  char* s_tree = reinterpret_cast<char*>(smem);  // top tree levels of this head
  float* s_lp = reinterpret_cast<float*>(s_tree + (size_t)top_rows * row_bytes) + g * p.S;
  int32_t* s_leaf = reinterpret_cast<int32_t*>(s_lp - g * p.S + kFwdGroups * p.S) + g * p.S;
  const char* kbase = p.k + ((int64_t)b * p.kb + (int64_t)h * p.kh) * sizeof(T);
  const uint32_t kstride = (uint32_t)(p.ks * (int64_t)sizeof(T));
  if (top_rows > 0) {
    stage_tree_rows(s_tree, kbase, kstride, top_rows, row_bytes);
    cp_async_wait_0();
    __syncthreads();
  }
  if (!MMA && !active) return;  // whole group leaves together

  const uint32_t K = (uint32_t)p.N - 1u;
  const uint32_t j0 = (uint32_t)(((int64_t)l * p.B + b) * p.H + h) * (uint32_t)p.S;
  // per-path σ(-sgn s) rows for the backward: [b*H + h][l*S + s][sig_stride]
  float* sig_row0 = p.sig ? p.sig + (((int64_t)b * p.H + h) * p.P + (int64_t)l * p.S) * p.sig_stride
                          : nullptr;

  // q slice of this lane, kept in its storage format (16-byte chunks)
  uint4 qraw[CPL];
  {
    const char* qrow = p.q + ((int64_t)l * p.qs + (int64_t)b * p.qb + (int64_t)h * p.qh) * sizeof(T);
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int c = i * 4 + t4;
      qraw[i] = c < p.nchunks ? ldg16(qrow + c * 16) : make_uint4(0, 0, 0, 0);
    }
  }
  const bool replay = p.mode == kReplay || p.mode == kReplaySoftmax;
  const bool causal = p.mode == kCausalTail;
  const uint32_t M = 2u * (uint32_t)p.L * (uint32_t)p.B * (uint32_t)p.H * (uint32_t)p.S;
  const int d0 = causal ? p.corrected[l] : 0;
  // causal draws: per (query, level), element 2 * ((b*H + h)*S + s) + side
  const uint32_t jq = (uint32_t)(b * p.H + h) * (uint32_t)p.S;
  const uint32_t Jq = (uint32_t)(p.B * p.H * p.S);

  // Gumbel pair of path s (of this query) at `depth`; its address depends on no decision, so
  // the walk fetches it one level ahead and its latency overlaps the row gather.
  auto noise = [&](int s, int depth) -> float2 {
    if (causal) {
      const uint32_t jl = jq + (uint32_t)s;
      if (p.gumbels != nullptr)
        return *reinterpret_cast<const float2*>(p.gumbels + (((uint64_t)l * p.log_n + depth) * Jq + jl) * 2u);
      const uint64_t off = p.offset + ((uint64_t)l * p.log_n + depth) * p.offset_step;
      return make_float2(torch_gumbel(p.seed, off, 2u * jl, p.stride),
                         torch_gumbel(p.seed, off, 2u * jl + 1u, p.stride));
    }
    const uint32_t jm_ = j0 + (uint32_t)s;
    if (p.gumbels != nullptr)
      return *reinterpret_cast<const float2*>(p.gumbels + (uint64_t)depth * M + 2u * jm_);
    const uint64_t off = p.offset + (uint64_t)depth * p.offset_step;
    return make_float2(torch_gumbel(p.seed, off, 2u * jm_, p.stride),
                       torch_gumbel(p.seed, off, 2u * jm_ + 1u, p.stride));
  };

  for (int s0 = 0; s0 < p.S; s0 += 4) {
    const int ns = min(4, p.S - s0);
    uint32_t node[4] = {0u, 0u, 0u, 0u};
    float lp = 0.0f;  // path s0 + t4
    const uint32_t jm = j0 + s0 + t4;
    float sig4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (causal) {
#pragma unroll
      for (int t = 0; t < 4; ++t)
        node[t] = t < ns ? (uint32_t)p.leaf[j0 + s0 + t] : 0u;
      if (t4 < ns) {
        lp = p.weights[jm];
        if (sig_row0 != nullptr && (d0 & 3)) {  // keep the prefix kernel's entries of this quad
          const float4 o = *reinterpret_cast<const float4*>(sig_row0 + (int64_t)(s0 + t4) * p.sig_stride + (d0 & ~3));
          sig4[0] = o.x; sig4[1] = o.y; sig4[2] = o.z; sig4[3] = o.w;
        }
      }
    }
    const bool draws = !replay && t4 < ns;
    float2 g_next = draws && d0 < p.log_n ? noise(s0 + t4, d0) : make_float2(0.0f, 0.0f);
    for (int depth = d0; depth < p.log_n; ++depth) {
      const float2 g_cur = g_next;
      if (draws && depth + 1 < p.log_n) g_next = noise(s0 + t4, depth + 1);
      uint4 raw[4][CPL];
      if (depth < p.top_levels) {
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const char* krow = s_tree + node[t] * (uint32_t)row_bytes;
#pragma unroll
          for (int i = 0; i < CPL; ++i) {
            const int c = i * 4 + t4;
            raw[t][i] = (t < ns && c < p.nchunks) ? lds16(krow + c * 16) : make_uint4(0, 0, 0, 0);
          }
        }
      } else {
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const char* krow = kbase + (uint64_t)node[t] * kstride;
#pragma unroll
          for (int i = 0; i < CPL; ++i) {
            const int c = i * 4 + t4;
            raw[t][i] = (t < ns && c < p.nchunks) ? ldg16(krow + c * 16) : make_uint4(0, 0, 0, 0);
          }
        }
      }
      float mine;
      if constexpr (MMA) {
        mine = mma_path_dots<T, CPL>(qraw, raw, t4, 0xffffffffu);
      } else {
        float dot[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          dot[t] = 0.0f;
#pragma unroll
          for (int i = 0; i < CPL; ++i) dot[t] = Dot<T>::chunk(qraw[i], raw[t][i], dot[t]);
        }
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          dot[t] += __shfl_xor_sync(gmask, dot[t], 1, 4);
          dot[t] += __shfl_xor_sync(gmask, dot[t], 2, 4);
        }
        mine = t4 == 0 ? dot[0] : (t4 == 1 ? dot[1] : (t4 == 2 ? dot[2] : dot[3]));
      }
      const float x = clamp_logit(mine, p.max_logit);
      int dir = 0;
      if (t4 < ns) {
        if (replay) {
          const uint8_t byte = p.packed[(int64_t)jm * p.pbytes + (depth >> 3)];
          dir = (byte >> (depth & 7)) & 1;
        } else {
          // The reference's decision lpr + gr > lpl + gl (ties left). Since lpl - lpr = x
          // exactly in real arithmetic, it is gr - gl > x unless the two sides are within
          // float32 rounding of each other; only then are the log-sigmoids evaluated here,
          // so the next level's row address does not wait for them.
          const float gl = g_cur.x, gr = g_cur.y;
          const float diff = gr - gl;
          const float guard = 1e-5f * (fabsf(x) + fabsf(gl) + fabsf(gr) + 2.0f);
          if (fabsf(diff - x) > guard) {
            dir = diff > x ? 1 : 0;
          } else {
            float a, b;
            log_sigmoid_pair(x, a, b);
            dir = (b + gr > a + gl) ? 1 : 0;
          }
        }
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int d = __shfl_sync(gmask, dir, t, 4);
        node[t] = 2u * node[t] + 1u + (uint32_t)d;
      }
      // log-probability bookkeeping, off the walk's dependency chain
      float lpl, lpr, e;
      log_sigmoid_pair_e(x, lpl, lpr, e);
      if (t4 < ns) {
        lp += dir ? lpr : lpl;
        if (sig_row0 != nullptr && active) {
          const float sv = branch_not_taken_prob(x, dir, e);
          const int slot = depth & 3;
          sig4[0] = slot == 0 ? sv : sig4[0];
          sig4[1] = slot == 1 ? sv : sig4[1];
          sig4[2] = slot == 2 ? sv : sig4[2];
          sig4[3] = slot == 3 ? sv : sig4[3];
          if (slot == 3 || depth == p.log_n - 1) {
            float* dst = sig_row0 + (int64_t)(s0 + t4) * p.sig_stride + (depth & ~3);
            *reinterpret_cast<float4*>(dst) = make_float4(sig4[0], sig4[1], sig4[2], sig4[3]);
          }
        }
      }
    }
    if (t4 < ns) {
      const uint32_t nm = t4 == 0 ? node[0] : (t4 == 1 ? node[1] : (t4 == 2 ? node[2] : node[3]));
      s_lp[s0 + t4] = lp;
      s_leaf[s0 + t4] = (int32_t)(nm - K);
    }
  }
  fwd_finish<T, CPL>(p, active, l, b, h, t4, gmask, s_lp, s_leaf, j0, replay);
}

// Streamlined non-causal sampler (kFull / kSampleOnly) for the common case: 16-bit inputs,
// head_dim a multiple of 32 (every lane holds CPL whole 16-byte chunks), a multiple of 4
// paths, noise prefilled by ta_gumbel_fill. Same decomposition and results as fwd_kernel,
// with the per-level work cut to what the walk needs: unconditional row loads, the four
// paths' logits as tensor-core products (mma_path_dots), the decision from the sign of
// (g_R - g_L) - s with an exact fallback near ties, one ballot for the group's four
// directions, and the log-probability bookkeeping off the dependency chain.
template <typename T, int CPL>
__global__ void __launch_bounds__(kFwdThreads, 2) fwd_fast_kernel(const FwdParams p) {
  constexpr int RB = CPL * 64;  // row bytes
  extern __shared__ float smem[];
  const int ltiles = (p.L + kFwdGroups - 1) / kFwdGroups;
  const int bh = blockIdx.x / ltiles;
  const int lt = blockIdx.x - bh * ltiles;
  const int b = bh / p.H;
  const int h = bh - b * p.H;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int g = threadIdx.x >> 2;
  const int t4 = threadIdx.x & 3;
  const bool active = lt * kFwdGroups + g < p.L;
  const int l = active ? lt * kFwdGroups + g : p.L - 1;
  const unsigned gmask = 0xFu << (threadIdx.x & 28);
  const int top_rows = (1 << p.top_levels) - 1;
  char* s_tree = reinterpret_cast<char*>(smem);
  float* s_lp = reinterpret_cast<float*>(s_tree + (size_t)top_rows * RB) + g * p.S;
  int32_t* s_leaf = reinterpret_cast<int32_t*>(s_lp - g * p.S + kFwdGroups * p.S) + g * p.S;
  const char* kbase = p.k + ((int64_t)b * p.kb + (int64_t)h * p.kh) * sizeof(T);
  const uint32_t kstride = (uint32_t)(p.ks * (int64_t)sizeof(T));
  {
    constexpr int PPR = RB / 16;
    const int total = top_rows * PPR;
    for (int i = threadIdx.x; i < total; i += kFwdThreads) {
      const int r = i / PPR, c = i - r * PPR;
      cp_async16(s_tree + r * RB + c * 16, kbase + (uint64_t)r * kstride + c * 16);
    }
    cp_async_commit();
    cp_async_wait_0();
    __syncthreads();
  }
  const uint32_t K = (uint32_t)p.N - 1u;
  const uint32_t j0 = (uint32_t)(((int64_t)l * p.B + b) * p.H + h) * (uint32_t)p.S;
  float* sig_row0 = p.sig ? p.sig + (((int64_t)b * p.H + h) * p.P + (int64_t)l * p.S) * p.sig_stride
                          : nullptr;
  uint4 qraw[CPL];
  {
    const char* qrow = p.q + ((int64_t)l * p.qs + (int64_t)b * p.qb + (int64_t)h * p.qh) * sizeof(T) + t4 * 16;
#pragma unroll
    for (int i = 0; i < CPL; ++i) qraw[i] = ldg16(qrow + i * 64);
  }
  const uint64_t M = 2ull * (uint64_t)p.L * p.B * p.H * p.S;  // one depth of noise
  const uint32_t s_row0 = (uint32_t)__cvta_generic_to_shared(s_tree) + t4 * 16;
  const char* k_row0 = kbase + t4 * 16;
  for (int s0 = 0; s0 < p.S; s0 += 4) {
    uint32_t node[4] = {0u, 0u, 0u, 0u};
    float lp = 0.0f;
    float sig4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const float* gp = p.gumbels + 2ull * (j0 + s0 + t4);
    // the noise addresses depend on no decision: each level's pair is requested two levels
    // before the walk reaches it
    float2 g_next = __ldg(reinterpret_cast<const float2*>(gp));
    float2 g_next2 = p.log_n > 1 ? __ldg(reinterpret_cast<const float2*>(gp + M)) : make_float2(0.0f, 0.0f);
    uint4 raw[4][CPL];
    // the rows of level `depth` (all four paths' nodes are known to every lane of the group)
    auto load_rows = [&](int depth) {
      if (depth < p.top_levels) {
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const uint32_t row = s_row0 + node[t] * (uint32_t)RB;
#pragma unroll
          for (int i = 0; i < CPL; ++i) raw[t][i] = lds16_sa(row + i * 64);
        }
      } else {
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const char* row = k_row0 + (uint64_t)node[t] * kstride;
#pragma unroll
          for (int i = 0; i < CPL; ++i) raw[t][i] = ldg16(row + i * 64);
        }
      }
    };
    load_rows(0);
    for (int depth = 0; depth < p.log_n; ++depth) {
      const float2 g_cur = g_next;
      g_next = g_next2;
      if (depth + 2 < p.log_n) g_next2 = __ldg(reinterpret_cast<const float2*>(gp + (uint64_t)(depth + 2) * M));
      const float x = clamp_logit(mma_path_dots<T, CPL>(qraw, raw, t4, 0xffffffffu), p.max_logit);
      // the reference's lpr + gr > lpl + gl (ties left) is gr - gl > x (lpl - lpr = x) unless
      // the two sides are within float32 rounding of each other; only then evaluate it as is
      const float gl = g_cur.x, gr = g_cur.y;
      const float diff = gr - gl;
      const float guard = 1e-5f * (fabsf(x) + fabsf(gl) + fabsf(gr) + 2.0f);
      int dir;
      if (fabsf(diff - x) > guard) {
        dir = diff > x ? 1 : 0;
      } else {
        float a, c;
        log_sigmoid_pair(x, a, c);
        dir = (c + gr > a + gl) ? 1 : 0;
      }
      const uint32_t bits = __ballot_sync(0xffffffffu, dir) >> (lane & 28);
#pragma unroll
      for (int t = 0; t < 4; ++t) node[t] = 2u * node[t] + 1u + ((bits >> t) & 1u);
      // the next level's rows are requested before this level's bookkeeping runs
      if (depth + 1 < p.log_n) load_rows(depth + 1);
      float lpl, lpr, e;
      log_sigmoid_pair_e(x, lpl, lpr, e);
      lp += dir ? lpr : lpl;
      if (sig_row0 != nullptr) {
        const float sv = branch_not_taken_prob(x, dir, e);
        const int slot = depth & 3;
        sig4[0] = slot == 0 ? sv : sig4[0];
        sig4[1] = slot == 1 ? sv : sig4[1];
        sig4[2] = slot == 2 ? sv : sig4[2];
        sig4[3] = slot == 3 ? sv : sig4[3];
        if ((slot == 3 || depth == p.log_n - 1) && active) {
          float* dst = sig_row0 + (int64_t)(s0 + t4) * p.sig_stride + (depth & ~3);
          *reinterpret_cast<float4*>(dst) = make_float4(sig4[0], sig4[1], sig4[2], sig4[3]);
        }
      }
    }
    const uint32_t nm = t4 == 0 ? node[0] : (t4 == 1 ? node[1] : (t4 == 2 ? node[2] : node[3]));
    s_lp[s0 + t4] = lp;
    s_leaf[s0 + t4] = (int32_t)(nm - K);
    if (p.mode == kFull) {
      // the value rows the final sum gathers: start pulling them into L2 now
      const char* vrow = p.v + ((int64_t)(nm - K) * p.vs + (int64_t)b * p.vb + (int64_t)h * p.vh) * sizeof(T);
      prefetch_l2(vrow);
      if (RB > 128) prefetch_l2(vrow + 128);
    }
  }
  // out is summed by value_gather_kernel, launched next at a higher occupancy than this walk
  fwd_finish<T, CPL>(p, active, l, b, h, t4, gmask, s_lp, s_leaf, j0, false, false);
}

// out = sum_s w_s v[clamp(leaf_s)] from leaves / weights in HBM (after the sampler, or supplied
// by the caller). Eight lanes per query, each holding C8 16-byte chunks of the row, four paths'
// rows in flight at a time; the sum runs in path order, as in the fused finish, so both give
// the same bits. Few registers: many warps per SM hide the gathers' latency.
constexpr int kGatherThreads = 256;
constexpr int kGatherQueries = kGatherThreads / 8;

template <typename T, int C8>
__global__ void __launch_bounds__(kGatherThreads, 4) value_gather_kernel(const FwdParams p) {
  using E = Elem<T>;
  constexpr int EPC = E::EPC;
  const int ltiles = (p.L + kGatherQueries - 1) / kGatherQueries;
  const int bh = blockIdx.x / ltiles;
  const int lt = blockIdx.x - bh * ltiles;
  const int b = bh / p.H;
  const int h = bh - b * p.H;
  const int g = threadIdx.x >> 3;
  const int t8 = threadIdx.x & 7;
  const int l = lt * kGatherQueries + g;
  if (l >= p.L) return;
  const uint32_t j0 = (uint32_t)(((int64_t)l * p.B + b) * p.H + h) * (uint32_t)p.S;
  float acc[C8 * EPC];
#pragma unroll
  for (int e = 0; e < C8 * EPC; ++e) acc[e] = 0.0f;
  const char* vbase = p.v + ((int64_t)b * p.vb + (int64_t)h * p.vh) * sizeof(T);
  const uint32_t vstride = (uint32_t)(p.vs * (int64_t)sizeof(T));
  for (int s0 = 0; s0 < p.S; s0 += 4) {
    uint4 vr[4][C8];
    float w[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int s = s0 + t < p.S ? s0 + t : p.S - 1;
      w[t] = s0 + t < p.S ? p.weights[j0 + s] : 0.0f;
      int32_t lf = p.leaf[j0 + s];
      lf = lf < 0 ? 0 : (lf >= p.N ? p.N - 1 : lf);
      const char* vrow = vbase + (uint64_t)(uint32_t)lf * vstride;
#pragma unroll
      for (int i = 0; i < C8; ++i) {
        const int c = i * 8 + t8;
        vr[t][i] = c < p.nchunks ? ldg16(vrow + c * 16) : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      if (s0 + t >= p.S) break;
#pragma unroll
      for (int i = 0; i < C8; ++i) {
        float vf[EPC];
        E::unpack(vr[t][i], vf);
#pragma unroll
        for (int e = 0; e < EPC; ++e) acc[i * EPC + e] = fmaf(w[t], vf[e], acc[i * EPC + e]);
      }
    }
  }
  char* orow = p.out + ((int64_t)l * p.os + (int64_t)b * p.ob + (int64_t)h * p.oh) * sizeof(T);
#pragma unroll
  for (int i = 0; i < C8; ++i) {
    const int c = i * 8 + t8;
    if (c < p.nchunks) st16(orow + c * 16, E::pack(acc + i * EPC));
  }
}

template <typename T>
static void launch_value_gather(const FwdParams& p, cudaStream_t st) {
  const int ltiles = (p.L + kGatherQueries - 1) / kGatherQueries;
  const dim3 grid((unsigned)(ltiles * p.B * p.H));
  TA_PROFILE("value_sum", st);
  switch ((p.nchunks + 7) / 8) {
    case 1: value_gather_kernel<T, 1><<<grid, kGatherThreads, 0, st>>>(p); break;
    case 2: value_gather_kernel<T, 2><<<grid, kGatherThreads, 0, st>>>(p); break;
    case 3: value_gather_kernel<T, 3><<<grid, kGatherThreads, 0, st>>>(p); break;
    default: value_gather_kernel<T, 4><<<grid, kGatherThreads, 0, st>>>(p); break;
  }
}

// Gumbel noise of `depths` draws of `numel` elements: one thread per (depth, call, subsequence)
// computes one philox 4-vector and writes the (up to) four elements torch's grid-stride
// loop would fill from it: e = tid + stride * (4 * call + c), c = 0..3.
__global__ void __launch_bounds__(256) gumbel_fill_kernel(float* out, uint32_t numel,
                                                          uint32_t stride, uint32_t calls,
                                                          uint64_t seed, uint64_t offset,
                                                          uint64_t offset_step, int depths) {
  const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const uint64_t per_depth = (uint64_t)stride * calls;
  if (t >= per_depth * depths) return;
  const int depth = (int)(t / per_depth);
  const uint32_t r = (uint32_t)(t - (uint64_t)depth * per_depth);
  const uint32_t call = r / stride;
  const uint32_t tid = r - call * stride;
  const uint32_t e0 = tid + stride * 4u * call;
  if (e0 >= numel) return;
  curandStatePhilox4_32_10_t st;
  curand_init(seed, tid, offset + (uint64_t)depth * offset_step + 4ull * call, &st);
  const float4 u4 = _curand_uniform4(st.output);
  float* o = out + (uint64_t)depth * numel;
  o[e0] = gumbel_from_uniform(u4.x);
  if (e0 + stride < numel) o[e0 + stride] = gumbel_from_uniform(u4.y);
  if (e0 + 2u * stride < numel) o[e0 + 2u * stride] = gumbel_from_uniform(u4.z);
  if (e0 + 3u * stride < numel) o[e0 + 3u * stride] = gumbel_from_uniform(u4.w);
}

// Gumbel noise of one shard of a larger (rows, batch, heads, row_elems) draw: local element
// (r, b, h, i) of the (row_count, batch_count, head_count, row_elems) output takes the value
// torch's draw puts at global element
// (((row0 + r) * batch_total + batch0 + b) * head_total + head0 + h) * row_elems + i.
struct ShardDivs {
  FastDiv row_elems, head_count, batch_count, stride;
  uint32_t row0, row_count, batch_total, batch0, head_total, head0, numel;
};

// General case: one philox 4-vector per element (a shard's elements may be spread over the
// subsequences so that no two share a vector).
__global__ void __launch_bounds__(256) gumbel_fill_shard_kernel(
    float* out, uint32_t local_numel, ShardDivs sd, uint64_t seed, uint64_t offset,
    uint64_t offset_step) {
  const uint32_t e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= local_numel) return;
  const int depth = blockIdx.y;
  // 32-bit index math throughout: the full draw is below 2^31 elements
  const uint32_t row = sd.row_elems.div(e);
  const uint32_t inner = e - row * sd.row_elems.d;
  const uint32_t t = sd.head_count.div(row);
  const uint32_t h = row - t * sd.head_count.d;
  const uint32_t r = sd.batch_count.div(t);
  const uint32_t b = t - r * sd.batch_count.d;
  const uint32_t g =
      (((sd.row0 + r) * sd.batch_total + sd.batch0 + b) * sd.head_total + sd.head0 + h) *
          sd.row_elems.d + inner;
  const float u = torch_uniform(seed, offset + (uint64_t)depth * offset_step, g, sd.stride);
  out[(uint64_t)depth * local_numel + e] = gumbel_from_uniform(u);
}

// Common case: the grid stride is a multiple of a global row (batch_total * head_total *
// row_elems elements), as for the benchmark shapes. A philox 4-vector then serves elements
// tid + stride (4 call + c) of the same column of rows (4 call + c) stride / row apart, so
// the vector belongs to the shard for all four or none: one thread per (call, shard column,
// row within a stride) computes it once and writes the components in the shard's rows.
struct ShardRowDivs {
  FastDiv per_call, cols, row_elems, head_count, row;
  uint32_t row_block, row0, row_count, batch0, head_total, head0, numel, stride, calls;
};

__global__ void __launch_bounds__(256) gumbel_fill_shard_rows_kernel(
    float* out, uint32_t local_numel, ShardRowDivs sd, uint64_t seed, uint64_t offset,
    uint64_t offset_step) {
  const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= sd.per_call.d * sd.calls) return;
  const int depth = blockIdx.y;
  const uint32_t call = sd.per_call.div(t);
  const uint32_t rem = t - call * sd.per_call.d;
  const uint32_t rr = sd.cols.div(rem);            // row within one stride
  const uint32_t lc = rem - rr * sd.cols.d;          // shard column (b, h, i)
  const uint32_t t2 = sd.row_elems.div(lc);
  const uint32_t i = lc - t2 * sd.row_elems.d;
  const uint32_t bl = sd.head_count.div(t2);
  const uint32_t hl = t2 - bl * sd.head_count.d;
  const uint32_t col = ((sd.batch0 + bl) * sd.head_total + sd.head0 + hl) * sd.row_elems.d + i;
  const uint32_t tid = rr * sd.row_block + col;
  curandStatePhilox4_32_10_t st;
  curand_init(seed, tid, offset + (uint64_t)depth * offset_step + 4ull * call, &st);
  const float4 u4 = _curand_uniform4(st.output);
  float* o = out + (uint64_t)depth * local_numel;
#pragma unroll
  for (uint32_t c = 0; c < 4; ++c) {
    const uint32_t g = tid + sd.stride * (4u * call + c);
    if (g >= sd.numel) break;
    const uint32_t row = sd.row.div(g);
    if (row < sd.row0 || row >= sd.row0 + sd.row_count) continue;
    o[(row - sd.row0) * sd.cols.d + lc] =
        gumbel_from_uniform(c == 0 ? u4.x : (c == 1 ? u4.y : (c == 2 ? u4.z : u4.w)));
  }
}

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------

int pick_cpl(int nchunks) {
  const int need = (nchunks + 3) / 4;
  const int opts[] = {1, 2, 3, 4, 6, 8};
  for (int c : opts)
    if (c >= need) return c;
  return -1;
}

static bool aligned16(const void* ptr) { return ((uintptr_t)ptr & 15u) == 0; }

int check_view(const char* name, const void* ptr, ta_layout lay, int esize, bool allow_null) {
  if (ptr == nullptr) {
    if (allow_null) return TA_OK;
    return fail(TA_ERR_INVALID, "%s is NULL", name);
  }
  if (!aligned16(ptr)) return fail(TA_ERR_INVALID, "%s is not 16-byte aligned", name);
  if ((lay.seq * esize) % 16 || (lay.batch * esize) % 16 || (lay.head * esize) % 16)
    return fail(TA_ERR_INVALID, "%s strides (%lld,%lld,%lld) are not 16-byte multiples", name,
                (long long)lay.seq, (long long)lay.batch, (long long)lay.head);
  return TA_OK;
}

int check_shape(const ta_shape* s, bool need_pow2) {
  if (s == nullptr) return fail(TA_ERR_INVALID, "shape is NULL");
  if (s->dtype != TA_F32 && s->dtype != TA_F16 && s->dtype != TA_BF16)
    return fail(TA_ERR_INVALID, "unknown dtype %d", s->dtype);
  if (s->batch <= 0 || s->num_queries <= 0 || s->num_heads <= 0 || s->head_dim <= 0 ||
      s->num_samples <= 0)
    return fail(TA_ERR_INVALID, "batch, num_queries, num_heads, head_dim and num_samples must be > 0");
  if (s->num_leaves < 2) return fail(TA_ERR_INVALID, "num_leaves must be >= 2 (got %lld)",
                                     (long long)s->num_leaves);
  if (need_pow2 && (s->num_leaves & (s->num_leaves - 1)))
    return fail(TA_ERR_UNSUPPORTED, "num_leaves must be a power of two (got %lld)",
                (long long)s->num_leaves);
  if (s->num_leaves > (1ll << 30)) return fail(TA_ERR_UNSUPPORTED, "num_leaves > 2^30");
  const int es = dtype_size(s->dtype);
  if ((s->head_dim * es) % 16) return fail(TA_ERR_UNSUPPORTED,
      "head_dim * element size must be a multiple of 16 bytes (head_dim=%lld)", (long long)s->head_dim);
  if (pick_cpl((int)(s->head_dim * es / 16)) < 0)
    return fail(TA_ERR_UNSUPPORTED, "head_dim %lld too large", (long long)s->head_dim);
  if (s->num_samples > 256) return fail(TA_ERR_UNSUPPORTED, "num_samples > 256");
  const int64_t draws = s->num_queries * s->batch * s->num_heads * s->num_samples * 2;
  if (draws >= (1ll << 31)) return fail(TA_ERR_UNSUPPORTED, "L*B*H*S*2 must be < 2^31");
  if (!(s->max_logit > 0.0f)) return fail(TA_ERR_INVALID, "max_logit must be > 0");
  return TA_OK;
}

namespace {
int g_tensor_dots = 1;  // forward dot products on mma.sync where the shape allows
}

template <typename T, int CPL, bool MMA>
static void launch_fwd_kernel(const FwdParams& p, dim3 grid, size_t smem, cudaStream_t st) {
  static std::atomic<uint64_t> attr_set{0};  // per device: the attribute is set once
  if (smem > 48 * 1024) {
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
      cudaFuncSetAttribute(fwd_kernel<T, CPL, MMA>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kTreeSmemBudget + kFwdGroups * 256 * 8);
      attr_set.fetch_or(bit);
    }
  }
  fwd_kernel<T, CPL, MMA><<<grid, kFwdThreads, smem, st>>>(p);
}

template <typename T, int CPL>
static void launch_fast_kernel(const FwdParams& p, dim3 grid, size_t smem, cudaStream_t st) {
  static std::atomic<uint64_t> attr_set{0};  // per device: the attribute is set once
  if (smem > 48 * 1024) {
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
      cudaFuncSetAttribute(fwd_fast_kernel<T, CPL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kTreeSmemBudget + kFwdGroups * 256 * 8);
      attr_set.fetch_or(bit);
    }
  }
  fwd_fast_kernel<T, CPL><<<grid, kFwdThreads, smem, st>>>(p);
}

template <typename T, int CPL>
static void launch_fwd(const FwdParams& p, cudaStream_t st, bool value_only) {
  const int ltiles = (p.L + kFwdGroups - 1) / kFwdGroups;
  const dim3 grid((unsigned)(ltiles * p.B * p.H));
  if (value_only) {
    launch_value_gather<T>(p, st);
    return;
  }
  const size_t smem = (size_t)kFwdGroups * p.S * 8 +
                      (size_t)((1 << p.top_levels) - 1) * p.nchunks * 16;
  if constexpr (!std::is_same<T, float>::value) {
    if (g_tensor_dots && p.nchunks == 4 * CPL && p.mode != kCausalTail) {
      if (CPL <= 4 && (p.mode == kFull || p.mode == kSampleOnly) && p.gumbels != nullptr &&
          p.S % 4 == 0 && p.weights != nullptr && p.leaf != nullptr) {
        {
          TA_PROFILE(p.mode == kFull ? "fwd_walk" : "sample_paths", st);
          launch_fast_kernel<T, (CPL <= 4 ? CPL : 4)>(p, grid, smem, st);
        }
        if (p.mode == kFull) launch_value_gather<T>(p, st);
        return;
      }
    }
  }
  TA_PROFILE(p.mode == kFull ? "fwd_fused" : p.mode == kSampleOnly ? "sample_paths"
             : p.mode == kCausalTail ? "causal_tail" : "replay_paths", st);
  if constexpr (!std::is_same<T, float>::value) {
    if (g_tensor_dots && p.nchunks == 4 * CPL && p.mode != kCausalTail) {
      launch_fwd_kernel<T, CPL, true>(p, grid, smem, st);
      return;
    }
  }
  launch_fwd_kernel<T, CPL, false>(p, grid, smem, st);
}

template <typename T>
static int dispatch_cpl(const FwdParams& p, cudaStream_t st, bool value_only) {
  switch (pick_cpl(p.nchunks)) {
    case 1: launch_fwd<T, 1>(p, st, value_only); break;
    case 2: launch_fwd<T, 2>(p, st, value_only); break;
    case 3: launch_fwd<T, 3>(p, st, value_only); break;
    case 4: launch_fwd<T, 4>(p, st, value_only); break;
    case 6: launch_fwd<T, 6>(p, st, value_only); break;
    case 8: launch_fwd<T, 8>(p, st, value_only); break;
    default: return fail(TA_ERR_UNSUPPORTED, "head_dim too large");
  }
  return check_launch("tree-attention forward");
}

static int run_fwd(const FwdParams& p, int32_t dtype, cudaStream_t st, bool value_only) {
  if (p.L == 0) return TA_OK;
  switch (dtype) {
    case TA_F32: return dispatch_cpl<float>(p, st, value_only);
    case TA_F16: return dispatch_cpl<__half>(p, st, value_only);
    case TA_BF16: return dispatch_cpl<__nv_bfloat16>(p, st, value_only);
  }
  return fail(TA_ERR_INVALID, "unknown dtype");
}

static void fill_common(FwdParams& p, const ta_shape* s) {
  p.B = (int32_t)s->batch;
  p.L = (int32_t)s->num_queries;
  p.H = (int32_t)s->num_heads;
  p.S = (int32_t)s->num_samples;
  p.N = (int32_t)s->num_leaves;
  p.log_n = floor_log2(s->num_leaves);
  p.nchunks = (int32_t)(s->head_dim * dtype_size(s->dtype) / 16);
  p.pbytes = (p.log_n + 7) / 8;
  p.top_levels = smem_tree_levels(p.log_n, p.nchunks * 16, kTreeSmemBudget);
  p.max_logit = s->max_logit;
}

static int fill_rng(FwdParams& p, const ta_rng* rng, const float* gumbels) {
  p.gumbels = gumbels;
  if (gumbels == nullptr) {
    if (rng == nullptr) return fail(TA_ERR_INVALID, "rng is NULL and no gumbels were given");
    if (rng->draw_stride <= 0 || rng->draw_stride >= (1ll << 31) || (rng->offset & 3) ||
        (rng->offset_step & 3))
      return fail(TA_ERR_INVALID, "invalid rng (draw_stride %lld, offset %llu, step %llu)",
                  (long long)rng->draw_stride, (unsigned long long)rng->offset,
                  (unsigned long long)rng->offset_step);
    p.seed = rng->seed;
    p.offset = rng->offset;
    p.offset_step = rng->offset_step;
    p.stride.init((uint32_t)rng->draw_stride);
  } else {
    p.stride.init(1);
  }
  return TA_OK;
}

}  // namespace ta

using namespace ta;

extern "C" int ta_forward(const ta_shape* shape, const void* q, ta_layout ql, const void* k,
                          ta_layout kl, const void* v, ta_layout vl, void* out, ta_layout ol,
                          const ta_rng* rng, const float* gumbels, int32_t* leaf, float* weights,
                          uint8_t* packed, float* branch_prob, ta_stream_t stream) {
  int rc = check_shape(shape, true);
  if (rc) return rc;
  const int es = dtype_size(shape->dtype);
  if ((rc = check_view("q", q, ql, es, false)) || (rc = check_view("k_int", k, kl, es, false)) ||
      (rc = check_view("v", v, vl, es, false)) || (rc = check_view("out", out, ol, es, false)))
    return rc;
  FwdParams p{};
  fill_common(p, shape);
  if ((rc = fill_rng(p, rng, gumbels))) return rc;
  p.q = (const char*)q; p.k = (const char*)k; p.v = (const char*)v; p.out = (char*)out;
  p.qs = ql.seq; p.qb = ql.batch; p.qh = ql.head;
  p.ks = kl.seq; p.kb = kl.batch; p.kh = kl.head;
  p.vs = vl.seq; p.vb = vl.batch; p.vh = vl.head;
  p.os = ol.seq; p.ob = ol.batch; p.oh = ol.head;
  p.leaf = leaf; p.weights = weights; p.packed = packed;
  p.sig = branch_prob;
  p.P = shape->num_queries * shape->num_samples;
  p.sig_stride = (p.log_n + 3) & ~3;
  if (branch_prob && ((uintptr_t)branch_prob & 15))
    return fail(TA_ERR_INVALID, "branch_prob must be 16-byte aligned");
  p.mode = kFull;
  return run_fwd(p, shape->dtype, (cudaStream_t)stream, false);
}

namespace ta {

// Levels after the causal prefix (see kCausalTail); called by ta_causal_forward once the
// prefix kernel has left each path's node in `leaf`, its log-probability in `weights`, its
// prefix branch probabilities in branch_prob and the prefix length in `corrected`.
int causal_tail(const ta_shape* shape, const void* q, ta_layout ql, const void* k, ta_layout kl,
                const void* v, ta_layout vl, void* out, ta_layout ol, const ta_rng* rng,
                const float* gumbels, const int32_t* corrected, int32_t* leaf, float* weights,
                float* branch_prob, cudaStream_t st) {
  FwdParams p{};
  fill_common(p, shape);
  int rc = fill_rng(p, rng, gumbels);
  if (rc) return rc;
  p.q = (const char*)q; p.k = (const char*)k; p.v = (const char*)v; p.out = (char*)out;
  p.qs = ql.seq; p.qb = ql.batch; p.qh = ql.head;
  p.ks = kl.seq; p.kb = kl.batch; p.kh = kl.head;
  p.vs = vl.seq; p.vb = vl.batch; p.vh = vl.head;
  p.os = ol.seq; p.ob = ol.batch; p.oh = ol.head;
  p.leaf = leaf; p.weights = weights; p.packed = nullptr;
  p.sig = branch_prob;
  p.P = shape->num_queries * shape->num_samples;
  p.sig_stride = (p.log_n + 3) & ~3;
  p.max_logit = INFINITY;  // treeattn-torch's causal sampler does not clamp
  p.corrected = corrected;
  p.mode = kCausalTail;
  return run_fwd(p, shape->dtype, st, false);
}

}  // namespace ta

extern "C" int ta_sample_paths(const ta_shape* shape, const void* q, ta_layout ql, const void* k,
                               ta_layout kl, const ta_rng* rng, const float* gumbels,
                               int32_t* leaf, float* log_prob, uint8_t* packed,
                               ta_stream_t stream) {
  int rc = check_shape(shape, false);
  if (rc) return rc;
  const int es = dtype_size(shape->dtype);
  if ((rc = check_view("q", q, ql, es, false)) || (rc = check_view("k_int", k, kl, es, false)))
    return rc;
  if (!leaf || !log_prob) return fail(TA_ERR_INVALID, "leaf and log_prob must not be NULL");
  FwdParams p{};
  fill_common(p, shape);
  if ((rc = fill_rng(p, rng, gumbels))) return rc;
  p.q = (const char*)q; p.k = (const char*)k;
  p.qs = ql.seq; p.qb = ql.batch; p.qh = ql.head;
  p.ks = kl.seq; p.kb = kl.batch; p.kh = kl.head;
  p.leaf = leaf; p.weights = log_prob; p.packed = packed;
  p.mode = kSampleOnly;
  return run_fwd(p, shape->dtype, (cudaStream_t)stream, false);
}

extern "C" int ta_replay_paths(const ta_shape* shape, const void* q, ta_layout ql, const void* k,
                               ta_layout kl, const uint8_t* packed, int32_t softmax,
                               int32_t* leaf, float* out_f, ta_stream_t stream) {
  int rc = check_shape(shape, false);
  if (rc) return rc;
  const int es = dtype_size(shape->dtype);
  if ((rc = check_view("q", q, ql, es, false)) || (rc = check_view("k_int", k, kl, es, false)))
    return rc;
  if (!leaf || !out_f || !packed)
    return fail(TA_ERR_INVALID, "packed, leaf and output must not be NULL");
  FwdParams p{};
  fill_common(p, shape);
  p.stride.init(1);
  p.q = (const char*)q; p.k = (const char*)k;
  p.qs = ql.seq; p.qb = ql.batch; p.qh = ql.head;
  p.ks = kl.seq; p.kb = kl.batch; p.kh = kl.head;
  p.leaf = leaf; p.weights = out_f; p.packed = const_cast<uint8_t*>(packed);
  p.mode = softmax ? kReplaySoftmax : kReplay;
  return run_fwd(p, shape->dtype, (cudaStream_t)stream, false);
}

extern "C" int ta_weighted_value_sum(const ta_shape* shape, const void* v, ta_layout vl,
                                     const int32_t* leaf, const float* weights, void* out,
                                     ta_layout ol, ta_stream_t stream) {
  int rc = check_shape(shape, false);
  if (rc) return rc;
  const int es = dtype_size(shape->dtype);
  if ((rc = check_view("v", v, vl, es, false)) || (rc = check_view("out", out, ol, es, false)))
    return rc;
  if (!leaf || !weights) return fail(TA_ERR_INVALID, "leaf and weights must not be NULL");
  FwdParams p{};
  fill_common(p, shape);
  p.v = (const char*)v; p.out = (char*)out;
  p.vs = vl.seq; p.vb = vl.batch; p.vh = vl.head;
  p.os = ol.seq; p.ob = ol.batch; p.oh = ol.head;
  p.leaf = const_cast<int32_t*>(leaf); p.weights = const_cast<float*>(weights);
  return run_fwd(p, shape->dtype, (cudaStream_t)stream, true);
}

extern "C" int ta_gumbel_fill(float* out, int64_t numel, const ta_rng* rng, int32_t depth0,
                              int32_t depths, ta_stream_t stream) {
  if (!out || !rng || numel < 0 || numel >= (1ll << 31) || depth0 < 0 || depths < 0)
    return fail(TA_ERR_INVALID, "ta_gumbel_fill: invalid arguments");
  if (rng->draw_stride <= 0 || rng->draw_stride >= (1ll << 31) || (rng->offset & 3) ||
      (rng->offset_step & 3))
    return fail(TA_ERR_INVALID, "ta_gumbel_fill: invalid rng");
  if (numel == 0 || depths == 0) return TA_OK;
  const uint32_t stride = (uint32_t)rng->draw_stride;
  const uint64_t bundles = ((uint64_t)numel + stride - 1) / stride;
  const uint32_t calls = (uint32_t)((bundles + 3) / 4);
  const uint64_t threads = (uint64_t)stride * calls * depths;
  const unsigned grid = (unsigned)((threads + 255) / 256);
  TA_PROFILE("gumbel_fill", (cudaStream_t)stream);
  gumbel_fill_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
      out, (uint32_t)numel, stride, calls, rng->seed,
      rng->offset + (uint64_t)depth0 * rng->offset_step, rng->offset_step, depths);
  return check_launch("gumbel fill");
}

extern "C" int ta_gumbel_fill_shard(float* out, const ta_rng* rng, const ta_shard* shard,
                                    int64_t row_elems, int32_t depth0, int32_t depths,
                                    ta_stream_t stream) {
  if (!out || !rng || !shard || row_elems <= 0 || depth0 < 0 || depths < 0 || depths > 65535)
    return fail(TA_ERR_INVALID, "ta_gumbel_fill_shard: invalid arguments");
  const ta_shard& s = *shard;
  if (s.row_total < 0 || s.batch_total <= 0 || s.head_total <= 0 || s.row_count < 0 ||
      s.batch_count <= 0 || s.head_count <= 0 || s.row0 < 0 || s.batch0 < 0 || s.head0 < 0 ||
      s.row0 + s.row_count > s.row_total || s.batch0 + s.batch_count > s.batch_total ||
      s.head0 + s.head_count > s.head_total)
    return fail(TA_ERR_INVALID, "ta_gumbel_fill_shard: shard outside the full draw");
  const double global = (double)s.row_total * s.batch_total * s.head_total * row_elems;
  if (global >= 2147483648.0)
    return fail(TA_ERR_UNSUPPORTED, "ta_gumbel_fill_shard: the full draw exceeds 2^31 elements");
  if (rng->draw_stride <= 0 || rng->draw_stride >= (1ll << 31) || (rng->offset & 3) ||
      (rng->offset_step & 3))
    return fail(TA_ERR_INVALID, "ta_gumbel_fill_shard: invalid rng");
  const uint64_t local = (uint64_t)s.row_count * s.batch_count * s.head_count * row_elems;
  if (local == 0 || depths == 0) return TA_OK;
  const uint64_t row_block = (uint64_t)s.batch_total * s.head_total * row_elems;
  const uint64_t numel = (uint64_t)s.row_total * row_block;
  const uint32_t stride = (uint32_t)rng->draw_stride;
  TA_PROFILE("gumbel_fill", (cudaStream_t)stream);
  // the row kernel computes the vectors of every row of the shard's columns: worth it unless
  // the shard holds under a quarter of the rows (then one vector per element costs less)
  if (stride % row_block == 0 && 4 * s.row_count >= s.row_total) {
    ShardRowDivs sd;
    const uint32_t cols = (uint32_t)((uint64_t)s.batch_count * s.head_count * row_elems);
    const uint32_t rows_per_stride = (uint32_t)(stride / row_block);
    const uint64_t bundles = (numel + stride - 1) / stride;
    sd.calls = (uint32_t)((bundles + 3) / 4);
    sd.per_call.init(rows_per_stride * cols);
    sd.cols.init(cols);
    sd.row_elems.init((uint32_t)row_elems);
    sd.head_count.init((uint32_t)s.head_count);
    sd.row.init((uint32_t)row_block);
    sd.row_block = (uint32_t)row_block;
    sd.row0 = (uint32_t)s.row0;
    sd.row_count = (uint32_t)s.row_count;
    sd.batch0 = (uint32_t)s.batch0;
    sd.head_total = (uint32_t)s.head_total;
    sd.head0 = (uint32_t)s.head0;
    sd.numel = (uint32_t)numel;
    sd.stride = stride;
    const uint64_t threads = (uint64_t)rows_per_stride * cols * sd.calls;
    dim3 grid((unsigned)((threads + 255) / 256), (unsigned)depths);
    gumbel_fill_shard_rows_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
        (float*)out, (uint32_t)local, sd, rng->seed,
        rng->offset + (uint64_t)depth0 * rng->offset_step, rng->offset_step);
  } else {
    ShardDivs sd;
    sd.row_elems.init((uint32_t)row_elems);
    sd.head_count.init((uint32_t)s.head_count);
    sd.batch_count.init((uint32_t)s.batch_count);
    sd.stride.init(stride);
    sd.row0 = (uint32_t)s.row0;
    sd.row_count = (uint32_t)s.row_count;
    sd.batch_total = (uint32_t)s.batch_total; sd.batch0 = (uint32_t)s.batch0;
    sd.head_total = (uint32_t)s.head_total; sd.head0 = (uint32_t)s.head0;
    sd.numel = (uint32_t)numel;
    dim3 grid((unsigned)((local + 255) / 256), (unsigned)depths);
    gumbel_fill_shard_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
        (float*)out, (uint32_t)local, sd, rng->seed,
        rng->offset + (uint64_t)depth0 * rng->offset_step, rng->offset_step);
  }
  return check_launch("gumbel fill (shard)");
}

extern "C" int32_t ta_forward_set_tensor_dots(int32_t enable) {
  const int32_t old = g_tensor_dots;
  g_tensor_dots = enable ? 1 : 0;
  return old;
}

extern "C" int32_t ta_branch_prob_stride(int64_t num_leaves) {
  return (floor_log2(num_leaves) + 3) & ~3;
}
