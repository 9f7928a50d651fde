// Exact (deterministic) tree attention over all leaves, sm_100a.
//
// Reference: _deterministic_attention (treeattn_torch/_tree_mha.py:271-321). For a query,
// log p(leaf) = sum over the leaf's path of logsigmoid(+-q . k[node]); non-causal weights are
// exp(log p) (they sum to one over a complete tree), causal weights mask leaves n > l + offset
// and softmax over the rest; out = sum_n w_n v_n.
//
// Per block of queries: node logits S = Q K^T (GEMM), one CTA per (query, batch, head) for
// the leaf weights, out = W V (GEMM). Backward: g = dO V^T (GEMM), the same per-query CTAs
// form two coefficient rows --
//   W[l][n] = w_n                                     (dV = W^T dO)
//   C[l][node] = sigmoid(-s) DL(left) - sigmoid(s) DL(right)   (dq = C K, dK = C^T Q)
// with dlp_n = w_n (g_n - sum_m w_m g_m) (causal) or w_n g_n (non-causal), g_n = dO . v_n, and
// DL(child) the sum of dlp over the child's leaves -- then three strided GEMMs with a fixed
// summation order produce the gradients (no atomics). Queries are processed in blocks so the
// per-query rows stay within the workspace.

#include <float.h>

#include <type_traits>

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
  float* partial;          // split-K partial tiles (kSplitPartialBytes)
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

// Leaf weights of one (query, batch, head) from its node logits (already in node_buf):
// log p(leaf) walks the leaf's path (root first, as the reference accumulates); causal rows
// mask leaves beyond the boundary and softmax the rest, non-causal rows take exp(log p).
// Consecutive leaves share their upper ancestors, so a warp's walk is mostly broadcast
// reads of the same logits.
__global__ void __launch_bounds__(kExactThreads) exact_weights_kernel(const ExactParams p) {
  __shared__ float s_red[32];
  const int64_t lb = blockIdx.x / (p.B * p.H);
  const int bh = (int)(blockIdx.x - lb * p.B * p.H);
  const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const int64_t l = p.l0 + lb;
  const int K = p.N - 1, N = p.N, ln = p.log_n;
  const int tid = threadIdx.x;
  const float* sd = p.node_buf + (lb * p.B * p.H + bh) * (int64_t)K;
  float* w = p.leaf_buf + (lb * p.B * p.H + bh) * (int64_t)N;
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
    // one walk per leaf: log p kept in w between the passes
    float m = -INFINITY;
    for (int n = tid; n < N; n += blockDim.x) {
      const float lp = n <= limit ? leaf_lp(n) : -INFINITY;
      w[n] = lp;
      m = fmaxf(m, lp);
    }
    m = block_reduce_max(m, s_red);
    float sum = 0.0f;
    for (int n = tid; n < N; n += blockDim.x)
      if (n <= limit) sum += expf(w[n] - m);
    sum = block_reduce_sum(sum, s_red);
    lse = m + logf(sum);
  }
  for (int n = tid; n < N; n += blockDim.x) {
    float wn;
    if (p.causal) wn = n <= limit ? expf(w[n] - lse) : 0.0f;
    else wn = expf(leaf_lp(n));
    w[n] = wn;
    if (p.weights) p.weights[((l * p.B + b) * p.H + h) * (int64_t)N + n] = wn;
  }
}

// Backward coefficients of one (query, batch, head): dlp_buf holds g_n = dO . v_n (from a
// GEMM), leaf_buf the weights w, node_buf the node logits. Writes
// C[node] = sigmoid(-s) DL(left) - sigmoid(s) DL(right) over the logits, with
// dlp_n = w_n (g_n - sum_m w_m g_m) (causal) or w_n g_n, and DL(child) the sum of dlp over
// the child's leaves (accumulated bottom-up over the weights, which the dV product has
// already consumed).
__global__ void __launch_bounds__(kExactThreads) exact_coef_kernel(const ExactParams p) {
  __shared__ float s_red[32];
  const int64_t lb = blockIdx.x / (p.B * p.H);
  const int bh = (int)(blockIdx.x - lb * p.B * p.H);
  const int K = p.N - 1, N = p.N, ln = p.log_n;
  const int tid = threadIdx.x;
  float* w = p.leaf_buf + (lb * p.B * p.H + bh) * (int64_t)N;
  float* dl = p.dlp_buf + (lb * p.B * p.H + bh) * (int64_t)N;
  float* cb = p.node_buf + (lb * p.B * p.H + bh) * (int64_t)K;
  float wg = 0.0f;
  if (p.causal) {
    for (int n = tid; n < N; n += blockDim.x) wg += w[n] * dl[n];
    wg = block_reduce_sum(wg, s_red);
  }
  for (int n = tid; n < N; n += blockDim.x) dl[n] = p.causal ? w[n] * (dl[n] - wg) : w[n] * dl[n];
  __syncthreads();
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
      const float sl = 1.0f / (1.0f + expf(s)), sr = 1.0f / (1.0f + expf(-s));
      cb[node] = sl * lsum - sr * rsum;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------------------
// strided batched GEMM, fixed summation order: Y[m][n] (+)= sum_k A[m][k] * B[k][n]
// A and B float32 or T, Y float32 or T; one batch per (b, h). Tiles of BM x BN with a 4x4
// register block per thread (BM * BN = 4096). With `splits` > 1 the k range is cut into
// that many slices whose partial tiles go to `partial` ([split][b*H+h][M][Nn], float32) and
// a second kernel sums them in slice order -- deterministic split-K for the skinny
// products (M = a query block, k = all nodes or leaves).
// ---------------------------------------------------------------------------------------
struct GemmParams {
  const char* A; int64_t sAm, sAk, sAb, sAh;  // elements of A's type
  const char* Bm; int64_t sBk, sBn, sBb, sBh; // elements of B's type
  char* Y; int64_t sYm, sYn, sYb, sYh;        // elements of the output type
  int32_t M, Nn, Kd, H, accumulate, y_f32;
  int32_t splits, kchunk;                     // split-K: slices of kchunk (multiple of 16)
  float* partial;
};

template <typename TA_, typename TB_, typename TY, int BM>
__global__ void __launch_bounds__(256) gemm_kernel(const GemmParams g) {
  constexpr int BN = 4096 / BM;
  constexpr int TX = BN / 4;  // threads along n
  __shared__ float sA[16][BM + 1];
  __shared__ float sB[16][BN + 1];
  const int z = blockIdx.z;
  const int split = z % g.splits, bh = z / g.splits;
  const int b = bh / g.H, h = bh - (bh / g.H) * g.H;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int tx = threadIdx.x % TX, ty = threadIdx.x / TX;
  const TA_* A = reinterpret_cast<const TA_*>(g.A) + (int64_t)b * g.sAb + (int64_t)h * g.sAh;
  const TB_* Bm = reinterpret_cast<const TB_*>(g.Bm) + (int64_t)b * g.sBb + (int64_t)h * g.sBh;
  const int kbeg = split * g.kchunk;
  const int kend = min(g.Kd, kbeg + g.kchunk);
  float acc[4][4] = {};
  for (int k0 = kbeg; k0 < kend; k0 += 16) {
    // the fast thread index runs along whichever operand axis is contiguous
    for (int i = threadIdx.x; i < 16 * BM; i += 256) {
      const int kk = g.sAk == 1 ? (i & 15) : i / BM;
      const int mm = g.sAk == 1 ? (i >> 4) : i - kk * BM;
      const int m = m0 + mm, k = k0 + kk;
      sA[kk][mm] = (m < g.M && k < kend) ? static_cast<float>(A[(int64_t)m * g.sAm + (int64_t)k * g.sAk]) : 0.0f;
    }
    for (int i = threadIdx.x; i < 16 * BN; i += 256) {
      const int kk = g.sBk == 1 ? (i & 15) : i / BN;
      const int nn = g.sBk == 1 ? (i >> 4) : i - kk * BN;
      const int n = n0 + nn, k = k0 + kk;
      sB[kk][nn] = (n < g.Nn && k < kend) ? static_cast<float>(Bm[(int64_t)k * g.sBk + (int64_t)n * g.sBn]) : 0.0f;
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
      if (g.splits > 1) {
        const int64_t BHn = gridDim.z / g.splits;
        g.partial[(((int64_t)split * BHn + bh) * g.M + m) * g.Nn + n] = acc[i][j];
        continue;
      }
      const int64_t off = (int64_t)b * g.sYb + (int64_t)h * g.sYh + (int64_t)m * g.sYm + (int64_t)n * g.sYn;
      TY* y = reinterpret_cast<TY*>(g.Y) + off;
      *y = static_cast<TY>(g.accumulate ? static_cast<float>(*y) + acc[i][j] : acc[i][j]);
    }
  }
}

// The same products on the tensor cores (16-bit models): operands staged in shared memory as
// 16-bit values -- a float32 operand (the leaf weights W, the coefficients C) as a high and a
// low 16-bit part, Y = A_hi B + A_lo B (about 16 more mantissa bits than one part) -- and
// multiplied with mma.sync m16n8k16 into float32. Tiles of BM x BN, BM = 16 (BN = 256, the
// skinny query-block products) or 64 (BN = 64); each of the 4 warps owns 16 rows x 64 columns.
// The summation order is fixed by the tile loop, so results are bitwise repeatable.
template <typename T16> __device__ __forceinline__ uint16_t bits16(float x);
template <> __device__ __forceinline__ uint16_t bits16<__nv_bfloat16>(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}
template <> __device__ __forceinline__ uint16_t bits16<__half>(float x) {
  return __half_as_ushort(__float2half_rn(x));
}
template <typename T16> __device__ __forceinline__ float from16(uint16_t r);
template <> __device__ __forceinline__ float from16<__nv_bfloat16>(uint16_t r) { return __uint_as_float((uint32_t)r << 16); }
template <> __device__ __forceinline__ float from16<__half>(uint16_t r) { return __half2float(__ushort_as_half(r)); }

// Stage a [R rows][32 k] tile of an operand X[row * s_row + k * s_k] (float or 16-bit) into
// 16-bit high (and, for float, low) parts. Eight consecutive elements along whichever axis is
// contiguous are read per step, with one 16-byte (two for float) vector load when aligned.
template <typename TX>
__device__ __forceinline__ bool load8(const TX* ptr, bool ok, float* v) {
  if (!ok) return false;
  if constexpr (std::is_same<TX, float>::value) {
    if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0) return false;
    const float4 a = __ldg(reinterpret_cast<const float4*>(ptr));
    const float4 b = __ldg(reinterpret_cast<const float4*>(ptr) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0) return false;
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(ptr));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = from16<TX>((uint16_t)(w[j] & 0xffffu));
      v[2 * j + 1] = from16<TX>((uint16_t)(w[j] >> 16));
    }
  }
  return true;
}

template <typename TX, typename T16, bool SPLIT, int R>
__device__ __forceinline__ void stage_tile(const TX* X, int64_t s_row, int64_t s_k, int r0, int nrows,
                                           int k0, int kend, uint16_t (*hi)[40], uint16_t (*lo)[40],
                                           int tid) {
  constexpr int BK = 32;
  auto put = [&](int rr, int kk, float x) {
    const uint16_t h = bits16<T16>(x);
    hi[rr][kk] = h;
    if constexpr (SPLIT) lo[rr][kk] = bits16<T16>(x - from16<T16>(h));
  };
  if (s_k == 1) {  // contiguous along k
    for (int i = tid; i < R * (BK / 8); i += 128) {
      const int rr = i / (BK / 8), kc = (i % (BK / 8)) * 8;
      const int r = r0 + rr, k = k0 + kc;
      const TX* ptr = X + (int64_t)r * s_row + k;
      float v[8];
      if (!load8(ptr, r < nrows && k + 8 <= kend, v))
        for (int j = 0; j < 8; ++j) v[j] = (r < nrows && k + j < kend) ? static_cast<float>(ptr[j]) : 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) put(rr, kc + j, v[j]);
    }
  } else if (s_row == 1) {  // contiguous along the rows
    for (int i = tid; i < BK * (R / 8); i += 128) {
      const int kk = i / (R / 8), rc = (i % (R / 8)) * 8;
      const int r = r0 + rc, k = k0 + kk;
      const TX* ptr = X + r + (int64_t)k * s_k;
      float v[8];
      if (!load8(ptr, k < kend && r + 8 <= nrows, v))
        for (int j = 0; j < 8; ++j) v[j] = (k < kend && r + j < nrows) ? static_cast<float>(ptr[j]) : 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) put(rc + j, kk, v[j]);
    }
  } else {
    for (int i = tid; i < R * BK; i += 128) {
      const int rr = i / BK, kk = i % BK;
      const int r = r0 + rr, k = k0 + kk;
      put(rr, kk, (r < nrows && k < kend) ? static_cast<float>(X[(int64_t)r * s_row + (int64_t)k * s_k]) : 0.0f);
    }
  }
}

template <typename TA_, typename TB_, typename TY, typename T16, int BM>
__global__ void __launch_bounds__(128) gemm_mma_kernel(const GemmParams g) {
  constexpr int BN = BM == 16 ? 256 : 64;
  constexpr int BK = 32, LDS = BK + 8;
  constexpr bool AF = std::is_same<TA_, float>::value, BF = std::is_same<TB_, float>::value;
  __shared__ __align__(16) uint16_t sAh[BM][LDS];
  __shared__ __align__(16) uint16_t sAl[AF ? BM : 1][LDS];
  __shared__ __align__(16) uint16_t sBh[BN][LDS];
  __shared__ __align__(16) uint16_t sBl[BF ? BN : 1][LDS];
  const int z = blockIdx.z;
  const int split = z % g.splits, bh = z / g.splits;
  const int b = bh / g.H, h = bh - (bh / g.H) * g.H;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wm = BM == 64 ? warp * 16 : 0, wn = BM == 64 ? 0 : warp * 64;
  const TA_* A = reinterpret_cast<const TA_*>(g.A) + (int64_t)b * g.sAb + (int64_t)h * g.sAh;
  const TB_* Bm = reinterpret_cast<const TB_*>(g.Bm) + (int64_t)b * g.sBb + (int64_t)h * g.sBh;
  const int kbeg = split * g.kchunk;
  const int kend = min(g.Kd, kbeg + g.kchunk);
  float acc[8][4] = {};
  for (int k0 = kbeg; k0 < kend; k0 += BK) {
    // eight consecutive elements along the operand's contiguous axis per load (16-byte vector
    // loads where aligned), written to the [row][k] tiles
    stage_tile<TA_, T16, AF, BM>(A, g.sAm, g.sAk, m0, g.M, k0, kend, sAh, sAl, tid);
    stage_tile<TB_, T16, BF, BN>(Bm, g.sBn, g.sBk, n0, g.Nn, k0, kend, sBh, sBl, tid);
    __syncthreads();
#pragma unroll
    for (int ks = 0; ks < BK; ks += 16) {
      uint32_t ah[4], al[4];
      ldsm_x4(ah, &sAh[wm + (lane & 15)][ks + (lane >> 4) * 8]);
      if constexpr (AF) ldsm_x4(al, &sAl[wm + (lane & 15)][ks + (lane >> 4) * 8]);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int nr = wn + np * 16 + (lane >> 4) * 8 + (lane & 7);
        const int kc = ks + ((lane >> 3) & 1) * 8;
        uint32_t bh4[4];
        ldsm_x4(bh4, &sBh[nr][kc]);
        Mma16<T16>::mma(acc[2 * np], ah, bh4);
        Mma16<T16>::mma(acc[2 * np + 1], ah, bh4 + 2);
        if constexpr (AF) {
          Mma16<T16>::mma(acc[2 * np], al, bh4);
          Mma16<T16>::mma(acc[2 * np + 1], al, bh4 + 2);
        }
        if constexpr (BF) {
          uint32_t bl4[4];
          ldsm_x4(bl4, &sBl[nr][kc]);
          Mma16<T16>::mma(acc[2 * np], ah, bl4);
          Mma16<T16>::mma(acc[2 * np + 1], ah, bl4 + 2);
        }
      }
    }
    __syncthreads();
  }
  const int gq = lane >> 2, tq = lane & 3;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int m = m0 + wm + gq + (e >> 1) * 8;
      const int n = n0 + wn + t * 8 + tq * 2 + (e & 1);
      if (m >= g.M || n >= g.Nn) continue;
      if (g.splits > 1) {
        const int64_t BHn = gridDim.z / g.splits;
        g.partial[(((int64_t)split * BHn + bh) * g.M + m) * g.Nn + n] = acc[t][e];
        continue;
      }
      const int64_t off = (int64_t)b * g.sYb + (int64_t)h * g.sYh + (int64_t)m * g.sYm + (int64_t)n * g.sYn;
      TY* y = reinterpret_cast<TY*>(g.Y) + off;
      *y = static_cast<TY>(g.accumulate ? static_cast<float>(*y) + acc[t][e] : acc[t][e]);
    }
  }
}

template <typename TY>
__global__ void __launch_bounds__(256) split_reduce_kernel(const GemmParams g, int BH) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t per = (int64_t)g.M * g.Nn;
  if (i >= per * BH) return;
  const int bh = (int)(i / per);
  const int64_t r = i - bh * per;
  const int m = (int)(r / g.Nn), n = (int)(r - (int64_t)m * g.Nn);
  float t = 0.0f;
  for (int s = 0; s < g.splits; ++s) t += g.partial[((int64_t)s * BH + bh) * per + r];
  const int b = bh / g.H, h = bh - (bh / g.H) * g.H;
  TY* y = reinterpret_cast<TY*>(g.Y) + (int64_t)b * g.sYb + (int64_t)h * g.sYh + (int64_t)m * g.sYm + (int64_t)n * g.sYn;
  *y = static_cast<TY>(g.accumulate ? static_cast<float>(*y) + t : t);
}

constexpr int64_t kSplitPartialBytes = (int64_t)64 << 20;  // split-K partial tiles

template <typename TA_, typename TB_, typename TY>
static void launch_gemm(GemmParams g, int BH, cudaStream_t st, const char* what) {
  TA_PROFILE(what, st);
  // tile shape: 16 x 256 or 32 x 128 for a handful of query rows, else 64 x 64
  const int BM = g.M <= 16 && g.Nn > 128 ? 16 : (g.M <= 32 ? 32 : 64), BN = 4096 / BM;
  const int64_t tiles = (int64_t)((g.Nn + BN - 1) / BN) * ((g.M + BM - 1) / BM) * BH;
  // split k when the tile grid cannot fill the GPU several times over and k is long
  constexpr int64_t kTarget = 8 * 148;
  int splits = 1;
  if (tiles < kTarget && g.Kd >= 1024 && g.partial) {
    splits = (int)((kTarget + tiles - 1) / tiles);
    const int64_t cap = kSplitPartialBytes / ((int64_t)BH * g.M * g.Nn * 4);
    if (splits > cap) splits = (int)cap;
    if (splits > g.Kd / 256) splits = g.Kd / 256;
    if (splits < 1) splits = 1;
  }
  g.kchunk = splits > 1 ? ((g.Kd + splits - 1) / splits + 15) / 16 * 16 : g.Kd;
  if (splits > 1) splits = (g.Kd + g.kchunk - 1) / g.kchunk;
  g.splits = splits;
  // 16-bit models: the tensor-core kernel (its 16-bit type is the model's, whichever operand
  // carries it); float32 models keep the CUDA-core kernel
  using T16 = typename std::conditional<std::is_same<TA_, float>::value, TB_, TA_>::type;
  // (short reductions -- dV and dK over one query block -- are bound by their output tiles and
  // stay on the CUDA-core kernel, whose epilogue writes whole row segments)
  if (!std::is_same<T16, float>::value && g.Kd >= 128) {
    const int MB = BM == 16 ? 16 : 64, NB = MB == 16 ? 256 : 64;
    const dim3 mgrid((unsigned)((g.Nn + NB - 1) / NB), (unsigned)((g.M + MB - 1) / MB),
                     (unsigned)(BH * splits));
    if constexpr (!std::is_same<T16, float>::value) {
      if (MB == 16) gemm_mma_kernel<TA_, TB_, TY, T16, 16><<<mgrid, 128, 0, st>>>(g);
      else gemm_mma_kernel<TA_, TB_, TY, T16, 64><<<mgrid, 128, 0, st>>>(g);
    }
  } else {
    const dim3 grid((unsigned)((g.Nn + BN - 1) / BN), (unsigned)((g.M + BM - 1) / BM),
                    (unsigned)(BH * splits));
    if (BM == 16) gemm_kernel<TA_, TB_, TY, 16><<<grid, 256, 0, st>>>(g);
    else if (BM == 32) gemm_kernel<TA_, TB_, TY, 32><<<grid, 256, 0, st>>>(g);
    else gemm_kernel<TA_, TB_, TY, 64><<<grid, 256, 0, st>>>(g);
  }
  if (splits > 1) {
    const int64_t n = (int64_t)BH * g.M * g.Nn;
    split_reduce_kernel<TY><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(g, BH);
  }
}

static int64_t exact_block(int64_t L, int64_t B, int64_t H, int64_t N) {
  const int64_t per_query = B * H * (3 * N) * 4;  // node logits/C, weights, dlp (K < N)
  const int64_t budget = (int64_t)512 << 20;
  int64_t qb = budget / per_query;
  if (qb < 1) qb = 1;
  return qb < L ? qb : L;
}

template <typename T>
static int run_exact(ExactParams p, int64_t L, cudaStream_t st, bool backward, float* partial,
                     char* dq, ta_layout dql, char* dk, ta_layout dkl, char* dv, ta_layout dvl,
                     int32_t accumulate) {
  const int64_t qb = exact_block(L, p.B, p.H, p.N);
  const int BH = p.B * p.H;
  const int K = p.N - 1;
  for (int64_t l0 = 0; l0 < L; l0 += qb) {
    p.l0 = l0;
    p.nq = qb < L - l0 ? qb : L - l0;
    const unsigned rows = (unsigned)(p.nq * BH);
    // node logits S = Q K^T for the block
    GemmParams g{};
    g.partial = partial;
    g.A = p.q + (l0 * p.qs) * sizeof(T); g.sAm = p.qs; g.sAk = 1; g.sAb = p.qb; g.sAh = p.qh;
    g.Bm = p.k; g.sBk = 1; g.sBn = p.ks; g.sBb = p.kb; g.sBh = p.kh;
    g.Y = (char*)p.node_buf; g.sYm = (int64_t)BH * K; g.sYn = 1; g.sYb = (int64_t)p.H * K; g.sYh = K;
    g.M = (int32_t)p.nq; g.Nn = K; g.Kd = p.D; g.H = p.H;
    launch_gemm<T, T, float>(g, BH, st, "exact_gemm_logits");
    {
      TA_PROFILE(backward ? "exact_bwd_weights" : "exact_fwd", st);
      exact_weights_kernel<<<rows, kExactThreads, 0, st>>>(p);
    }
    int rc = check_launch("exact attention");
    if (rc) return rc;
    if (!backward) {
      // out = W V
      g = GemmParams{};
      g.partial = partial;
      g.A = (const char*)p.leaf_buf; g.sAm = (int64_t)BH * p.N; g.sAk = 1; g.sAb = (int64_t)p.H * p.N; g.sAh = p.N;
      g.Bm = p.v; g.sBk = p.vs; g.sBn = 1; g.sBb = p.vb; g.sBh = p.vh;
      g.Y = p.out + (l0 * p.os) * sizeof(T); g.sYm = p.os; g.sYn = 1; g.sYb = p.ob; g.sYh = p.oh;
      g.M = (int32_t)p.nq; g.Nn = p.D; g.Kd = p.N; g.H = p.H;
      launch_gemm<float, T, T>(g, BH, st, "exact_gemm_out");
      if ((rc = check_launch("exact attention gemm"))) return rc;
      continue;
    }
    // g_n = dO . v_n for the block
    g = GemmParams{};
    g.partial = partial;
    g.A = p.dout + (l0 * p.gs) * sizeof(T); g.sAm = p.gs; g.sAk = 1; g.sAb = p.gb; g.sAh = p.gh;
    g.Bm = p.v; g.sBk = 1; g.sBn = p.vs; g.sBb = p.vb; g.sBh = p.vh;
    g.Y = (char*)p.dlp_buf; g.sYm = (int64_t)BH * p.N; g.sYn = 1; g.sYb = (int64_t)p.H * p.N; g.sYh = p.N;
    g.M = (int32_t)p.nq; g.Nn = p.N; g.Kd = p.D; g.H = p.H;
    launch_gemm<T, T, float>(g, BH, st, "exact_gemm_g");
    // dV (+)= W^T dO
    g = GemmParams{};
    g.partial = partial;
    g.A = (const char*)p.leaf_buf; g.sAm = 1; g.sAk = (int64_t)BH * p.N; g.sAb = (int64_t)p.H * p.N; g.sAh = p.N;
    g.Bm = p.dout + (l0 * p.gs) * sizeof(T); g.sBk = p.gs; g.sBn = 1; g.sBb = p.gb; g.sBh = p.gh;
    g.Y = dv; g.sYm = dvl.seq; g.sYn = 1; g.sYb = dvl.batch; g.sYh = dvl.head;
    g.M = p.N; g.Nn = p.D; g.Kd = (int32_t)p.nq; g.H = p.H;
    g.accumulate = (accumulate || l0 > 0) ? 1 : 0;
    launch_gemm<float, T, float>(g, BH, st, "exact_gemm_dv");
    {
      TA_PROFILE("exact_bwd_coef", st);
      exact_coef_kernel<<<rows, kExactThreads, 0, st>>>(p);
    }
    if ((rc = check_launch("exact attention backward"))) return rc;
    // dq = C K   (rows of this block; written, not accumulated)
    g = GemmParams{};
    g.partial = partial;
    g.A = (const char*)p.node_buf; g.sAm = (int64_t)BH * K; g.sAk = 1; g.sAb = (int64_t)p.H * K; g.sAh = K;
    g.Bm = p.k; g.sBk = p.ks; g.sBn = 1; g.sBb = p.kb; g.sBh = p.kh;
    g.Y = dq + (l0 * dql.seq) * sizeof(T); g.sYm = dql.seq; g.sYn = 1; g.sYb = dql.batch; g.sYh = dql.head;
    g.M = (int32_t)p.nq; g.Nn = p.D; g.Kd = K; g.H = p.H;
    launch_gemm<float, T, T>(g, BH, st, "exact_gemm_dq");
    // dK (+)= C^T Q
    g = GemmParams{};
    g.partial = partial;
    g.A = (const char*)p.node_buf; g.sAm = 1; g.sAk = (int64_t)BH * K; g.sAb = (int64_t)p.H * K; g.sAh = K;
    g.Bm = p.q + (l0 * p.qs) * sizeof(T); g.sBk = p.qs; g.sBn = 1; g.sBb = p.qb; g.sBh = p.qh;
    g.Y = dk; g.sYm = dkl.seq; g.sYn = 1; g.sYb = dkl.batch; g.sYh = dkl.head;
    g.M = K; g.Nn = p.D; g.Kd = (int32_t)p.nq; g.H = p.H;
    g.accumulate = (accumulate || l0 > 0) ? 1 : 0;
    launch_gemm<float, T, float>(g, BH, st, "exact_gemm_dk");
    if ((rc = check_launch("exact attention gemm"))) return rc;
  }
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
  return (size_t)(qb * shape->batch * shape->num_heads * 3 * shape->num_leaves * 4) + 256 +
         (size_t)kSplitPartialBytes;
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
  p.partial = (float*)(((uintptr_t)(p.dlp_buf + qb * p.B * p.H * (int64_t)p.N) + 255) & ~(uintptr_t)255);
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
    case TA_F32: return run_exact<float>(p, shape->num_queries, st, false, p.partial, nullptr, {}, nullptr, {}, nullptr, {}, 0);
    case TA_F16: return run_exact<__half>(p, shape->num_queries, st, false, p.partial, nullptr, {}, nullptr, {}, nullptr, {}, 0);
    default: return run_exact<__nv_bfloat16>(p, shape->num_queries, st, false, p.partial, nullptr, {}, nullptr, {}, nullptr, {}, 0);
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
    case TA_F32: return run_exact<float>(p, shape->num_queries, st, true, p.partial, (char*)dq, dql, (char*)dk, dkl, (char*)dv, dvl, accumulate);
    case TA_F16: return run_exact<__half>(p, shape->num_queries, st, true, p.partial, (char*)dq, dql, (char*)dk, dkl, (char*)dv, dvl, accumulate);
    default: return run_exact<__nv_bfloat16>(p, shape->num_queries, st, true, p.partial, (char*)dq, dql, (char*)dk, dkl, (char*)dv, dvl, accumulate);
  }
}
