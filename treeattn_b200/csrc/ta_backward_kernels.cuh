// Fused deterministic backward of stochastic tree attention, sm_100a (typed kernels).
//
// Math (reference: _autograd.py:707-860, accumulate_qk_non_causal_all_depths_prepared.cu,
// scatter_weighted_grad_v.cu):
//   g_s   = dO . v[leaf_s]
//   dlp_s = w_s (g_s - sum_t w_t g_t)
//   gl_sd = sgn sigmoid(-sgn s_sd) dlp_s      (s_sd = clamp(q . k[node_sd]); sgn = +1 left)
//   dq    = sum_s sum_d gl_sd k[node_sd]
//   dk[n] = sum_{(s,d) through n} gl_sd q
//   dv[l] = sum_{s ending at l} w_s dO
// sigmoid(-sgn s_sd) comes from the forward (branch_prob), so no node logit is recomputed.
//
// The reference scatters dK/dV with float atomics (order-dependent results). Here the
// scatter becomes a gather over paths sorted by leaf, so every node's sum has a fixed
// order and the result is bitwise repeatable:
//   1. query pass (one 4-lane group per query): g, dlp (stored), dq (written); emits
//      (path bits, path id) records in head-major path order.
//   2. stable LSD radix sort of the records of each head by path bits (8-bit digits).
//   3. node pass: each warp owns a chunk of consecutive sorted paths. Paths through a node
//      are contiguous in this order, so the warp keeps one accumulator per depth in
//      registers and writes a node's total when the node closes. Nodes cut by a chunk
//      boundary leave a partial per side; nodes no path reaches are written as zeros.
//   4. fix-up: the chunk where a cut node starts sums the partials of the chunks it spans
//      (a fixed split over the CTA's warps, combined in warp order) and writes the node.
#pragma once

#include <type_traits>

#include "ta_common.cuh"

namespace ta {

constexpr int kBwdThreads = 256;
constexpr int kBwdGroups = kBwdThreads / 4;
constexpr int kSortThreads = 256;
constexpr int kSortItems = 8;
constexpr int kSortTile = kSortThreads * kSortItems;  // 2048 records per tile
constexpr int kRadixBits = 8;
constexpr int kRadix = 1 << kRadixBits;
constexpr int kChunk = 512;  // sorted paths per node-pass warp
constexpr int kNodeWarps = 4;
constexpr int kFixThreads = 256;

struct BwdParams {
  const char* q; const char* k; const char* v; const char* dout;
  char* dq; char* dk; char* dv;
  int64_t qs, qb, qh, ks, kb, kh, vs, vb, vh, gs, gb, gh;
  int64_t dqs, dqb, dqh, dks, dkb, dkh, dvs, dvb, dvh;
  const int32_t* leaf;
  const float* weights;
  const float* sig;    // [HB][P][sig_stride]  sigmoid(-sgn s) from the forward
  float* dlp;          // [HB][P]
  uint32_t* keys[2];   // [HB][P]
  uint32_t* vals[2];
  uint32_t* hist;      // [HB][256][tiles_per_seg]
  float* partial;      // [chunks][log_n + 1][2][D]
  uint8_t* flags;      // [chunks][log_n + 1][2]: head kind (0 none, 1 ends here, 2 through), tail
  int32_t B, L, H, S, N, D, log_n, nchunks, sig_stride;
  int32_t dk_f32;      // dk written as float32 (else input dtype)
  int64_t P;           // paths per head = L * S
  int32_t tiles_per_seg, chunks_per_seg;
  int32_t sorted_buf;  // which keys/vals buffer holds the sorted records
  float max_logit;
  int32_t top_levels;  // tree levels staged in shared memory by the query pass
  int32_t chunk;       // sorted paths per node-pass chunk
  int32_t coef_mode;   // sig holds final per-level coefficients, dlp holds value weights
  int32_t records_apart;  // the sort records were written by sort_records_kernel (not the query pass)
  int32_t dv_f32;      // dv written as float32 (else input dtype)
  int32_t node_range_chunks;  // tensor-core node pass: chunks per CTA range (0 = from the shape)
  int32_t qtable_levels;      // query pass: top levels reduced on the tensor cores (0 = none)
};

// Query pass, bf16 with head_dim a multiple of 16 (at most 128): the dq contributions of the
// top kQTableLevels levels of a CTA's 64 queries are one dense product
//     dq_top[64 x D] = C[64 x nodes] * K_top[nodes x D],  C[l][n] = sum of l's coefficients at n,
// run with mma.sync (C split into bf16 high and low parts, K exact in bf16); the deeper
// levels keep the per-lane row gathers.
constexpr int kQTableLevels = 7;
__host__ __device__ inline int qtable_cstride(int tl, int D) {
  const int a = (1 << tl) + 8, b = D + 4;  // C rows, then dq_top rows, in one region
  return a > b ? a : b;
}
__host__ __device__ inline size_t qtable_smem(int tl, int row_bytes, int D) {
  return (size_t)(1 << tl) * (row_bytes + 16) + (size_t)64 * qtable_cstride(tl, D) * 4;
}

constexpr int kChunkMma = 128;      // paths per tensor-core node-pass chunk (one per thread)
constexpr int kMTile = 32;          // G rows per MMA pass (two m16 tiles)
constexpr int kGK = 2 * kChunkMma;  // K of the product: high | low coefficient halves
constexpr int kGStride = kGK + 8;   // padded row (elements) of the G tile
constexpr int kMaxLev = 31;

__host__ __device__ inline int mma_row_stride(int D) { return D + 8; }  // padded Q/dO rows
// Shared memory of one tensor-core node-pass CTA for head_dim D and a tree of 2^ln leaves.
__host__ __device__ inline size_t mma_node_smem(int D, int ln) {
  const int lev = ln + 1;
  return (size_t)2 * kChunkMma * mma_row_stride(D) * 2  // q, dO rows (bf16)
         + (size_t)kMTile * kGStride * 2                 // G tile (bf16)
         + (size_t)lev * kChunkMma * 4                   // coefficients [level][path]
         + (size_t)2 * lev * D * 4                       // carried node rows, two parities
         + (size_t)2 * kChunkMma * 4                     // query rows of two sub-chunks
         + (size_t)kMTile * 4 * 2                        // tile rows: run key, level
         + (size_t)4 * kMaxLev * 4                       // run-start masks [warp][level]
         + (size_t)kMaxLev * 4 * 2                       // rows per level, row offsets
         + (size_t)2 * kMaxLev * 4                       // carried-node origin, two parities
         + (size_t)4 * kMaxLev * 4 + 64;                 // per-warp run prefixes
}
constexpr size_t kMaxBlockSmem = 227 * 1024;

// The tensor-core node pass serves 16-bit inputs whose head_dim is a multiple of 32 (<= 256)
// and whose CTA fits the shared-memory limit.
inline bool use_mma_node_pass(int32_t dtype, int64_t D, int ln) {
  return (dtype == TA_BF16 || dtype == TA_F16) && D % 32 == 0 && D <= 256 && D / 32 != 5 && D / 32 != 6 && D / 32 != 7 &&
         mma_node_smem((int)D, ln) <= kMaxBlockSmem;
}

// radix-sort kernels (ta_backward.cu)
__global__ void sort_hist_kernel(const BwdParams p, int src, int shift);
__global__ void sort_scan_kernel(const BwdParams p);
__global__ void sort_scatter_kernel(const BwdParams p, int src, int shift);
int run_sort(BwdParams& p, cudaStream_t st);

// ---------------------------------------------------------------------------------------
// 1. query pass
// ---------------------------------------------------------------------------------------
template <typename T, int CPL>
__global__ void __launch_bounds__(kBwdThreads, 2) bwd_query_kernel(const BwdParams p) {
  using E = Elem<T>;
  constexpr int EPC = E::EPC;
  constexpr int NE = CPL * EPC;
  constexpr int DU = 4;  // depths whose rows are in flight together
  extern __shared__ float smem[];

  const int ltiles = (p.L + kBwdGroups - 1) / kBwdGroups;
  const int bh = blockIdx.x / ltiles;
  const int lt = blockIdx.x - bh * ltiles;
  const int b = bh / p.H;
  const int h = bh - b * p.H;
  const int g = threadIdx.x >> 2;
  const int t4 = threadIdx.x & 3;
  const int l = lt * kBwdGroups + g;
  const unsigned gmask = 0xFu << (threadIdx.x & 28);
  const int row_bytes = p.nchunks * 16;
  const int top_rows = (1 << p.top_levels) - 1;
  const int tlq = p.qtable_levels;
  char* s_tree = reinterpret_cast<char*>(smem);
  const uint32_t s_tree_sa = (uint32_t)__cvta_generic_to_shared(s_tree);
  // table mode: K_top rows (padded by 16 bytes) then the C / dq_top region
  const int kts = row_bytes + 16;
  const int cstride = qtable_cstride(tlq, p.nchunks * 8);
  float* s_C = reinterpret_cast<float*>(s_tree + (size_t)(1 << tlq) * kts);
  char* s_after = tlq > 0 ? s_tree + qtable_smem(tlq, row_bytes, p.nchunks * 8)
                          : s_tree + (size_t)top_rows * row_bytes;
  float* s_dlp = reinterpret_cast<float*>(s_after) + g * p.S;

  const uint32_t K = (uint32_t)p.N - 1u;
  const uint32_t base_node = (1u << p.log_n) - 1u;
  const int64_t j0 = (((int64_t)l * p.B + b) * p.H + h) * p.S;
  const int64_t hb = (int64_t)b * p.H + h;
  const int64_t path0 = hb * p.P + (int64_t)l * p.S;  // head-major path index of sample 0

  const char* vbase = p.v + ((int64_t)b * p.vb + (int64_t)h * p.vh) * sizeof(T);
  const uint32_t vstride = (uint32_t)(p.vs * (int64_t)sizeof(T));
  const char* kbase = p.k + ((int64_t)b * p.kb + (int64_t)h * p.kh) * sizeof(T);
  const uint32_t kstride = (uint32_t)(p.ks * (int64_t)sizeof(T));
  if (top_rows > 0) {
    stage_tree_rows(s_tree, kbase, kstride, top_rows, row_bytes);
    cp_async_wait_0();
    __syncthreads();
  }
  if (tlq > 0) {  // K_top rows 0 .. 2^tlq - 2 (padded stride), then one zero row
    const int rows = (1 << tlq) - 1, ppr = row_bytes >> 4;
    for (int i = threadIdx.x; i < rows * ppr; i += kBwdThreads) {
      const int r = i / ppr, c = i - r * ppr;
      cp_async16(s_tree + r * kts + c * 16, kbase + (uint64_t)r * kstride + c * 16);
    }
    cp_async_commit();
    for (int c = threadIdx.x; c < ppr; c += kBwdThreads)
      *reinterpret_cast<uint4*>(s_tree + rows * kts + c * 16) = make_uint4(0, 0, 0, 0);
  }
  // groups past the last query stay until the table product's barriers are done
  const bool active = l < p.L;
  if (tlq == 0 && !active) return;

  // g_s = dO . v[leaf_s]
  if (active && !p.coef_mode) {
    uint4 graw[CPL];
    const char* grow = p.dout + ((int64_t)l * p.gs + (int64_t)b * p.gb + (int64_t)h * p.gh) * sizeof(T);
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int c = i * 4 + t4;
      graw[i] = c < p.nchunks ? ldg16(grow + c * 16) : make_uint4(0, 0, 0, 0);
    }
    for (int s0 = 0; s0 < p.S; s0 += 4) {
      uint4 raw[4][CPL];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int s = min(s0 + t, p.S - 1);
        int32_t lf = p.leaf[j0 + s];
        lf = lf < 0 ? 0 : (lf >= p.N ? p.N - 1 : lf);
        const char* vrow = vbase + (uint64_t)(uint32_t)lf * vstride;
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
          const int c = i * 4 + t4;
          raw[t][i] = c < p.nchunks ? ldg16(vrow + c * 16) : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        float d = 0.0f;
#pragma unroll
        for (int i = 0; i < CPL; ++i) d = Dot<T>::chunk(graw[i], raw[t][i], d);
        d += __shfl_xor_sync(gmask, d, 1, 4);
        d += __shfl_xor_sync(gmask, d, 2, 4);
        if (t4 == t && s0 + t < p.S) s_dlp[s0 + t] = d;
      }
    }
  }
  __syncwarp(gmask);
  if (active && !p.coef_mode) {
    // dlp_s = w_s (g_s - sum_t w_t g_t)
    float wg = 0.0f;
    for (int s = 0; s < p.S; ++s) wg = fmaf(p.weights[j0 + s], s_dlp[s], wg);
    __syncwarp(gmask);
    for (int s = t4; s < p.S; s += 4) {
      const float d = p.weights[j0 + s] * (s_dlp[s] - wg);
      s_dlp[s] = d;
      p.dlp[path0 + s] = d;
      // sort record of path s: (path bits, path id within its head)
      if (!p.records_apart) {
        p.keys[0][path0 + s] = (uint32_t)p.leaf[j0 + s] + K - base_node;
        p.vals[0][path0 + s] = (uint32_t)(l * p.S + s);
      }
    }
  }
  __syncwarp(gmask);

  // dq = sum_s sum_d sgn sig dlp k[node]
  float acc[NE];
#pragma unroll
  for (int e = 0; e < NE; ++e) acc[e] = 0.0f;
  if constexpr (std::is_same<T, __nv_bfloat16>::value && CPL <= 4) {
    if (tlq > 0) {
      // C row of this query: lane t4 adds the levels d = t4 (mod 4), paths in order
      float* crow = s_C + g * cstride;
      for (int c = t4; c < (1 << tlq); c += 4) crow[c] = 0.0f;
      __syncwarp(gmask);
      if (active) {
        for (int s = 0; s < p.S; ++s) {
          const uint32_t bits = p.coef_mode ? p.keys[0][path0 + s] : (uint32_t)p.leaf[j0 + s] + K - base_node;
          const float dlp = p.coef_mode ? 1.0f : s_dlp[s];
          const float* sig = p.sig + (path0 + s) * p.sig_stride;
          for (int d = t4; d < tlq; d += 4) {
            const uint32_t node = (1u << d) - 1u + (bits >> (p.log_n - d));
            const float sgn = (!p.coef_mode && ((bits >> (p.log_n - 1 - d)) & 1u)) ? -1.0f : 1.0f;
            crow[node] += sgn * __ldg(sig + d) * dlp;
          }
        }
      }
      cp_async_wait_0();
      __syncthreads();
      // dq_top: warp w takes query rows [16 (w % 4), +16) and column half w / 4
      const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
      const int mt = warp & 3, gq = lane >> 2, tq = lane & 3;
      const int D = p.nchunks * 8, ntiles = D / 16;
      const int n0 = (warp >> 2) * (D / 2);
      const T* s_kt = reinterpret_cast<const T*>(s_tree);
      const int kre = kts / 2;  // padded row in elements
      float dacc[2 * CPL][4];
#pragma unroll
      for (int nt = 0; nt < 2 * CPL; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) dacc[nt][e] = 0.0f;
      auto split = [](float2 x, uint32_t& hi, uint32_t& lo) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(x.x, x.y);
        const __nv_bfloat162 r = __floats2bfloat162_rn(x.x - __bfloat162float(h.x), x.y - __bfloat162float(h.y));
        hi = *reinterpret_cast<const uint32_t*>(&h);
        lo = *reinterpret_cast<const uint32_t*>(&r);
      };
      for (int nb = 0; nb < (1 << tlq) / 16; ++nb) {
        const float* c0 = s_C + (mt * 16 + gq) * cstride + nb * 16 + 2 * tq;
        const float* c1 = c0 + 8 * cstride;
        uint32_t ahi[4], alo[4];
        split(*reinterpret_cast<const float2*>(c0), ahi[0], alo[0]);
        split(*reinterpret_cast<const float2*>(c1), ahi[1], alo[1]);
        split(*reinterpret_cast<const float2*>(c0 + 8), ahi[2], alo[2]);
        split(*reinterpret_cast<const float2*>(c1 + 8), ahi[3], alo[3]);
#pragma unroll
        for (int nt = 0; nt < 2 * CPL; ++nt) {
          if (nt < ntiles) {
            uint32_t bfr[2];
            ldsm_x2_trans(bfr, s_kt + (nb * 16 + (lane & 15)) * kre + n0 + nt * 8);
            mma_bf16(dacc[nt], ahi, bfr);
            mma_bf16(dacc[nt], alo, bfr);
          }
        }
      }
      __syncthreads();  // C reads done: the region takes dq_top [64][D + 4]
#pragma unroll
      for (int nt = 0; nt < 2 * CPL; ++nt) {
        if (nt < ntiles) {
          const int col = n0 + nt * 8 + 2 * tq;
          *reinterpret_cast<float2*>(s_C + (mt * 16 + gq) * cstride + col) = make_float2(dacc[nt][0], dacc[nt][1]);
          *reinterpret_cast<float2*>(s_C + (mt * 16 + gq + 8) * cstride + col) = make_float2(dacc[nt][2], dacc[nt][3]);
        }
      }
      __syncthreads();
      if (!active) return;
#pragma unroll
      for (int i = 0; i < CPL; ++i) {
        const int c = i * 4 + t4;
        if (c < p.nchunks) {
#pragma unroll
          for (int e = 0; e < EPC; ++e) acc[i * EPC + e] = s_C[g * cstride + c * EPC + e];
        }
      }
    }
  }
  for (int s = 0; s < p.S; ++s) {
    // coefficient mode: the records were written by the caller (before the sort)
    const uint32_t bits = p.coef_mode ? p.keys[0][path0 + s] : (uint32_t)p.leaf[j0 + s] + K - base_node;
    const float dlp = p.coef_mode ? 1.0f : s_dlp[s];
    const float* sig = p.sig + (path0 + s) * p.sig_stride;
    for (int d0 = tlq; d0 < p.log_n; d0 += DU) {
      uint4 raw[DU][CPL];
      float gl[DU];
#pragma unroll
      for (int u = 0; u < DU; ++u) {
        const int d = min(d0 + u, p.log_n - 1);
        const uint32_t node = (1u << d) - 1u + (bits >> (p.log_n - d));
        if (d < p.top_levels) {
          const uint32_t krow = s_tree_sa + node * (uint32_t)row_bytes;
#pragma unroll
          for (int i = 0; i < CPL; ++i) {
            const int c = i * 4 + t4;
            raw[u][i] = c < p.nchunks ? lds16_sa(krow + c * 16) : make_uint4(0, 0, 0, 0);
          }
        } else {
          const char* krow = kbase + (uint64_t)node * kstride;
#pragma unroll
          for (int i = 0; i < CPL; ++i) {
            const int c = i * 4 + t4;
            raw[u][i] = c < p.nchunks ? ldg16(krow + c * 16) : make_uint4(0, 0, 0, 0);
          }
        }
        const float sgn = (!p.coef_mode && ((bits >> (p.log_n - 1 - d)) & 1u)) ? -1.0f : 1.0f;
        gl[u] = d0 + u < p.log_n ? sgn * __ldg(sig + d) * dlp : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < DU; ++u) {
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
          float kf[EPC];
          E::unpack(raw[u][i], kf);
#pragma unroll
          for (int e = 0; e < EPC; e += 2) ffma2(acc[i * EPC + e], acc[i * EPC + e + 1], gl[u], kf[e], kf[e + 1]);
        }
      }
    }
  }
  char* orow = p.dq + ((int64_t)l * p.dqs + (int64_t)b * p.dqb + (int64_t)h * p.dqh) * sizeof(T);
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = i * 4 + t4;
    if (c < p.nchunks) st16(orow + c * 16, E::pack(acc + i * EPC));
  }
}

// ---------------------------------------------------------------------------------------
// 3. node pass over leaf-sorted paths
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void ffma2(float2& acc, float2 a, float2 b) {
  uint64_t c, x, y;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a.x), "f"(a.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(y) : "f"(b.x), "f"(b.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(c) : "f"(acc.x), "f"(acc.y));
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(c) : "l"(x), "l"(y));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(acc.x), "=f"(acc.y) : "l"(c));
}

// A lane's slice of a row: EP element pairs (2*EP consecutive elements), packed on load.
template <typename T, int EP>
struct Slice {
  uint32_t w[sizeof(T) == 2 ? EP : 2 * EP];
  __device__ __forceinline__ void load(const char* row, int lane, int D) {
    const bool ok = lane * 2 * EP < D;
    if constexpr (sizeof(T) == 2) {
      const uint32_t* r = reinterpret_cast<const uint32_t*>(row) + lane * EP;
      if constexpr (EP == 2) {
        const uint2 u = ok ? __ldg(reinterpret_cast<const uint2*>(r)) : make_uint2(0, 0);
        w[0] = u.x; w[1] = u.y;
      } else {
#pragma unroll
        for (int i = 0; i < EP; ++i) w[i] = ok ? __ldg(r + i) : 0u;
      }
    } else if constexpr (EP == 2) {
      const uint4 u = ok ? __ldg(reinterpret_cast<const uint4*>(row) + lane) : make_uint4(0, 0, 0, 0);
      w[0] = u.x; w[1] = u.y; w[2] = u.z; w[3] = u.w;
    } else {
      const uint32_t* r = reinterpret_cast<const uint32_t*>(row) + lane * 2 * EP;
#pragma unroll
      for (int i = 0; i < 2 * EP; ++i) w[i] = ok ? __ldg(r + i) : 0u;
    }
  }
  // plain (generic) loads, for rows staged in shared memory
  __device__ __forceinline__ void load_plain(const char* row, int lane, int D) {
    const bool ok = lane * 2 * EP < D;
    if constexpr (sizeof(T) == 2 && EP == 2) {
      const uint2 u = ok ? *reinterpret_cast<const uint2*>(reinterpret_cast<const uint32_t*>(row) + lane * EP)
                         : make_uint2(0, 0);
      w[0] = u.x; w[1] = u.y;
    } else if constexpr (sizeof(T) == 4 && EP == 2) {
      const uint4 u = ok ? *(reinterpret_cast<const uint4*>(row) + lane) : make_uint4(0, 0, 0, 0);
      w[0] = u.x; w[1] = u.y; w[2] = u.z; w[3] = u.w;
    } else {
      constexpr int NW = sizeof(T) == 2 ? EP : 2 * EP;
      const uint32_t* r = reinterpret_cast<const uint32_t*>(row) + lane * NW;
#pragma unroll
      for (int i = 0; i < NW; ++i) w[i] = ok ? r[i] : 0u;
    }
  }
  __device__ __forceinline__ float2 pair(int i) const {
    if constexpr (sizeof(T) == 2) {
      float f[2];
      Elem<T>::unpack2(w[i], f);
      return make_float2(f[0], f[1]);
    } else {
      return make_float2(__uint_as_float(w[2 * i]), __uint_as_float(w[2 * i + 1]));
    }
  }
};

template <typename T>
__device__ __forceinline__ void store_pairs(char* row, int lane, int EP, int D, const float2* f,
                                            bool f32) {
  for (int i = 0; i < EP; ++i) {
    const int c = (lane * EP + i) * 2;
    if (c < D) {
      if (f32) {
        *reinterpret_cast<float2*>(reinterpret_cast<float*>(row) + c) = f[i];
      } else {
        reinterpret_cast<T*>(row)[c] = static_cast<T>(f[i].x);
        reinterpret_cast<T*>(row)[c + 1] = static_cast<T>(f[i].y);
      }
    }
  }
}

constexpr int kNodeBatch = 8;  // paths staged per batch
constexpr int kMaxLevels = 31;  // tree depths + 1 (leaf level)

// Per-warp shared memory of the node pass (bytes): two staging buffers of one batch (q rows,
// dO rows, per-depth coefficients, weight, key) plus the open-node accumulators of every
// level and the prefix of each open node.
__host__ __device__ inline int node_stage_bytes(int row_bytes) {
  return kNodeBatch * (2 * row_bytes + 32 * 4 + 4 + 4 + 4) + 33 * kNodeBatch * 4;
}
__host__ __device__ inline int node_warp_bytes(int row_bytes, int D, int levels) {
  return 2 * node_stage_bytes(row_bytes) + levels * D * 4 + 32 * 4;
}

// One warp walks a chunk of kChunk consecutive leaf-sorted paths of one head. Lanes own
// 2*EP consecutive elements of D. Batches of kNodeBatch paths are staged into shared
// memory with cp.async (double-buffered); then, level by level (depth d in [0, log_n) for
// dK, d == log_n for dV), the warp adds the batch's contributions gl_{p,d} q_p (or w_p dO_p)
// into the accumulator of the open node of that level, writing a node out whenever the
// run of paths through it ends. Paths through one node are consecutive, so each node's sum
// is formed in sorted-path order: deterministic.
template <typename T, int EP>
__global__ void __launch_bounds__(kNodeWarps * 32) bwd_node_kernel(const BwdParams p) {
  extern __shared__ __align__(16) unsigned char s_node[];
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  const int64_t chunk = (int64_t)blockIdx.x * kNodeWarps + wid;
  const int64_t nchunks_total = (int64_t)p.B * p.H * p.chunks_per_seg;
  if (chunk >= nchunks_total) return;
  const int row_bytes = p.D * (int)sizeof(T);
  const int stage_bytes = node_stage_bytes(row_bytes);
  unsigned char* wmem = s_node + (size_t)wid * node_warp_bytes(row_bytes, p.D, p.log_n + 1);
  float* s_acc = reinterpret_cast<float*>(wmem + 2 * stage_bytes);  // [log_n + 1][D]
  uint32_t* s_pre = reinterpret_cast<uint32_t*>(s_acc + (p.log_n + 1) * p.D);  // open node prefix

  const int seg = (int)(chunk / p.chunks_per_seg);
  const int cis = (int)(chunk - (int64_t)seg * p.chunks_per_seg);
  const int b = seg / p.H, h = seg - (seg / p.H) * p.H;
  const int ln = p.log_n;
  const int64_t i0 = (int64_t)cis * p.chunk;
  const int64_t i1 = min(i0 + p.chunk, p.P);
  const uint32_t* keys = p.keys[p.sorted_buf] + (int64_t)seg * p.P;
  const uint32_t* vals = p.vals[p.sorted_buf] + (int64_t)seg * p.P;
  const float* sig = p.sig + (int64_t)seg * p.P * p.sig_stride;
  const float* dlp = p.dlp + (int64_t)seg * p.P;

  const int64_t base_node = ((int64_t)1 << ln) - 1;
  const int64_t K = (int64_t)p.N - 1;
  const int64_t dk_es = p.dk_f32 ? 4 : (int64_t)sizeof(T);
  char* dkb = p.dk + ((int64_t)b * p.dkb + (int64_t)h * p.dkh) * dk_es;
  const int64_t dk_row = p.dks * dk_es;
  const int64_t dv_es = p.dv_f32 ? 4 : (int64_t)sizeof(T);
  char* dvb = p.dv + ((int64_t)b * p.dvb + (int64_t)h * p.dvh) * dv_es;
  const int64_t dv_row = p.dvs * dv_es;
  const char* qbase = p.q + ((int64_t)b * p.qb + (int64_t)h * p.qh) * sizeof(T);
  const int64_t q_row = p.qs * (int64_t)sizeof(T);
  const char* gbase = p.dout + ((int64_t)b * p.gb + (int64_t)h * p.gh) * sizeof(T);
  const int64_t g_row = p.gs * (int64_t)sizeof(T);
  float* part = p.partial + chunk * (int64_t)(ln + 1) * 2 * p.D;
  uint8_t* flg = p.flags + chunk * (int64_t)(ln + 1) * 2;

  // node of level d with prefix `pre` (d == ln: the leaf)
  auto node_index = [&](int d, uint32_t pre) -> int64_t {
    return d < ln ? ((int64_t)1 << d) - 1 + pre : (int64_t)pre + base_node - K;
  };
  auto write_row = [&](int d, int64_t node, const float2* f) {
    if (d < ln) store_pairs<T>(dkb + node * dk_row, lane, EP, p.D, f, p.dk_f32);
    else store_pairs<T>(dvb + node * dv_row, lane, EP, p.D, f, p.dv_f32);
  };
  auto put_partial = [&](int slot, const float2* f) {
    float* dst = part + (int64_t)slot * p.D;
    for (int i = 0; i < EP; ++i) {
      const int c = (lane * EP + i) * 2;
      if (c < p.D) *reinterpret_cast<float2*>(dst + c) = f[i];
    }
  };
  const float2 zero2[EP] = {};
  // zero the nodes of level d with prefixes in [lo, hi]
  auto zero_range = [&](int d, int64_t lo, int64_t hi) {
    for (int64_t pf = lo; pf <= hi; ++pf) write_row(d, node_index(d, (uint32_t)pf), zero2);
  };
  auto shared_depths = [&](uint32_t a, uint32_t c) -> int {
    const uint32_t x = a ^ c;
    return x == 0 ? ln + 1 : ln - (32 - __clz(x)) + 1;
  };
  // stage the batch starting at sorted index ib into buffer `buf` (asynchronous)
  auto stage = [&](int buf, int64_t ib) {
    unsigned char* st = wmem + (size_t)buf * stage_bytes;
    char* sq = reinterpret_cast<char*>(st);
    char* sg = sq + kNodeBatch * row_bytes;
    float* sco = reinterpret_cast<float*>(sg + kNodeBatch * row_bytes);
    float* sdl = sco + kNodeBatch * 32;
    float* sw = sdl + kNodeBatch;
    uint32_t* skey = reinterpret_cast<uint32_t*>(sw + kNodeBatch);
    const int nb = (int)min((int64_t)kNodeBatch, i1 - ib);
    uint32_t pl = 0, l = 0;
    if (lane < nb) {
      const uint32_t key = keys[ib + lane];
      pl = vals[ib + lane];
      l = pl / (uint32_t)p.S;
      const uint32_t s = pl - l * (uint32_t)p.S;
      skey[lane] = key;
      cp_async4(sdl + lane, dlp + pl);
      if (p.coef_mode) cp_async4(sw + lane, dlp + pl);  // value weight of the path
      else cp_async4(sw + lane, p.weights + (((int64_t)l * p.B + b) * p.H + h) * p.S + s);
    }
    const int cpr = row_bytes / 16;
    const int q4 = p.sig_stride >> 2;
    for (int r = 0; r < nb; ++r) {
      const uint32_t lr = __shfl_sync(0xffffffffu, l, r);
      const uint32_t pr = __shfl_sync(0xffffffffu, pl, r);
      for (int c = lane; c < cpr; c += 32) {
        cp_async16(sq + r * row_bytes + c * 16, qbase + (int64_t)lr * q_row + c * 16);
        cp_async16(sg + r * row_bytes + c * 16, gbase + (int64_t)lr * g_row + c * 16);
      }
      if (lane < q4) cp_async16(sco + r * 32 + 4 * lane, sig + (int64_t)pr * p.sig_stride + 4 * lane);
    }
    cp_async_commit();
  };

  // chunk start: open nodes, accumulators, flags
  const uint32_t first = keys[i0];
  uint32_t open_before = 0;  // levels whose open node started before this chunk
  if (i0 > 0) {
    const int sd = shared_depths(keys[i0 - 1], first);
    open_before = sd >= 32 ? 0xffffffffu : ((1u << sd) - 1u);
  }
  for (int i = lane; i < (ln + 1) * p.D; i += 32) s_acc[i] = 0.0f;
  for (int d = lane; d <= ln; d += 32) {
    s_pre[d] = first >> (ln - d);
    flg[2 * d] = 0;
    flg[2 * d + 1] = 0;
  }
  if (i0 == 0) {  // nodes left of the head's first path are unreached
    for (int d = 0; d <= ln; ++d) {
      const int64_t hi = (int64_t)(first >> (ln - d)) - 1;
      if (hi >= 0) zero_range(d, 0, hi);
    }
  }
  __syncwarp();

  stage(0, i0);
  int buf = 0;
  uint32_t prev = first;  // key of the path before the current batch (chunk start: itself)
  for (int64_t ib = i0; ib < i1; ib += kNodeBatch, buf ^= 1) {
    if (ib + kNodeBatch < i1) {
      stage(buf ^ 1, ib + kNodeBatch);
      cp_async_wait_1();
    } else {
      cp_async_wait_0();
    }
    __syncwarp();
    unsigned char* st = wmem + (size_t)buf * stage_bytes;
    const char* sq = reinterpret_cast<const char*>(st);
    const char* sg = sq + kNodeBatch * row_bytes;
    float* sco = reinterpret_cast<float*>(const_cast<char*>(sg) + kNodeBatch * row_bytes);
    const float* sdl = sco + kNodeBatch * 32;
    const float* sw = sdl + kNodeBatch;
    const uint32_t* skey = reinterpret_cast<const uint32_t*>(sw + kNodeBatch);
    const int nb = (int)min((int64_t)kNodeBatch, i1 - ib);
    // coefficients gl = sgn * sigmoid(-sgn s) * dlp, transposed to [level][path] (level ln:
    // the weights, for dV) so one level's coefficients of the batch are two float4 loads
    float* sct = reinterpret_cast<float*>(const_cast<uint32_t*>(skey) + kNodeBatch);  // [33][8]
    for (int idx = lane; idx < nb * 32; idx += 32) {
      const int r = idx >> 5, d = idx & 31;
      float co = 0.0f;
      if (d < ln) {
        const float sv = sco[r * 32 + d];
        co = p.coef_mode ? sv : (((skey[r] >> (ln - 1 - d)) & 1u) ? -sv : sv) * sdl[r];
      } else if (d == ln) {
        co = sw[r];
      }
      if (d <= ln) sct[d * kNodeBatch + r] = co;
    }
    if (nb < kNodeBatch)
      for (int idx = lane; idx < (ln + 1) * kNodeBatch; idx += 32)
        if ((idx % kNodeBatch) >= nb) sct[idx] = 0.0f;
    // run boundaries: lane d holds the bitmask of batch paths that start a new node at level d
    uint32_t bmask = 0;
    {
      uint32_t pk = prev;
      for (int r = 0; r < nb; ++r) {
        const uint32_t kk = skey[r];
        const int sd = shared_depths(pk, kk);
        if (sd <= lane) bmask |= 1u << r;
        pk = kk;
      }
    }
    __syncwarp();
    // this batch's q slices, unpacked
    float2 qv[kNodeBatch][EP];
#pragma unroll
    for (int r = 0; r < kNodeBatch; ++r) {
      if (r < nb) {  // staged rows past the batch end are stale: keep them out of the sums
        Slice<T, EP> row;
        row.load_plain(sq + r * row_bytes, lane, p.D);
#pragma unroll
        for (int i = 0; i < EP; ++i) qv[r][i] = row.pair(i);
      } else {
#pragma unroll
        for (int i = 0; i < EP; ++i) qv[r][i] = make_float2(0.0f, 0.0f);
      }
    }
    for (int d = 0; d <= ln; ++d) {
      const bool leaf = d == ln;
      float2 a[EP];
      float* ad = s_acc + d * p.D;
#pragma unroll
      for (int i = 0; i < EP; ++i) {
        const int c = (lane * EP + i) * 2;
        a[i] = c < p.D ? *reinterpret_cast<const float2*>(ad + c) : make_float2(0.0f, 0.0f);
      }
      const float4 c0 = reinterpret_cast<const float4*>(sct + d * kNodeBatch)[0];
      const float4 c1 = reinterpret_cast<const float4*>(sct + d * kNodeBatch)[1];
      const float co[kNodeBatch] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      const uint32_t m = __shfl_sync(0xffffffffu, bmask, d & 31);
      if (!leaf && m == 0) {
        // no node of this level ends inside the batch
#pragma unroll
        for (int r = 0; r < kNodeBatch; ++r)
#pragma unroll
          for (int i = 0; i < EP; ++i) {
            a[i].x = fmaf(co[r], qv[r][i].x, a[i].x);
            a[i].y = fmaf(co[r], qv[r][i].y, a[i].y);
          }
      } else {
        uint32_t pre = s_pre[d];
#pragma unroll
        for (int r = 0; r < kNodeBatch; ++r) {
          if ((m >> r) & 1u) {  // the run of node `pre` ends before path r
            if ((open_before >> d) & 1u) {
              put_partial(2 * d, a);
              if (lane == 0) flg[2 * d] = 1;
              open_before &= ~(1u << d);
            } else {
              write_row(d, node_index(d, pre), a);
            }
#pragma unroll
            for (int i = 0; i < EP; ++i) a[i] = make_float2(0.0f, 0.0f);
            const uint32_t npre = skey[r] >> (ln - d);
            if (npre > pre + 1u) zero_range(d, (int64_t)pre + 1, (int64_t)npre - 1);
            pre = npre;
          }
          float2 v[EP];
          if (leaf && r < nb) {
            Slice<T, EP> row;
            row.load_plain(sg + r * row_bytes, lane, p.D);
#pragma unroll
            for (int i = 0; i < EP; ++i) v[i] = row.pair(i);
          } else {
#pragma unroll
            for (int i = 0; i < EP; ++i) v[i] = qv[r][i];
          }
#pragma unroll
          for (int i = 0; i < EP; ++i) {
            a[i].x = fmaf(co[r], v[i].x, a[i].x);
            a[i].y = fmaf(co[r], v[i].y, a[i].y);
          }
        }
        if (lane == 0) s_pre[d] = pre;
      }
#pragma unroll
      for (int i = 0; i < EP; ++i) {
        const int c = (lane * EP + i) * 2;
        if (c < p.D) *reinterpret_cast<float2*>(ad + c) = a[i];
      }
    }
    prev = skey[nb - 1];
    __syncwarp();
  }

  // chunk end: close or hand over every open node
  const bool has_next = i1 < p.P;
  const uint32_t nxt = has_next ? keys[i1] : 0u;
  const int sd_next = has_next ? shared_depths(prev, nxt) : 0;
  for (int d = 0; d <= ln; ++d) {
    float2 a[EP];
    const float* ad = s_acc + d * p.D;
#pragma unroll
    for (int i = 0; i < EP; ++i) {
      const int c = (lane * EP + i) * 2;
      a[i] = c < p.D ? *reinterpret_cast<const float2*>(ad + c) : make_float2(0.0f, 0.0f);
    }
    const uint32_t pre = s_pre[d];
    const bool cont = d < sd_next;  // node continues into the next chunk
    const bool before = (open_before >> d) & 1u;
    if (cont) {
      put_partial(2 * d + (before ? 0 : 1), a);
      if (lane == 0) {
        if (before) flg[2 * d] = 2;      // passes through this chunk
        else flg[2 * d + 1] = 1;         // starts here: this chunk owns the fix-up
      }
    } else {
      if (before) {
        put_partial(2 * d, a);
        if (lane == 0) flg[2 * d] = 1;
      } else {
        write_row(d, node_index(d, pre), a);
      }
      // unreached nodes up to the next path (or to the end of the level)
      const int64_t hi = has_next ? (int64_t)(nxt >> (ln - d)) - 1 : ((int64_t)1 << d) - 1;
      if (hi > (int64_t)pre) zero_range(d, (int64_t)pre + 1, hi);
    }
  }
}

// ---------------------------------------------------------------------------------------
// 4. fix-up of nodes cut by chunk boundaries: one CTA per chunk, for every level at which
// the chunk owns a cut node. The chunks the node spans are split into contiguous ranges,
// one per warp (each summed in chunk order), and the warp sums are added in warp order.
// ---------------------------------------------------------------------------------------
constexpr int kFixWarps = 4;

template <typename T>
__global__ void __launch_bounds__(kFixWarps * 32) bwd_fixup_kernel(const BwdParams p) {
  __shared__ float s_part[kFixWarps][256];
  __shared__ int64_t s_cend;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t chunk = blockIdx.x;
  const int ln = p.log_n;
  const int seg = (int)(chunk / p.chunks_per_seg);
  const int64_t cis = chunk - (int64_t)seg * p.chunks_per_seg;
  const int64_t seg_end = (int64_t)(seg + 1) * p.chunks_per_seg;  // first chunk of the next head
  const int b = seg / p.H, h = seg - (seg / p.H) * p.H;
  const int64_t stride = (int64_t)(ln + 1) * 2;
  const uint8_t* flg = p.flags;
  const int64_t base_node = ((int64_t)1 << ln) - 1;
  uint32_t key = 0;
  bool have_key = false;
  for (int d = 0; d <= ln; ++d) {
    if (flg[chunk * stride + 2 * d + 1] == 0) continue;  // not the owner of a cut node
    if (!have_key) {
      const int64_t i_last = min((cis + 1) * (int64_t)p.chunk, p.P) - 1;
      key = p.keys[p.sorted_buf][(int64_t)seg * p.P + i_last];
      have_key = true;
    }
    // the node spans chunk+1 .. c_end: chunks flagged "through" followed by one "ends here"
    if (warp == 0) {
      int64_t c_end = chunk + 1;
      for (int64_t c0 = chunk + 1; c0 < seg_end; c0 += 32) {
        const int64_t c = c0 + lane;
        const bool ends = c < seg_end && flg[c * stride + 2 * d] != 2;
        const unsigned m = __ballot_sync(0xffffffffu, ends);
        if (m) {
          c_end = c0 + __ffs(m) - 1;
          break;
        }
      }
      if (lane == 0) s_cend = c_end;
    }
    __syncthreads();
    const int64_t c_end = s_cend;
    const int64_t span = c_end - chunk;  // chunks after this one
    const int64_t per = (span + kFixWarps - 1) / kFixWarps;
    const int64_t c_lo = chunk + 1 + warp * per;
    const int64_t c_hi = min(chunk + 1 + (warp + 1) * per, c_end + 1);
    for (int c0 = lane * 2; c0 < p.D; c0 += 64) {
      float2 tot = make_float2(0.0f, 0.0f);
      int64_t c = c_lo;
      for (; c + 8 <= c_hi; c += 8) {
        float2 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          v[u] = *reinterpret_cast<const float2*>(p.partial + ((c + u) * stride + 2 * d) * p.D + c0);
#pragma unroll
        for (int u = 0; u < 8; ++u) { tot.x += v[u].x; tot.y += v[u].y; }
      }
      for (; c < c_hi; ++c) {
        const float2 v = *reinterpret_cast<const float2*>(p.partial + (c * stride + 2 * d) * p.D + c0);
        tot.x += v.x;
        tot.y += v.y;
      }
      s_part[warp][c0] = tot.x;
      s_part[warp][c0 + 1] = tot.y;
    }
    __syncthreads();
    if (warp == 0) {
      const int64_t node = d < ln ? heap_node(d, key, ln) : (int64_t)key + base_node - (p.N - 1);
      for (int c0 = lane * 2; c0 < p.D; c0 += 64) {
        float2 tot = *reinterpret_cast<const float2*>(p.partial + (chunk * stride + 2 * d + 1) * p.D + c0);
        for (int w = 0; w < kFixWarps; ++w) {
          tot.x += s_part[w][c0];
          tot.y += s_part[w][c0 + 1];
        }
        if (d < ln) {
          char* row = p.dk + ((int64_t)b * p.dkb + (int64_t)h * p.dkh + node * p.dks) *
                                 (p.dk_f32 ? 4 : (int64_t)sizeof(T));
          if (p.dk_f32) {
            *reinterpret_cast<float2*>(reinterpret_cast<float*>(row) + c0) = tot;
          } else {
            reinterpret_cast<T*>(row)[c0] = static_cast<T>(tot.x);
            reinterpret_cast<T*>(row)[c0 + 1] = static_cast<T>(tot.y);
          }
        } else if (p.dv_f32) {
          char* row = p.dv + ((int64_t)b * p.dvb + (int64_t)h * p.dvh + node * p.dvs) * 4;
          *reinterpret_cast<float2*>(reinterpret_cast<float*>(row) + c0) = tot;
        } else {
          char* row = p.dv + ((int64_t)b * p.dvb + (int64_t)h * p.dvh + node * p.dvs) * (int64_t)sizeof(T);
          reinterpret_cast<T*>(row)[c0] = static_cast<T>(tot.x);
          reinterpret_cast<T*>(row)[c0 + 1] = static_cast<T>(tot.y);
        }
      }
    }
    __syncthreads();
  }
}

// One warp per chunk (no block barriers: most chunks own only a few short-span cut nodes):
// the owner of a cut node finds the span with ballots and sums the span's partial rows in
// chunk order after its own, lanes over columns (float4), 16 rows in flight.
constexpr int kFixWarpsPerBlock = 4;

template <typename T>
__global__ void __launch_bounds__(kFixWarpsPerBlock * 32) bwd_fixup_warp_kernel(const BwdParams p, int64_t nchunks) {
  const int lane = threadIdx.x & 31;
  const int64_t chunk = (int64_t)blockIdx.x * kFixWarpsPerBlock + (threadIdx.x >> 5);
  if (chunk >= nchunks) return;  // whole warp
  const int ln = p.log_n;
  const int seg = (int)(chunk / p.chunks_per_seg);
  const int64_t cis = chunk - (int64_t)seg * p.chunks_per_seg;
  const int64_t seg_end = (int64_t)(seg + 1) * p.chunks_per_seg;
  const int b = seg / p.H, h = seg - (seg / p.H) * p.H;
  const int64_t stride = (int64_t)(ln + 1) * 2;
  const uint8_t* flg = p.flags;
  const int64_t base_node = ((int64_t)1 << ln) - 1;
  uint32_t key = 0;
  bool have_key = false;
  for (int d = 0; d <= ln; ++d) {
    if (flg[chunk * stride + 2 * d + 1] == 0) continue;  // not the owner of a cut node
    if (!have_key) {
      const int64_t i_last = min((cis + 1) * (int64_t)p.chunk, p.P) - 1;
      key = p.keys[p.sorted_buf][(int64_t)seg * p.P + i_last];
      have_key = true;
    }
    // the node spans chunk+1 .. c_end: chunks flagged "through" followed by one "ends here"
    int64_t c_end = chunk + 1;
    for (int64_t c0 = chunk + 1; c0 < seg_end; c0 += 32) {
      const int64_t c = c0 + lane;
      const bool ends = c < seg_end && flg[c * stride + 2 * d] != 2;
      const unsigned m = __ballot_sync(0xffffffffu, ends);
      if (m) {
        c_end = c0 + __ffs(m) - 1;
        break;
      }
    }
    const int64_t node = d < ln ? heap_node(d, key, ln) : (int64_t)key + base_node - (p.N - 1);
    for (int c4 = lane * 4; c4 < p.D; c4 += 128) {
      float4 tot = *reinterpret_cast<const float4*>(p.partial + (chunk * stride + 2 * d + 1) * p.D + c4);
      int64_t c = chunk + 1;
      for (; c + 16 <= c_end + 1; c += 16) {
        float4 v[16];
#pragma unroll
        for (int u = 0; u < 16; ++u)
          v[u] = *reinterpret_cast<const float4*>(p.partial + ((c + u) * stride + 2 * d) * p.D + c4);
#pragma unroll
        for (int u = 0; u < 16; ++u) { tot.x += v[u].x; tot.y += v[u].y; tot.z += v[u].z; tot.w += v[u].w; }
      }
      for (; c <= c_end; ++c) {
        const float4 v = *reinterpret_cast<const float4*>(p.partial + (c * stride + 2 * d) * p.D + c4);
        tot.x += v.x; tot.y += v.y; tot.z += v.z; tot.w += v.w;
      }
      const float tv[4] = {tot.x, tot.y, tot.z, tot.w};
      if (d < ln) {
        char* row = p.dk + ((int64_t)b * p.dkb + (int64_t)h * p.dkh + node * p.dks) *
                               (p.dk_f32 ? 4 : (int64_t)sizeof(T));
        if (p.dk_f32) *reinterpret_cast<float4*>(reinterpret_cast<float*>(row) + c4) = tot;
        else for (int e = 0; e < 4; ++e) reinterpret_cast<T*>(row)[c4 + e] = static_cast<T>(tv[e]);
      } else if (p.dv_f32) {
        char* row = p.dv + ((int64_t)b * p.dvb + (int64_t)h * p.dvh + node * p.dvs) * 4;
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(row) + c4) = tot;
      } else {
        char* row = p.dv + ((int64_t)b * p.dvb + (int64_t)h * p.dvh + node * p.dvs) * (int64_t)sizeof(T);
        for (int e = 0; e < 4; ++e) reinterpret_cast<T*>(row)[c4 + e] = static_cast<T>(tv[e]);
      }
    }
  }
}

}  // namespace ta
#include "ta_backward_mma.cuh"
namespace ta {

// ---------------------------------------------------------------------------------------
// typed launchers
// ---------------------------------------------------------------------------------------
template <typename T, int CPL>
void launch_query(const BwdParams& p, cudaStream_t st) {
  const int ltiles = (p.L + kBwdGroups - 1) / kBwdGroups;
  const size_t smem = (size_t)kBwdGroups * p.S * 4 +
                      (p.qtable_levels > 0 ? qtable_smem(p.qtable_levels, p.nchunks * 16, p.nchunks * 8)
                                           : (size_t)((1 << p.top_levels) - 1) * p.nchunks * 16);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(bwd_query_kernel<T, CPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  TA_PROFILE("bwd_query", st);
  bwd_query_kernel<T, CPL><<<ltiles * p.B * p.H, kBwdThreads, smem, st>>>(p);
}

template <typename T>
int run_query(const BwdParams& p, cudaStream_t st) {
  switch (pick_cpl(p.nchunks)) {
    case 1: launch_query<T, 1>(p, st); break;
    case 2: launch_query<T, 2>(p, st); break;
    case 3: launch_query<T, 3>(p, st); break;
    case 4: launch_query<T, 4>(p, st); break;
    case 6: launch_query<T, 6>(p, st); break;
    case 8: launch_query<T, 8>(p, st); break;
    default: return fail(TA_ERR_UNSUPPORTED, "head_dim too large");
  }
  return check_launch("backward query pass");
}

template <typename T, int EP>
void launch_node_el(const BwdParams& p, cudaStream_t st, unsigned grid) {
  TA_PROFILE("bwd_node", st);
  const int smem = kNodeWarps * node_warp_bytes(p.D * (int)sizeof(T), p.D, p.log_n + 1);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(bwd_node_kernel<T, EP>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  bwd_node_kernel<T, EP><<<grid, kNodeWarps * 32, smem, st>>>(p);
}

template <typename T>
int run_rest(BwdParams& p, cudaStream_t st, bool sorted = false) {
  int rc = sorted ? TA_OK : run_sort(p, st);
  if (rc) return rc;
  if constexpr (sizeof(T) == 2) {
    if (p.chunk == kChunkMma) {
      {
        TA_PROFILE("bwd_node", st);
        switch (p.D / 32) {
          case 1: launch_node_mma<T, 1>(p, st); break;
          case 2: launch_node_mma<T, 2>(p, st); break;
          case 3: launch_node_mma<T, 3>(p, st); break;
          case 4: launch_node_mma<T, 4>(p, st); break;
          default: launch_node_mma<T, 8>(p, st); break;
        }
      }
      if ((rc = check_launch("backward node pass"))) return rc;
      // the node pass cuts nodes only at range boundaries: the fix-up's chunks are the ranges
      int range_chunks, ranges_per_seg;
      node_mma_ranges(p, range_chunks, ranges_per_seg);
      BwdParams pf = p;
      pf.chunk = range_chunks * kChunkMma;
      pf.chunks_per_seg = ranges_per_seg;
      const int64_t nranges_total = (int64_t)p.B * p.H * ranges_per_seg;
      {
        TA_PROFILE("bwd_fixup", st);
        if (p.D % 4 == 0)
          bwd_fixup_warp_kernel<T><<<(unsigned)((nranges_total + kFixWarpsPerBlock - 1) / kFixWarpsPerBlock),
                                     kFixWarpsPerBlock * 32, 0, st>>>(pf, nranges_total);
        else
          bwd_fixup_kernel<T><<<(unsigned)nranges_total, kFixWarps * 32, 0, st>>>(pf);
      }
      return check_launch("backward fix-up");
    }
  }
  const int64_t nchunks_total = (int64_t)p.B * p.H * p.chunks_per_seg;
  const unsigned grid = (unsigned)((nchunks_total + kNodeWarps - 1) / kNodeWarps);
  const int ep = (p.D + 63) / 64;  // element pairs per lane
  switch (ep) {
    case 1: launch_node_el<T, 1>(p, st, grid); break;
    case 2: launch_node_el<T, 2>(p, st, grid); break;
    case 3: case 4: launch_node_el<T, 4>(p, st, grid); break;
    default: return fail(TA_ERR_UNSUPPORTED, "head_dim too large for the node pass");
  }
  if ((rc = check_launch("backward node pass"))) return rc;
  {
    TA_PROFILE("bwd_fixup", st);
    if (p.D % 4 == 0)
          bwd_fixup_warp_kernel<T><<<(unsigned)((nchunks_total + kFixWarpsPerBlock - 1) / kFixWarpsPerBlock),
                                     kFixWarpsPerBlock * 32, 0, st>>>(p, nchunks_total);
        else
          bwd_fixup_kernel<T><<<(unsigned)nchunks_total, kFixWarps * 32, 0, st>>>(p);
  }
  return check_launch("backward fix-up");
}

// the typed half of ta_backward: query pass, then sort + node pass + fix-up
// The sort records of every path from the forward's leaves alone: (path bits, path id within
// its head), the same values the query pass writes. One thread per path.
static __global__ void __launch_bounds__(256) sort_records_kernel(const BwdParams p) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // head-major path index
  const int64_t total = (int64_t)p.B * p.H * p.P;
  if (i >= total) return;
  const int64_t hb = i / p.P, pl = i - hb * p.P;
  const int64_t l = pl / p.S, s = pl - l * p.S;
  const int b = (int)(hb / p.H), h = (int)(hb - (hb / p.H) * p.H);
  const uint32_t K = (uint32_t)p.N - 1u, base_node = (1u << p.log_n) - 1u;
  p.keys[0][i] = (uint32_t)p.leaf[((l * p.B + b) * p.H + h) * p.S + s] + K - base_node;
  p.vals[0][i] = (uint32_t)pl;
}

// A side stream and two events for the calling host thread on the current device (created on
// first use; thread-local, so concurrent callers never share an event); false when `st` is on
// another device or a handle cannot be created (the caller then stays on one stream).
bool backward_fork_handles(cudaStream_t& side, cudaEvent_t& fork, cudaEvent_t& join,
                           cudaStream_t st);

template <typename T>
int run_backward_typed(BwdParams& p, cudaStream_t st) {
  // The sort of the paths by leaf needs only the forward's leaves, not the query pass: it runs
  // on a side stream beside the query pass, and the node pass waits for both.
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  const bool apart = !p.coef_mode && backward_fork_handles(side, fork, join, st);
  int rc;
  if (apart) {
    p.records_apart = 1;
    cudaEventRecord(fork, st);
    cudaStreamWaitEvent(side, fork, 0);
    {
      TA_PROFILE("sort_records", side);
      const int64_t total = (int64_t)p.B * p.H * p.P;
      sort_records_kernel<<<(unsigned)((total + 255) / 256), 256, 0, side>>>(p);
    }
    if ((rc = run_sort(p, side))) return rc;
    cudaEventRecord(join, side);
    if ((rc = run_query<T>(p, st))) return rc;
    cudaStreamWaitEvent(st, join, 0);
    return run_rest<T>(p, st, /*sorted=*/true);
  }
  if ((rc = run_query<T>(p, st))) return rc;
  return run_rest<T>(p, st);
}

}  // namespace ta
