// Tensor-core leaf-block attention of the generalised tree (bf16 / fp16 inputs), sm_100a.
//
// After the tree walk, a head's (query, path) pairs are sorted by leaf block, so the pairs
// of one block are contiguous and share that block's Lb keys and values: a dense product.
// One CTA per (batch*head, leaf block) keeps K_blk and V_blk in shared memory and walks its
// pairs in tiles (their query rows gathered into shared memory):
//   forward   S = Q_g K^T (scaled, causal rows masked), P = softmax_rows(S), O = P V;
//             each pair's w_s * o_s goes to a float32 per-path buffer, summed per query in
//             path order by a second kernel (deterministic, no atomics);
//   backward  S, P again; dP = w_s dO_q V^T; dS = P (dP - delta) with delta = dO_q . (w_s o_s);
//             dV += (w P)^T dO_q and dK += scale dS^T Q_g accumulate in registers over the
//             block's tiles in sorted order; dq of each pair = scale dS K goes to a per-path
//             buffer.
// All products run on mma.sync m16n8k16 (16-bit operands, float32 accumulation); P, w P and
// dS are rounded to the input's 16-bit type for their products, as FlashAttention does.
#pragma once

#include "ta_common.cuh"

namespace ta {

template <typename T> struct Mma;
template <> struct Mma<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float* c, const uint32_t* a, const uint32_t* b) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
  __device__ __forceinline__ static uint32_t pack(float x, float y) {
    __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static uint16_t half_bits(float x) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
  }
};
template <> struct Mma<__half> {
  __device__ __forceinline__ static void run(float* c, const uint32_t* a, const uint32_t* b) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
  __device__ __forceinline__ static uint32_t pack(float x, float y) {
    __half2 h = __floats2half2_rn(x, y);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static uint16_t half_bits(float x) {
    return __half_as_ushort(__float2half_rn(x));
  }
};

__device__ __forceinline__ void ldsm4(uint32_t* r, const void* p) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
__device__ __forceinline__ void ldsm4t(uint32_t* r, const void* p) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}

// Fragment loaders (element strides in 16-bit units, rows 16-byte aligned).
// A 16x16 from a row-major [m][k] tile.
__device__ __forceinline__ void frag_a(uint32_t* r, const uint16_t* base, int ld, int m0, int k0, int lane) {
  ldsm4(r, base + (m0 + (lane & 15)) * ld + k0 + (lane >> 4) * 8);
}
// A 16x16 (m = columns of the stored tile) from a stored [k][m] tile: the transpose.
__device__ __forceinline__ void frag_a_t(uint32_t* r, const uint16_t* base, int ld, int m0, int k0, int lane) {
  ldsm4t(r, base + (k0 + (lane >> 4) * 8 + (lane & 7)) * ld + m0 + ((lane >> 3) & 1) * 8);
}
// B for two n8 tiles (n0, n0 + 8), k16, from a stored [n][k] tile (k contiguous):
// r[0..1] = tile n0, r[2..3] = tile n0 + 8.
__device__ __forceinline__ void frag_b_nk(uint32_t* r, const uint16_t* base, int ld, int n0, int k0, int lane) {
  ldsm4(r, base + (n0 + (lane >> 4) * 8 + (lane & 7)) * ld + k0 + ((lane >> 3) & 1) * 8);
}
// B for two n8 tiles from a stored [k][n] tile (n contiguous).
__device__ __forceinline__ void frag_b_kn(uint32_t* r, const uint16_t* base, int ld, int n0, int k0, int lane) {
  ldsm4t(r, base + (k0 + ((lane >> 3) & 1) * 8 + (lane & 7)) * ld + n0 + (lane >> 4) * 8);
}

constexpr float kLog2e = 1.4426950408889634f;

// Keys of a leaf block a pair may attend: its first `visible_keys` keys (keys past the pair's
// causal boundary `bnd` are masked; INT64_MAX = no boundary).
template <int LB>
__device__ __forceinline__ int visible_keys(int64_t bnd, int64_t key0) {
  const int64_t v = bnd - key0 + 1;
  return v >= LB ? LB : (v < 0 ? 0 : (int)v);
}

struct BlkMmaParams {
  const char* q; const char* k; const char* v; const char* dout;
  int64_t qs, qb, qh, ks, kb, kh, vs, vb, vh, gs, gb, gh;
  const uint32_t* skeys; const uint32_t* svals;  // [B*H][P] sorted by leaf block
  const uint32_t* ranges;  // [B*H][nb + 1] first sorted pair of each leaf block (or null)
  const float* weights;    // [L][B][H][S] path weights
  void* path_out;          // [B*H][P][D] input dtype: w_s o_s (forward out, backward in)
  float* lse;              // [B*H][P]: base-2 log-sum-exp of each pair's scaled scores
  const float* delta;      // [B*H][P] dO_q . (w_s o_s) (backward)
  void* dq_path;           // [B*H][P][D] input dtype (backward)
  float* dk_attn;          // [B*H][N][D] (backward)
  const float* dz_rows;    // [B*H][P][DF] per-path summary coefficients (backward)
  float* dc_part;          // [B*H][nb][DF][D] per-block summary partials (backward)
  int32_t DF;              // levels * fanout (<= kDFMax)
  char* dv; int64_t dvs, dvb, dvh;
  int32_t B, H, L, N, S, nb, causal;
  int64_t P, row0, row_total;
  float scale;
  volatile int32_t* status;  // tensor-core wait status (0 = ok), mapped host memory
  uint64_t wait_ns;          // bound of one tensor-core mbarrier wait
};

template <int LB, int D>
struct BlkMmaGeom {
  static constexpr int LD = D + 8;      // padded row of q / k / v / dO tiles (elements)
  static constexpr int LDP = LB + 8;    // padded row of P / dS tiles
  static constexpr int NT_S = LB / 8;   // n8 tiles of a score row
  static constexpr int NT_D = D / 8;    // n8 tiles of an output row
};

template <int LB, int D>
__host__ __device__ constexpr size_t blk_mma_fwd_smem() {
  return (size_t)(2 * LB + 64) * (D + 8) * 2 + 64 * 16;
}

// ---------------------------------------------------------------------------------------
// forward: 4 warps, 64 pairs per tile (16 rows per warp)
// ---------------------------------------------------------------------------------------
template <typename T, int LB, int D>
__global__ void __launch_bounds__(128, LB * D > 8192 ? 2 : 4) blk_attn_fwd_mma_kernel(const BlkMmaParams p) {
  using G = BlkMmaGeom<LB, D>;
  extern __shared__ __align__(16) unsigned char smraw[];
  uint16_t* s_k = reinterpret_cast<uint16_t*>(smraw);
  uint16_t* s_v = s_k + LB * G::LD;
  uint16_t* s_q = s_v + LB * G::LD;
  int64_t* s_bnd = reinterpret_cast<int64_t*>(s_q + 64 * G::LD);  // [64] causal boundary per row
  __shared__ int64_t range[2];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bh = blockIdx.x / p.nb;
  const int j = blockIdx.x - bh * p.nb;
  const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const uint32_t* keys = p.skeys + (int64_t)bh * p.P;
  const uint32_t* vals = p.svals + (int64_t)bh * p.P;
  if (tid < 2) {
    const uint32_t target = (uint32_t)j + tid;
    int64_t lo = 0, hi = p.P;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if (keys[mid] < target) lo = mid + 1; else hi = mid;
    }
    range[tid] = lo;
  }
  // K and V of the block
  constexpr int CPR = D * 2 / 16;  // 16-byte chunks per row
  for (int i = tid; i < LB * CPR; i += blockDim.x) {
    const int r = i / CPR, c = i - r * CPR;
    const int64_t key = (int64_t)j * LB + r;
    cp_async16(s_k + r * G::LD + c * 8, p.k + (key * p.ks + (int64_t)b * p.kb + (int64_t)h * p.kh) * 2 + c * 16);
    cp_async16(s_v + r * G::LD + c * 8, p.v + (key * p.vs + (int64_t)b * p.vb + (int64_t)h * p.vh) * 2 + c * 16);
  }
  cp_async_commit();
  __syncthreads();
  const int64_t beg = range[0], end = range[1];
  for (int64_t t0 = beg; t0 < end; t0 += 64) {
    const int n = (int)min((int64_t)64, end - t0);
    __syncthreads();  // previous tile's readers are done with s_q
    for (int i = tid; i < 64 * CPR; i += blockDim.x) {
      const int r = i / CPR, c = i - r * CPR;
      uint16_t* dst = s_q + r * G::LD + c * 8;
      if (r < n) {
        const int64_t l = vals[t0 + r] / p.S;
        cp_async16(dst, p.q + (l * p.qs + (int64_t)b * p.qb + (int64_t)h * p.qh) * 2 + c * 16);
      } else {
        *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
      }
    }
    if (tid < 64) {
      const int64_t l = tid < n ? (int64_t)(vals[t0 + tid] / p.S) : 0;
      s_bnd[tid] = p.causal ? (p.row0 + l) + p.N - p.row_total : INT64_MAX;
    }
    cp_async_commit();
    cp_async_wait_0();
    __syncthreads();
    const int m0 = warp * 16;
    if (m0 >= n) continue;
    // S = Q K^T
    float sc[G::NT_S][4];
#pragma unroll
    for (int t = 0; t < G::NT_S; ++t) sc[t][0] = sc[t][1] = sc[t][2] = sc[t][3] = 0.0f;
#pragma unroll
    for (int k0 = 0; k0 < D; k0 += 16) {
      uint32_t a[4];
      frag_a(a, s_q, G::LD, m0, k0, lane);
#pragma unroll
      for (int t = 0; t < G::NT_S; t += 2) {
        uint32_t bb[4];
        frag_b_nk(bb, s_k, G::LD, t * 8, k0, lane);
        Mma<T>::run(sc[t], a, bb);
        Mma<T>::run(sc[t + 1], a, bb + 2);
      }
    }
    // masked softmax of rows g and g + 8 (quad lanes share a row)
    const int g = lane >> 2, tq = lane & 3;
    const int64_t key0 = (int64_t)j * LB;
    const int lim0 = visible_keys<LB>(s_bnd[m0 + g], key0), lim1 = visible_keys<LB>(s_bnd[m0 + g + 8], key0);
    const float sl2 = p.scale * kLog2e;  // scores in base 2: exp(scale s) = exp2(scale log2(e) s)
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int t = 0; t < G::NT_S; ++t) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int c = t * 8 + tq * 2 + e;
        sc[t][e] = c >= lim0 ? -INFINITY : sc[t][e] * sl2;
        sc[t][2 + e] = c >= lim1 ? -INFINITY : sc[t][2 + e] * sl2;
        mx0 = fmaxf(mx0, sc[t][e]);
        mx1 = fmaxf(mx1, sc[t][2 + e]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    float sum0 = 0.0f, sum1 = 0.0f;
#pragma unroll
    for (int t = 0; t < G::NT_S; ++t) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        sc[t][e] = exp2f(sc[t][e] - mx0);
        sc[t][2 + e] = exp2f(sc[t][2 + e] - mx1);
        sum0 += sc[t][e];
        sum1 += sc[t][2 + e];
      }
    }
    sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
    sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
    sum1 += __shfl_xor_sync(0xffffffffu, sum1, 1);
    sum1 += __shfl_xor_sync(0xffffffffu, sum1, 2);
    // O = P V, P as A fragments straight from the score registers
    float oc[G::NT_D][4];
#pragma unroll
    for (int t = 0; t < G::NT_D; ++t) oc[t][0] = oc[t][1] = oc[t][2] = oc[t][3] = 0.0f;
#pragma unroll
    for (int kc = 0; kc < LB / 16; ++kc) {
      uint32_t a[4];
      a[0] = Mma<T>::pack(sc[2 * kc][0], sc[2 * kc][1]);
      a[1] = Mma<T>::pack(sc[2 * kc][2], sc[2 * kc][3]);
      a[2] = Mma<T>::pack(sc[2 * kc + 1][0], sc[2 * kc + 1][1]);
      a[3] = Mma<T>::pack(sc[2 * kc + 1][2], sc[2 * kc + 1][3]);
#pragma unroll
      for (int t = 0; t < G::NT_D; t += 2) {
        uint32_t bb[4];
        frag_b_kn(bb, s_v, G::LD, t * 8, kc * 16, lane);
        Mma<T>::run(oc[t], a, bb);
        Mma<T>::run(oc[t + 1], a, bb + 2);
      }
    }
    // epilogue: w_s / rowsum, float32 per-path rows
    const int r0 = m0 + g, r1 = m0 + g + 8;
    if (r0 < n) {
      const int64_t path = vals[t0 + r0];
      const int64_t l = path / p.S, s = path - l * p.S;
      const float w = p.weights[(((int64_t)l * p.B + b) * p.H + h) * p.S + s] / sum0;
      T* dst = reinterpret_cast<T*>(p.path_out) + ((int64_t)bh * p.P + path) * D;
      if (tq == 0 && p.lse != nullptr) p.lse[(int64_t)bh * p.P + path] = mx0 + __log2f(sum0);
#pragma unroll
      for (int t = 0; t < G::NT_D; ++t)
        *reinterpret_cast<uint32_t*>(dst + t * 8 + tq * 2) = Mma<T>::pack(oc[t][0] * w, oc[t][1] * w);
    }
    if (r1 < n) {
      const int64_t path = vals[t0 + r1];
      const int64_t l = path / p.S, s = path - l * p.S;
      const float w = p.weights[(((int64_t)l * p.B + b) * p.H + h) * p.S + s] / sum1;
      T* dst = reinterpret_cast<T*>(p.path_out) + ((int64_t)bh * p.P + path) * D;
      if (tq == 0 && p.lse != nullptr) p.lse[(int64_t)bh * p.P + path] = mx1 + __log2f(sum1);
#pragma unroll
      for (int t = 0; t < G::NT_D; ++t)
        *reinterpret_cast<uint32_t*>(dst + t * 8 + tq * 2) = Mma<T>::pack(oc[t][2] * w, oc[t][3] * w);
    }
  }  cp_async_wait_0();  // a block without pairs never waited for its K / V copies
}

// ---------------------------------------------------------------------------------------
// backward: 8 warps, 128 pairs per tile. Phase 1 (warp w: pair rows [16w, 16w + 16)):
// S, P, dP, dS -> shared memory (w P and dS as 16-bit [pair][key]); phase 2: dq rows of the
// same pairs = dS K; phase 3 (warp w: key rows [16 (w % MT), +16) x its column slice):
// dV += (w P)^T dO, dK += dS^T Q over the tile's pairs.
// ---------------------------------------------------------------------------------------
constexpr int kDFMax = 32;  // levels * fanout handled by the tensor-core backward
constexpr int kZLd = kDFMax + 8;  // row stride (16-bit units) of the dz tiles

template <int LB, int D>
__host__ __device__ constexpr size_t blk_mma_bwd_smem() {
  return (size_t)(2 * LB + 2 * 128) * (D + 8) * 2   // k, v, q, dO
         + (size_t)2 * 128 * (LB + 8) * 2            // w P, dS
         + (size_t)128 * 16                           // boundary, delta, w
         + (size_t)2 * 128 * kZLd * 2;                // dz rows of the tile, 16-bit high / low
}

template <typename T> __device__ __forceinline__ float raw_to_float(uint16_t r);
template <> __device__ __forceinline__ float raw_to_float<__nv_bfloat16>(uint16_t r) {
  return __uint_as_float((uint32_t)r << 16);
}
template <> __device__ __forceinline__ float raw_to_float<__half>(uint16_t r) {
  return __half2float(__ushort_as_half(r));
}

template <typename T, int LB, int D>
__global__ void __launch_bounds__(256) blk_attn_bwd_mma_kernel(const BlkMmaParams p) {
  using G = BlkMmaGeom<LB, D>;
  constexpr int MT = LB / 16;          // key m16 tiles
  constexpr int SPLITS = 8 / MT;       // column slices per key tile
  constexpr int DW = D / SPLITS;       // columns per warp in phase 3
  constexpr int NT_W = DW / 8;
  static_assert(MT * SPLITS == 8 && DW % 16 == 0, "unsupported leaf block / head_dim");
  extern __shared__ __align__(16) unsigned char smraw[];
  uint16_t* s_k = reinterpret_cast<uint16_t*>(smraw);
  uint16_t* s_v = s_k + LB * G::LD;
  uint16_t* s_q = s_v + LB * G::LD;
  uint16_t* s_g = s_q + 128 * G::LD;
  uint16_t* s_wp = s_g + 128 * G::LD;
  uint16_t* s_ds = s_wp + 128 * G::LDP;
  int64_t* s_bnd = reinterpret_cast<int64_t*>(s_ds + 128 * G::LDP);
  float* s_delta = reinterpret_cast<float*>(s_bnd + 128);
  float* s_w = s_delta + 128;
  // dz rows of the tile as 16-bit high and low parts, [pair][DF row] (A^T of the summary
  // product dc += dz^T Q)
  uint16_t* s_zh = reinterpret_cast<uint16_t*>(s_w + 128);
  uint16_t* s_zl = s_zh + 128 * kZLd;
  __shared__ int64_t range[2];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bh = blockIdx.x / p.nb;
  const int j = blockIdx.x - bh * p.nb;
  const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const uint32_t* keys = p.skeys + (int64_t)bh * p.P;
  const uint32_t* vals = p.svals + (int64_t)bh * p.P;
  if (tid < 2) {
    const uint32_t target = (uint32_t)j + tid;
    int64_t lo = 0, hi = p.P;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if (keys[mid] < target) lo = mid + 1; else hi = mid;
    }
    range[tid] = lo;
  }
  constexpr int CPR = D * 2 / 16;
  for (int i = tid; i < LB * CPR; i += blockDim.x) {
    const int r = i / CPR, c = i - r * CPR;
    const int64_t key = (int64_t)j * LB + r;
    cp_async16(s_k + r * G::LD + c * 8, p.k + (key * p.ks + (int64_t)b * p.kb + (int64_t)h * p.kh) * 2 + c * 16);
    cp_async16(s_v + r * G::LD + c * 8, p.v + (key * p.vs + (int64_t)b * p.vb + (int64_t)h * p.vh) * 2 + c * 16);
  }
  cp_async_commit();
  const int DF = p.DF;
  const int zmt = (DF + 15) >> 4;  // m16 tiles of the summary product
  // summary product items (m16 tile, pair of n8 column tiles), at most two per warp; their
  // float32 accumulators live in registers across the block's pair tiles
  constexpr int NPAIR = D / 16;
  float acc_dc[2][2][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc_dc[i][t][e] = 0.0f;
  __syncthreads();
  const int64_t beg = range[0], end = range[1];
  const int g = lane >> 2, tq = lane & 3;
  const int km = (warp % MT) * 16;     // phase 3 key rows
  const int kc0 = (warp / MT) * DW;    // phase 3 columns
  float adv[NT_W][4], adk[NT_W][4];
#pragma unroll
  for (int t = 0; t < NT_W; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) adv[t][e] = adk[t][e] = 0.0f;
  const int64_t key0 = (int64_t)j * LB;
  __shared__ uint32_t s_path[128], s_lq[128];  // the tile's (query, path) pairs and queries
  const int zsh = zmt == 1 ? 4 : 5;  // log2 of the dz tile width (16 or 32 rows of DF)
  for (int64_t t0 = beg; t0 < end; t0 += 128) {
    const int n = (int)min((int64_t)128, end - t0);
    __syncthreads();
    if (tid < 128) {
      // per pair, once: its path, query, causal boundary, delta and weight
      int64_t bnd = INT64_MAX;
      float dl = 0.0f, w = 0.0f;
      uint32_t path = 0, l = 0;
      if (tid < n) {
        path = vals[t0 + tid];
        l = path / (uint32_t)p.S;
        const uint32_t s = path - l * (uint32_t)p.S;
        if (p.causal) bnd = (p.row0 + (int64_t)l) + p.N - p.row_total;
        dl = p.delta[(int64_t)bh * p.P + path];
        w = p.weights[(((int64_t)l * p.B + b) * p.H + h) * p.S + s];
      }
      s_path[tid] = path;
      s_lq[tid] = l;
      s_bnd[tid] = bnd;
      s_delta[tid] = dl;
      s_w[tid] = w;
    }
    __syncthreads();
    for (int i = tid; i < 128 * CPR; i += blockDim.x) {
      const int r = i / CPR, c = i - r * CPR;
      uint16_t* dq_ = s_q + r * G::LD + c * 8;
      uint16_t* dg_ = s_g + r * G::LD + c * 8;
      if (r < n) {
        const int64_t l = s_lq[r];
        cp_async16(dq_, p.q + (l * p.qs + (int64_t)b * p.qb + (int64_t)h * p.qh) * 2 + c * 16);
        cp_async16(dg_, p.dout + (l * p.gs + (int64_t)b * p.gb + (int64_t)h * p.gh) * 2 + c * 16);
      } else {
        *reinterpret_cast<uint4*>(dq_) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(dg_) = make_uint4(0, 0, 0, 0);
      }
    }
    for (int i = tid; i < (128 << zsh); i += blockDim.x) {
      const int r = i >> zsh, c = i & ((1 << zsh) - 1);
      const float z = (r < n && c < DF) ? p.dz_rows[((int64_t)bh * p.P + s_path[r]) * DF + c] : 0.0f;
      const uint16_t hi = Mma<T>::half_bits(z);
      s_zh[r * kZLd + c] = hi;
      s_zl[r * kZLd + c] = Mma<T>::half_bits(z - raw_to_float<T>(hi));
    }
    cp_async_commit();
    cp_async_wait_0();
    __syncthreads();
    const int m0 = warp * 16;
    if (m0 < n) {
      // phase 1: S = Q K^T, P; dP = dO V^T
      float sc[G::NT_S][4], dp[G::NT_S][4];
#pragma unroll
      for (int t = 0; t < G::NT_S; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[t][e] = dp[t][e] = 0.0f;
#pragma unroll
      for (int k0 = 0; k0 < D; k0 += 16) {
        uint32_t a[4], ag[4];
        frag_a(a, s_q, G::LD, m0, k0, lane);
        frag_a(ag, s_g, G::LD, m0, k0, lane);
#pragma unroll
        for (int t = 0; t < G::NT_S; t += 2) {
          uint32_t bb[4];
          frag_b_nk(bb, s_k, G::LD, t * 8, k0, lane);
          Mma<T>::run(sc[t], a, bb);
          Mma<T>::run(sc[t + 1], a, bb + 2);
          frag_b_nk(bb, s_v, G::LD, t * 8, k0, lane);
          Mma<T>::run(dp[t], ag, bb);
          Mma<T>::run(dp[t + 1], ag, bb + 2);
        }
      }
      const int r0 = m0 + g, r1 = m0 + g + 8;
      const int lim0 = visible_keys<LB>(s_bnd[r0], key0), lim1 = visible_keys<LB>(s_bnd[r1], key0);
      const float sl2 = p.scale * kLog2e;
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int t = 0; t < G::NT_S; ++t)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int c = t * 8 + tq * 2 + e;
          sc[t][e] = c >= lim0 ? -INFINITY : sc[t][e] * sl2;
          sc[t][2 + e] = c >= lim1 ? -INFINITY : sc[t][2 + e] * sl2;
          mx0 = fmaxf(mx0, sc[t][e]);
          mx1 = fmaxf(mx1, sc[t][2 + e]);
        }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      float sum0 = 0.0f, sum1 = 0.0f;
#pragma unroll
      for (int t = 0; t < G::NT_S; ++t)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          sc[t][e] = r0 < n ? exp2f(sc[t][e] - mx0) : 0.0f;
          sc[t][2 + e] = r1 < n ? exp2f(sc[t][2 + e] - mx1) : 0.0f;
          sum0 += sc[t][e];
          sum1 += sc[t][2 + e];
        }
      sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
      sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
      sum1 += __shfl_xor_sync(0xffffffffu, sum1, 1);
      sum1 += __shfl_xor_sync(0xffffffffu, sum1, 2);
      const float inv0 = sum0 > 0.0f ? 1.0f / sum0 : 0.0f, inv1 = sum1 > 0.0f ? 1.0f / sum1 : 0.0f;
      const float w0 = s_w[r0], w1 = s_w[r1], d0 = s_delta[r0], d1 = s_delta[r1];
#pragma unroll
      for (int t = 0; t < G::NT_S; ++t) {
        const float p0 = sc[t][0] * inv0, p1 = sc[t][1] * inv0;
        const float p2 = sc[t][2] * inv1, p3 = sc[t][3] * inv1;
        // dS = P (w dP' - delta), dP' = dO_q . v_k
        const float s0 = p0 * (w0 * dp[t][0] - d0), s1 = p1 * (w0 * dp[t][1] - d0);
        const float s2 = p2 * (w1 * dp[t][2] - d1), s3 = p3 * (w1 * dp[t][3] - d1);
        const int c = t * 8 + tq * 2;
        *reinterpret_cast<uint32_t*>(s_wp + r0 * G::LDP + c) = Mma<T>::pack(w0 * p0, w0 * p1);
        *reinterpret_cast<uint32_t*>(s_wp + r1 * G::LDP + c) = Mma<T>::pack(w1 * p2, w1 * p3);
        *reinterpret_cast<uint32_t*>(s_ds + r0 * G::LDP + c) = Mma<T>::pack(s0, s1);
        *reinterpret_cast<uint32_t*>(s_ds + r1 * G::LDP + c) = Mma<T>::pack(s2, s3);
      }
      __syncwarp();
      // phase 2: dq rows = scale dS K
      float dq[G::NT_D][4];
#pragma unroll
      for (int t = 0; t < G::NT_D; ++t) dq[t][0] = dq[t][1] = dq[t][2] = dq[t][3] = 0.0f;
#pragma unroll
      for (int kc = 0; kc < LB; kc += 16) {
        uint32_t a[4];
        frag_a(a, s_ds, G::LDP, m0, kc, lane);
#pragma unroll
        for (int t = 0; t < G::NT_D; t += 2) {
          uint32_t bb[4];
          frag_b_kn(bb, s_k, G::LD, t * 8, kc, lane);
          Mma<T>::run(dq[t], a, bb);
          Mma<T>::run(dq[t + 1], a, bb + 2);
        }
      }
      if (r0 < n) {
        T* dst = reinterpret_cast<T*>(p.dq_path) + ((int64_t)bh * p.P + s_path[r0]) * D;
#pragma unroll
        for (int t = 0; t < G::NT_D; ++t)
          *reinterpret_cast<uint32_t*>(dst + t * 8 + tq * 2) = Mma<T>::pack(dq[t][0] * p.scale, dq[t][1] * p.scale);
      }
      if (r1 < n) {
        T* dst = reinterpret_cast<T*>(p.dq_path) + ((int64_t)bh * p.P + s_path[r1]) * D;
#pragma unroll
        for (int t = 0; t < G::NT_D; ++t)
          *reinterpret_cast<uint32_t*>(dst + t * 8 + tq * 2) = Mma<T>::pack(dq[t][2] * p.scale, dq[t][3] * p.scale);
      }
    } else {
      // rows of an absent warp tile: zero so phase 3 may read the whole tile
      for (int i = lane; i < 16 * LB / 2; i += 32) {
        const int r = m0 + i / (LB / 2), c = (i % (LB / 2)) * 2;
        *reinterpret_cast<uint32_t*>(s_wp + r * G::LDP + c) = 0u;
        *reinterpret_cast<uint32_t*>(s_ds + r * G::LDP + c) = 0u;
      }
    }
    __syncthreads();
    // summary partials dc[row][c] += sum over the tile's pairs of dz[pair][row] q[pair][c], as
    // tensor-core products of dz^T (high and low 16-bit parts) with the tile's q rows
    const int kend = (n + 15) & ~15;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int item = warp + 8 * i;
      if (item < zmt * NPAIR) {
        const int zm = (item / NPAIR) * 16, zn = (item % NPAIR) * 16;
        for (int kc = 0; kc < kend; kc += 16) {
          uint32_t ah[4], al[4], bb[4];
          frag_a_t(ah, s_zh, kZLd, zm, kc, lane);
          frag_a_t(al, s_zl, kZLd, zm, kc, lane);
          frag_b_kn(bb, s_q, G::LD, zn, kc, lane);
          Mma<T>::run(acc_dc[i][0], ah, bb);
          Mma<T>::run(acc_dc[i][0], al, bb);
          Mma<T>::run(acc_dc[i][1], ah, bb + 2);
          Mma<T>::run(acc_dc[i][1], al, bb + 2);
        }
      }
    }
    // phase 3: dV += (wP)^T dO, dK += dS^T Q over the tile's (up to) 128 pairs
    for (int kc = 0; kc < kend; kc += 16) {
      uint32_t a[4], ad[4];
      frag_a_t(a, s_wp, G::LDP, km, kc, lane);
      frag_a_t(ad, s_ds, G::LDP, km, kc, lane);
#pragma unroll
      for (int t = 0; t < NT_W; t += 2) {
        uint32_t bb[4];
        frag_b_kn(bb, s_g, G::LD, kc0 + t * 8, kc, lane);
        Mma<T>::run(adv[t], a, bb);
        Mma<T>::run(adv[t + 1], a, bb + 2);
        frag_b_kn(bb, s_q, G::LD, kc0 + t * 8, kc, lane);
        Mma<T>::run(adk[t], ad, bb);
        Mma<T>::run(adk[t + 1], ad, bb + 2);
      }
    }
  }
  cp_async_wait_0();  // a block without pairs never waited for its K / V copies
  {
    float* dcp = p.dc_part + ((int64_t)bh * p.nb + j) * DF * D;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int item = warp + 8 * i;
      if (item < zmt * NPAIR) {
        const int zm = (item / NPAIR) * 16, zn = (item % NPAIR) * 16;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int c = zn + t * 8 + tq * 2;
          if (zm + g < DF)
            *reinterpret_cast<float2*>(dcp + (zm + g) * D + c) = make_float2(acc_dc[i][t][0], acc_dc[i][t][1]);
          if (zm + g + 8 < DF)
            *reinterpret_cast<float2*>(dcp + (zm + g + 8) * D + c) = make_float2(acc_dc[i][t][2], acc_dc[i][t][3]);
        }
      }
    }
  }
  // dV (input dtype) and dK of the attention part (float32, the per-key pass adds the
  // summary gradients)
  const int kr0 = km + g, kr1 = km + g + 8;
#pragma unroll
  for (int t = 0; t < NT_W; ++t) {
    const int c = kc0 + t * 8 + tq * 2;
    const int64_t key_a = key0 + kr0, key_b = key0 + kr1;
    T* va = reinterpret_cast<T*>(p.dv) + key_a * p.dvs + (int64_t)b * p.dvb + (int64_t)h * p.dvh + c;
    T* vb = reinterpret_cast<T*>(p.dv) + key_b * p.dvs + (int64_t)b * p.dvb + (int64_t)h * p.dvh + c;
    *reinterpret_cast<uint32_t*>(va) = Mma<T>::pack(adv[t][0], adv[t][1]);
    *reinterpret_cast<uint32_t*>(vb) = Mma<T>::pack(adv[t][2], adv[t][3]);
    float* ka = p.dk_attn + ((int64_t)bh * p.N + key_a) * D + c;
    float* kb = p.dk_attn + ((int64_t)bh * p.N + key_b) * D + c;
    *reinterpret_cast<float2*>(ka) = make_float2(adk[t][0] * p.scale, adk[t][1] * p.scale);
    *reinterpret_cast<float2*>(kb) = make_float2(adk[t][2] * p.scale, adk[t][3] * p.scale);
  }
}

}  // namespace ta
