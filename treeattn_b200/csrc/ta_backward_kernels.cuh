// Fused deterministic backward of stochastic tree attention, sm_100a.
//
// Math (reference: _autograd.py:707-860, accumulate_qk_non_causal_all_depths_prepared.cu,
// scatter_weighted_grad_v.cu):
//   g_s   = dO . v[leaf_s]
//   dlp_s = w_s (g_s - sum_t w_t g_t)
//   gl_sd = sgn sigmoid(-sgn s_sd) dlp_s      (s_sd = clamp(q . k[node_sd]); sgn = +1 left)
//   dq    = sum_s sum_d gl_sd k[node_sd]
//   dk[n] = sum_{(s,d) through n} gl_sd q
//   dv[l] = sum_{s ending at l} w_s dO
//
// The reference scatters dK/dV with float atomics (order-dependent results). Here the
// scatter becomes a gather over paths sorted by leaf, so every node's sum has a fixed
// order and the result is bitwise repeatable:
//   1. query pass (one 4-lane group per query): g, dlp, per-depth gl (stored), dq (written);
//      emits (path bits, path id) records in head-major path order.
//   2. stable LSD radix sort of the records of each head by path bits (8-bit digits).
//   3. node pass: each warp owns a chunk of consecutive sorted paths. Paths through a node
//      are contiguous in this order, so the warp keeps one accumulator per depth in
//      registers and writes a node's total when the node closes. Nodes cut by a chunk
//      boundary leave a partial per side; nodes no path reaches are written as zeros.
//   4. fix-up: the chunk where a cut node starts adds the partials of the following chunks
//      in chunk order and writes the node.

#pragma once
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
constexpr int kNodeWarps = 8;

struct BwdParams {
  const char* q; const char* k; const char* v; const char* dout;
  char* dq; char* dk; char* dv;
  int64_t qs, qb, qh, ks, kb, kh, vs, vb, vh, gs, gb, gh;
  int64_t dqs, dqb, dqh, dks, dkb, dkh, dvs, dvb, dvh;
  const int32_t* leaf;
  const float* weights;
  float* gl;           // [HB][P][log_n]
  uint32_t* keys[2];   // [HB][P]
  uint32_t* vals[2];
  uint32_t* hist;      // [HB][256][tiles_per_seg]
  float* partial;      // [chunks][log_n + 1][2][D]
  uint8_t* flags;      // [chunks][log_n + 1][2]: head kind (0 none, 1 ends here, 2 through), tail
  int32_t B, L, H, S, N, D, log_n, nchunks;
  int32_t dk_f32;      // dk written as float32 (else input dtype)
  int64_t P;           // paths per head = L * S
  int32_t tiles_per_seg, chunks_per_seg;
  int32_t sorted_buf;  // which keys/vals buffer holds the sorted records
  float max_logit;
};

// radix-sort kernels (ta_backward.cu)
__global__ void sort_hist_kernel(const BwdParams p, int src, int shift);
__global__ void sort_scan_kernel(const BwdParams p);
__global__ void sort_scatter_kernel(const BwdParams p, int src, int shift);
int run_sort(BwdParams& p, cudaStream_t st);

// ---------------------------------------------------------------------------------------
// 1. query pass
// ---------------------------------------------------------------------------------------
template <typename T, int CPL>
__global__ void __launch_bounds__(kBwdThreads) bwd_query_kernel(const BwdParams p) {
  using E = Elem<T>;
  constexpr int EPC = E::EPC;
  constexpr int NE = CPL * EPC;
  constexpr int ILP = 2;
  extern __shared__ float smem[];

  const int ltiles = (p.L + kBwdGroups - 1) / kBwdGroups;
  const int bh = blockIdx.x / ltiles;
  const int lt = blockIdx.x - bh * ltiles;
  const int b = bh / p.H;
  const int h = bh - b * p.H;
  const int g = threadIdx.x >> 2;
  const int t4 = threadIdx.x & 3;
  const int l = lt * kBwdGroups + g;
  if (l >= p.L) return;
  const unsigned gmask = 0xFu << (threadIdx.x & 28);
  float* s_dlp = smem + g * p.S;

  const int64_t K = (int64_t)p.N - 1;
  const int64_t base_node = ((int64_t)1 << p.log_n) - 1;
  const int64_t j0 = (((int64_t)l * p.B + b) * p.H + h) * p.S;
  const int64_t hb = (int64_t)b * p.H + h;
  const int64_t path0 = hb * p.P + (int64_t)l * p.S;  // head-major path index of sample 0

  float qf[NE], acc[NE];
  {
    const char* qrow = p.q + ((int64_t)l * p.qs + (int64_t)b * p.qb + (int64_t)h * p.qh) * sizeof(T);
    const char* grow = p.dout + ((int64_t)l * p.gs + (int64_t)b * p.gb + (int64_t)h * p.gh) * sizeof(T);
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int c = i * 4 + t4;
      if (c < p.nchunks) {
        E::unpack(ldg16(qrow + c * 16), qf + i * EPC);
        E::unpack(ldg16(grow + c * 16), acc + i * EPC);  // dO, reused as dq accumulator later
      } else {
#pragma unroll
        for (int e = 0; e < EPC; ++e) { qf[i * EPC + e] = 0.0f; acc[i * EPC + e] = 0.0f; }
      }
    }
  }
  const char* vbase = p.v + ((int64_t)b * p.vb + (int64_t)h * p.vh) * sizeof(T);
  const char* kbase = p.k + ((int64_t)b * p.kb + (int64_t)h * p.kh) * sizeof(T);

  // g_s = dO . v[leaf_s]
  for (int s = 0; s < p.S; ++s) {
    int64_t lf = p.leaf[j0 + s];
    lf = lf < 0 ? 0 : (lf >= p.N ? p.N - 1 : lf);
    const char* vrow = vbase + lf * p.vs * (int64_t)sizeof(T);
    float d = 0.0f;
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int c = i * 4 + t4;
      if (c < p.nchunks) {
        float vf[EPC];
        E::unpack(ldg16(vrow + c * 16), vf);
#pragma unroll
        for (int e = 0; e < EPC; ++e) d = fmaf(acc[i * EPC + e], vf[e], d);
      }
    }
    d += __shfl_xor_sync(gmask, d, 1, 4);
    d += __shfl_xor_sync(gmask, d, 2, 4);
    if (t4 == 0) s_dlp[s] = d;
  }
  __syncwarp(gmask);
  // dlp_s = w_s (g_s - sum_t w_t g_t)
  float wg = 0.0f;
  for (int s = 0; s < p.S; ++s) wg = fmaf(p.weights[j0 + s], s_dlp[s], wg);
  __syncwarp(gmask);
  for (int s = t4; s < p.S; s += 4) {
    const float w = p.weights[j0 + s];
    s_dlp[s] = w * (s_dlp[s] - wg);
  }
  __syncwarp(gmask);

#pragma unroll
  for (int e = 0; e < NE; ++e) acc[e] = 0.0f;
  const int64_t kstride = p.ks * (int64_t)sizeof(T);

  for (int s0 = 0; s0 < p.S; s0 += ILP) {
    const int ns = min(ILP, p.S - s0);
    uint32_t bits[ILP];
    float dlp[ILP];
#pragma unroll
    for (int t = 0; t < ILP; ++t) {
      const int s = s0 + (t < ns ? t : 0);
      bits[t] = (uint32_t)((int64_t)p.leaf[j0 + s] + K - base_node);
      dlp[t] = t < ns ? s_dlp[s] : 0.0f;
    }
    if (t4 < ns) {  // sort record of path s0 + t4: (path bits, path id within its head)
      const int s = s0 + t4;
      uint32_t bt = bits[0];
#pragma unroll
      for (int t = 1; t < ILP; ++t) bt = t == t4 ? bits[t] : bt;
      p.keys[0][path0 + s] = bt;
      p.vals[0][path0 + s] = (uint32_t)((int64_t)l * p.S + s);
    }
    for (int depth = 0; depth < p.log_n; ++depth) {
      uint4 raw[ILP][CPL];
      float dot[ILP];
#pragma unroll
      for (int t = 0; t < ILP; ++t) {
        const int64_t node = heap_node(depth, bits[t], p.log_n);
        const char* krow = kbase + node * kstride;
        dot[t] = 0.0f;
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
          const int c = i * 4 + t4;
          raw[t][i] = (c < p.nchunks && t < ns) ? ldg16(krow + c * 16) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
          float kf[EPC];
          E::unpack(raw[t][i], kf);
#pragma unroll
          for (int e = 0; e < EPC; ++e) dot[t] = fmaf(qf[i * EPC + e], kf[e], dot[t]);
        }
      }
#pragma unroll
      for (int t = 0; t < ILP; ++t) {
        dot[t] += __shfl_xor_sync(gmask, dot[t], 1, 4);
        dot[t] += __shfl_xor_sync(gmask, dot[t], 2, 4);
      }
      float gl[ILP];
#pragma unroll
      for (int t = 0; t < ILP; ++t) {
        const float x = clamp_logit(dot[t], p.max_logit);
        const int bit = (bits[t] >> (p.log_n - 1 - depth)) & 1;
        const float sgn = bit ? -1.0f : 1.0f;
        gl[t] = sgn * dlp[t] / (1.0f + expf(sgn * x));
        if (t == t4 && t < ns) p.gl[(path0 + s0 + t) * p.log_n + depth] = gl[t];
      }
#pragma unroll
      for (int t = 0; t < ILP; ++t) {
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
          float kf[EPC];
          E::unpack(raw[t][i], kf);
#pragma unroll
          for (int e = 0; e < EPC; ++e) acc[i * EPC + e] = fmaf(gl[t], kf[e], acc[i * EPC + e]);
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
template <int EL>
struct LaneRow {  // EL consecutive row elements per lane, lanes cover the row
  template <typename T>
  __device__ __forceinline__ static void load(const char* row, int lane, int D, float* f) {
#pragma unroll
    for (int e = 0; e < EL; ++e) {
      const int c = lane * EL + e;
      f[e] = c < D ? static_cast<float>(reinterpret_cast<const T*>(row)[c]) : 0.0f;
    }
  }
};

template <typename T>
__device__ __forceinline__ void store_row_elems(char* row, int lane, int EL, int D, const float* f,
                                                bool f32) {
  for (int e = 0; e < EL; ++e) {
    const int c = lane * EL + e;
    if (c < D) {
      if (f32) reinterpret_cast<float*>(row)[c] = f[e];
      else reinterpret_cast<T*>(row)[c] = static_cast<T>(f[e]);
    }
  }
}

template <typename T, int EL, int MAXD>
__global__ void __launch_bounds__(kNodeWarps * 32) bwd_node_kernel(const BwdParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t chunk = (int64_t)blockIdx.x * kNodeWarps + (threadIdx.x >> 5);
  const int64_t nchunks_total = (int64_t)p.B * p.H * p.chunks_per_seg;
  if (chunk >= nchunks_total) return;
  const int seg = (int)(chunk / p.chunks_per_seg);
  const int cis = (int)(chunk - (int64_t)seg * p.chunks_per_seg);
  const int b = seg / p.H, h = seg - (seg / p.H) * p.H;
  const int ln = p.log_n;
  const int64_t i0 = (int64_t)cis * kChunk;
  const int64_t i1 = min(i0 + kChunk, p.P);
  const uint32_t* keys = p.keys[p.sorted_buf] + (int64_t)seg * p.P;
  const uint32_t* vals = p.vals[p.sorted_buf] + (int64_t)seg * p.P;

  const int64_t base_node = ((int64_t)1 << ln) - 1;
  const int64_t K = (int64_t)p.N - 1;
  char* dkb = p.dk + ((int64_t)b * p.dkb + (int64_t)h * p.dkh) * (p.dk_f32 ? 4 : (int64_t)sizeof(T));
  const int64_t dk_row = p.dks * (p.dk_f32 ? 4 : (int64_t)sizeof(T));
  char* dvb = p.dv + ((int64_t)b * p.dvb + (int64_t)h * p.dvh) * (int64_t)sizeof(T);
  const int64_t dv_row = p.dvs * (int64_t)sizeof(T);
  float* part = p.partial + chunk * (int64_t)(ln + 1) * 2 * p.D;
  uint8_t* flg = p.flags + chunk * (int64_t)(ln + 1) * 2;
  const float zeros[EL] = {};

  // depth levels d in [0, ln) are internal nodes, d == ln is the leaf (dv)
  auto node_of = [&](int d, uint32_t key) -> int64_t {
    return d < ln ? heap_node(d, key, ln) : (int64_t)key + base_node - K;
  };
  auto write_node = [&](int d, int64_t node, const float* f) {
    if (d < ln) store_row_elems<T>(dkb + node * dk_row, lane, EL, p.D, f, p.dk_f32);
    else store_row_elems<T>(dvb + node * dv_row, lane, EL, p.D, f, false);
  };
  // number of depths (of ln + 1) whose node two keys share
  auto shared_depths = [&](uint32_t a, uint32_t c) -> int {
    const uint32_t x = a ^ c;
    return x == 0 ? ln + 1 : ln - (32 - __clz(x)) + 1;
  };
  // zero every node strictly between key a and key c (a < c) at depths >= d0
  auto zero_gap = [&](uint32_t a, uint32_t c, int d0, bool incl_a, bool incl_c) {
    for (int d = d0; d <= ln; ++d) {
      const int sh = ln - d;
      int64_t lo = (int64_t)(a >> sh) + (incl_a ? 0 : 1);
      int64_t hi = (int64_t)(c >> sh) - (incl_c ? 0 : 1);
      for (int64_t pf = lo; pf <= hi; ++pf) {
        const int64_t node = d < ln ? ((int64_t)1 << d) - 1 + pf : pf + base_node - K;
        write_node(d, node, zeros);
      }
    }
  };

  float acc[MAXD + 1][EL];
#pragma unroll
  for (int d = 0; d <= MAXD; ++d)
#pragma unroll
    for (int e = 0; e < EL; ++e) acc[d][e] = 0.0f;

  uint32_t first = keys[i0];
  uint32_t open_before = 0;  // depths whose current node started before this chunk
  if (i0 > 0) {
    const int sd = shared_depths(keys[i0 - 1], first);
    open_before = sd >= 32 ? 0xffffffffu : ((1u << sd) - 1u);
  } else {
    // nodes left of the segment's first path are unreached
    const uint32_t lo_key = 0;
    if (first > 0) zero_gap(lo_key, first, 0, true, false);
  }
  for (int d = 0; d <= ln; ++d) {
    flg[2 * d] = 0;
    flg[2 * d + 1] = 0;
  }

  uint32_t prev = first;
  for (int64_t i = i0; i < i1; ++i) {
    const uint32_t key = keys[i];
    const uint32_t pl = vals[i];
    if (i > i0 && key != prev) {
      const int sd = shared_depths(prev, key);
      // close nodes at depths >= sd
#pragma unroll
      for (int d = 0; d <= MAXD; ++d) {
        if (d >= sd && d <= ln) {
          const int64_t node = node_of(d, prev);
          if ((open_before >> d) & 1u) {  // started in an earlier chunk: head partial
            float* dst = part + (int64_t)(2 * d) * p.D;
            for (int e = 0; e < EL; ++e)
              if (lane * EL + e < p.D) dst[lane * EL + e] = acc[d][e];
            flg[2 * d] = 1;
          } else {
            write_node(d, node, acc[d]);
          }
#pragma unroll
          for (int e = 0; e < EL; ++e) acc[d][e] = 0.0f;
        }
      }
      open_before &= (sd >= 32 ? 0xffffffffu : ((1u << sd) - 1u));
      zero_gap(prev, key, sd, false, false);
    }
    prev = key;
    // accumulate this path
    const int l = (int)(pl / (uint32_t)p.S);
    const int s = (int)(pl - (uint32_t)l * (uint32_t)p.S);
    const float w = p.weights[(((int64_t)l * p.B + b) * p.H + h) * p.S + s];
    const float glv = lane < ln ? p.gl[((int64_t)seg * p.P + pl) * ln + lane] : 0.0f;
    float qf[EL], of[EL];
    LaneRow<EL>::template load<T>(p.q + ((int64_t)l * p.qs + (int64_t)b * p.qb + (int64_t)h * p.qh) * sizeof(T), lane, p.D, qf);
    LaneRow<EL>::template load<T>(p.dout + ((int64_t)l * p.gs + (int64_t)b * p.gb + (int64_t)h * p.gh) * sizeof(T), lane, p.D, of);
#pragma unroll
    for (int d = 0; d < MAXD; ++d) {
      const float gd = __shfl_sync(0xffffffffu, glv, d & 31);
      if (d < ln) {
#pragma unroll
        for (int e = 0; e < EL; ++e) acc[d][e] = fmaf(gd, qf[e], acc[d][e]);
      }
    }
    // leaf accumulator lives at index ln; MAXD >= ln so index it statically
#pragma unroll
    for (int d = 0; d <= MAXD; ++d) {
      if (d == ln) {
#pragma unroll
        for (int e = 0; e < EL; ++e) acc[d][e] = fmaf(w, of[e], acc[d][e]);
      }
    }
  }

  // chunk end: close or hand over every open node
  const bool has_next = i1 < p.P;
  const uint32_t nxt = has_next ? keys[i1] : 0u;
  const int sd_next = has_next ? shared_depths(prev, nxt) : 0;
#pragma unroll
  for (int d = 0; d <= MAXD; ++d) {
    if (d <= ln) {
      const bool cont = d < sd_next;  // node continues into the next chunk
      const bool before = (open_before >> d) & 1u;
      if (cont) {
        float* dst = part + (int64_t)(2 * d + (before ? 0 : 1)) * p.D;
        for (int e = 0; e < EL; ++e)
          if (lane * EL + e < p.D) dst[lane * EL + e] = acc[d][e];
        if (before) flg[2 * d] = 2;      // passes through this chunk
        else flg[2 * d + 1] = 1;         // starts here: this chunk owns the fix-up
      } else if (before) {
        float* dst = part + (int64_t)(2 * d) * p.D;
        for (int e = 0; e < EL; ++e)
          if (lane * EL + e < p.D) dst[lane * EL + e] = acc[d][e];
        flg[2 * d] = 1;
      } else {
        write_node(d, node_of(d, prev), acc[d]);
      }
    }
  }
  if (has_next) {
    zero_gap(prev, nxt, sd_next, false, false);
  } else {
    // nodes right of the segment's last path are unreached
    const uint32_t hi_key = (uint32_t)(((uint64_t)1 << ln) - 1);
    if (prev < hi_key) zero_gap(prev, hi_key, 0, false, true);
  }
}

// ---------------------------------------------------------------------------------------
// 4. fix-up of nodes cut by chunk boundaries
// ---------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) bwd_fixup_kernel(const BwdParams p) {
  const int lane = threadIdx.x & 31;
  const int ln = p.log_n;
  const int64_t item = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int64_t nchunks_total = (int64_t)p.B * p.H * p.chunks_per_seg;
  if (item >= nchunks_total * (ln + 1)) return;
  const int64_t chunk = item / (ln + 1);
  const int d = (int)(item - chunk * (ln + 1));
  const uint8_t* flg = p.flags;
  const int64_t stride = (int64_t)(ln + 1) * 2;
  if (flg[chunk * stride + 2 * d + 1] == 0) return;  // not the owner of a cut node
  const int seg = (int)(chunk / p.chunks_per_seg);
  const int b = seg / p.H, h = seg - (seg / p.H) * p.H;
  const int64_t cis = chunk - (int64_t)seg * p.chunks_per_seg;
  const int64_t i_last = min((cis + 1) * (int64_t)kChunk, p.P) - 1;
  const uint32_t key = p.keys[p.sorted_buf][(int64_t)seg * p.P + i_last];
  const int64_t base_node = ((int64_t)1 << ln) - 1;
  const int64_t node = d < ln ? heap_node(d, key, ln) : (int64_t)key + base_node - (p.N - 1);
  for (int c0 = lane; c0 < p.D; c0 += 32) {
    float tot = p.partial[(chunk * (ln + 1) * 2 + 2 * d + 1) * p.D + c0];
    int64_t c = chunk + 1;
    while (true) {
      tot += p.partial[(c * (ln + 1) * 2 + 2 * d) * p.D + c0];
      if (flg[c * stride + 2 * d] != 2) break;
      ++c;
    }
    if (d < ln) {
      char* row = p.dk + ((int64_t)b * p.dkb + (int64_t)h * p.dkh + node * p.dks) *
                             (p.dk_f32 ? 4 : (int64_t)sizeof(T));
      if (p.dk_f32) reinterpret_cast<float*>(row)[c0] = tot;
      else reinterpret_cast<T*>(row)[c0] = static_cast<T>(tot);
    } else {
      char* row = p.dv + ((int64_t)b * p.dvb + (int64_t)h * p.dvh + node * p.dvs) * (int64_t)sizeof(T);
      reinterpret_cast<T*>(row)[c0] = static_cast<T>(tot);
    }
  }
}

template <typename T, int CPL>
void launch_query(const BwdParams& p, cudaStream_t st) {
  const int ltiles = (p.L + kBwdGroups - 1) / kBwdGroups;
  const size_t smem = (size_t)kBwdGroups * p.S * 4;
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

template <typename T, int EL>
void launch_node_el(const BwdParams& p, cudaStream_t st, unsigned grid) {
  TA_PROFILE("bwd_node", st);
  if (p.log_n <= 16) bwd_node_kernel<T, EL, 16><<<grid, kNodeWarps * 32, 0, st>>>(p);
  else bwd_node_kernel<T, EL, 30><<<grid, kNodeWarps * 32, 0, st>>>(p);
}

template <typename T>
int run_rest(BwdParams& p, cudaStream_t st) {
  int rc = run_sort(p, st);
  if (rc) return rc;
  const int64_t nchunks_total = (int64_t)p.B * p.H * p.chunks_per_seg;
  const unsigned grid = (unsigned)((nchunks_total + kNodeWarps - 1) / kNodeWarps);
  const int el = (p.D + 31) / 32;
  switch (el) {
    case 1: launch_node_el<T, 1>(p, st, grid); break;
    case 2: launch_node_el<T, 2>(p, st, grid); break;
    case 3: launch_node_el<T, 3>(p, st, grid); break;
    case 4: launch_node_el<T, 4>(p, st, grid); break;
    case 5: case 6: case 7: case 8: launch_node_el<T, 8>(p, st, grid); break;
    default: return fail(TA_ERR_UNSUPPORTED, "head_dim too large for the node pass");
  }
  if ((rc = check_launch("backward node pass"))) return rc;
  const int64_t items = nchunks_total * (p.log_n + 1);
  TA_PROFILE("bwd_fixup", st);
  bwd_fixup_kernel<T><<<(unsigned)((items + 7) / 8), 256, 0, st>>>(p);
  return check_launch("backward fix-up");
}


// the typed half of ta_backward: query pass, then sort + node pass + fix-up
template <typename T>
int run_backward_typed(BwdParams& p, cudaStream_t st) {
  int rc = run_query<T>(p, st);
  if (rc) return rc;
  return run_rest<T>(p, st);
}
}  // namespace ta
