// Tensor-core node pass of the deterministic backward (bf16 inputs), sm_100a.
//
// For one chunk of kMmaChunk consecutive leaf-sorted paths of a head, every tree level's
// nodes are contiguous runs of paths, so the chunk's dK contributions form one small dense
// product
//     C[rows x D] = G[rows x paths] * Q[paths x D],
// with one row per (level, node) the chunk touches and G[row(p, d)][p] = gl_{p,d}; dV is the
// same with the weights and dO rows. The rows are few (about 30 for 128 densely sampled
// paths), so a CTA forms G in shared memory and runs the product on the tensor cores with
// mma.sync m16n8k16 (bf16 operands, f32 accumulate). G's f32 coefficients are split into
// bf16 high and low parts concatenated along K (Q is exact in bf16), which keeps ~16 more
// mantissa bits than a single bf16 coefficient. The MMA fixes the summation order, so the
// result is bitwise repeatable. Nodes cut by a chunk boundary go to the partial buffer and
// the fix-up kernel, as in the CUDA-core node pass.
#pragma once

#include "ta_common.cuh"

namespace ta {

constexpr int kMmaChunk = 128;    // paths per CTA
constexpr int kMmaThreads = 128;  // 4 warps; warp w owns columns [w D/4, (w+1) D/4)
constexpr int kMTile = 32;        // G rows per MMA pass (two m16 tiles)
constexpr int kGK = 2 * kMmaChunk;  // K of the product: high | low coefficient halves
constexpr int kGStride = kGK + 8;   // padded row (elements) of the G tile
constexpr int kMaxLev = 31;

__host__ __device__ inline int mma_row_stride(int D) { return D + 8; }  // padded Q/dO rows
__host__ __device__ inline size_t mma_node_smem(int D) {
  return (size_t)2 * kMmaChunk * mma_row_stride(D) * 2  // q, dO (bf16)
         + (size_t)kMTile * kGStride * 2                // G tile (bf16)
         + (size_t)kMmaChunk * 32 * 4                   // coefficients [level][path]
         + (size_t)kMmaChunk * 4 * 3                    // keys, shared depths, query rows
         + (size_t)kMTile * 4 * 2                       // tile rows: run key, level
         + (size_t)4 * kMaxLev * 4                      // run-start masks [warp][level]
         + (size_t)kMaxLev * 4 * 2 + 64;                // rows per level, row offsets
}

__device__ __forceinline__ void ldsm_x4(uint32_t* r, const void* p) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
__device__ __forceinline__ void ldsm_x2_trans(uint32_t* r, const void* p) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1]) : "r"(a));
}
__device__ __forceinline__ void mma_bf16(float* c, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// position of the n-th (0-based) set bit of a 32-bit mask
__device__ __forceinline__ int nth_set_bit(uint32_t m, int n) {
  for (int i = 0; i < n; ++i) m &= m - 1;
  return __ffs(m) - 1;
}

// NT = n8 tiles per warp (D / 32)
template <int NT>
__global__ void __launch_bounds__(kMmaThreads) bwd_node_mma_kernel(const BwdParams p) {
  using T = __nv_bfloat16;
  extern __shared__ __align__(16) unsigned char s_mma[];
  const int D = p.D;
  const int RS = mma_row_stride(D);
  T* s_q = reinterpret_cast<T*>(s_mma);
  T* s_g = s_q + kMmaChunk * RS;
  T* s_G = s_g + kMmaChunk * RS;
  float* s_co = reinterpret_cast<float*>(s_G + kMTile * kGStride);  // [32][path]
  uint32_t* s_key = reinterpret_cast<uint32_t*>(s_co + kMmaChunk * 32);
  int* s_sd = reinterpret_cast<int*>(s_key + kMmaChunk);
  uint32_t* s_l = reinterpret_cast<uint32_t*>(s_sd + kMmaChunk);     // query row of each path
  uint32_t* s_rkey = s_l + kMmaChunk;                                // [kMTile] run keys of a tile
  int* s_rlev = reinterpret_cast<int*>(s_rkey + kMTile);             // [kMTile] levels of a tile
  uint32_t* s_mask = reinterpret_cast<uint32_t*>(s_rlev + kMTile);   // [4][kMaxLev]
  int* s_runs = reinterpret_cast<int*>(s_mask + 4 * kMaxLev);       // runs per level
  int* s_off = s_runs + kMaxLev;                                    // first row of level

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t chunk = blockIdx.x;
  const int seg = (int)(chunk / p.chunks_per_seg);
  const int cis = (int)(chunk - (int64_t)seg * p.chunks_per_seg);
  const int b = seg / p.H, h = seg - (seg / p.H) * p.H;
  const int ln = p.log_n;
  const int64_t i0 = (int64_t)cis * kMmaChunk;
  const int n = (int)min((int64_t)kMmaChunk, p.P - i0);
  const uint32_t* keys = p.keys[p.sorted_buf] + (int64_t)seg * p.P;
  const uint32_t* vals = p.vals[p.sorted_buf] + (int64_t)seg * p.P;
  const int64_t base_node = ((int64_t)1 << ln) - 1;
  const int64_t K = (int64_t)p.N - 1;
  const int64_t dk_es = p.dk_f32 ? 4 : 2;
  char* dkb = p.dk + ((int64_t)b * p.dkb + (int64_t)h * p.dkh) * dk_es;
  const int64_t dv_es = p.dv_f32 ? 4 : 2;
  char* dvb = p.dv + ((int64_t)b * p.dvb + (int64_t)h * p.dvh) * dv_es;
  float* part = p.partial + chunk * (int64_t)(ln + 1) * 2 * D;
  uint8_t* flg = p.flags + chunk * (int64_t)(ln + 1) * 2;

  // 1. stage: records, q / dO rows (cp.async), coefficients
  const char* qbase = p.q + ((int64_t)b * p.qb + (int64_t)h * p.qh) * 2;
  const char* gbase = p.dout + ((int64_t)b * p.gb + (int64_t)h * p.gh) * 2;
  uint32_t my_key = 0, my_pl = 0;
  if (tid < n) {
    my_key = keys[i0 + tid];
    my_pl = vals[i0 + tid];
    s_key[tid] = my_key;
    s_l[tid] = my_pl / (uint32_t)p.S;
  }
  __syncthreads();
  const int cpr = D * 2 / 16;  // 16-byte pieces per row
  for (int idx = tid; idx < n * cpr; idx += kMmaThreads) {
    const int r = idx / cpr, c = idx - r * cpr;
    const uint32_t l = s_l[r];
    cp_async16(reinterpret_cast<char*>(s_q + r * RS) + c * 16, qbase + (int64_t)l * p.qs * 2 + c * 16);
    cp_async16(reinterpret_cast<char*>(s_g + r * RS) + c * 16, gbase + (int64_t)l * p.gs * 2 + c * 16);
  }
  cp_async_commit();
  for (int idx = tid; idx < (kMmaChunk - n) * cpr; idx += kMmaThreads) {  // rows past the chunk
    const int r = n + idx / cpr, c = idx % cpr;
    *reinterpret_cast<uint4*>(reinterpret_cast<char*>(s_q + r * RS) + c * 16) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(reinterpret_cast<char*>(s_g + r * RS) + c * 16) = make_uint4(0, 0, 0, 0);
  }
  if (tid < n) {
    const uint32_t l = my_pl / (uint32_t)p.S;
    const uint32_t s = my_pl - l * (uint32_t)p.S;
    const float dl = p.dlp[(int64_t)seg * p.P + my_pl];
    const float4* sg4 = reinterpret_cast<const float4*>(p.sig + ((int64_t)seg * p.P + my_pl) * p.sig_stride);
    for (int d4 = 0; d4 < p.sig_stride / 4; ++d4) {
      const float4 v = __ldg(sg4 + d4);
      const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int d = 4 * d4 + u;
        if (d < ln)
          s_co[d * kMmaChunk + tid] = p.coef_mode ? vv[u] : (((my_key >> (ln - 1 - d)) & 1u) ? -vv[u] : vv[u]) * dl;
      }
    }
    s_co[ln * kMmaChunk + tid] = p.coef_mode ? dl : p.weights[(((int64_t)l * p.B + b) * p.H + h) * p.S + s];
  }
  cp_async_wait_0();
  __syncthreads();

  // 2. run structure: path i opens a new node at level d iff d >= sd(i)
  auto shared_depths = [&](uint32_t a, uint32_t c) -> int {
    const uint32_t x = a ^ c;
    return x == 0 ? ln + 1 : ln - (32 - __clz(x)) + 1;
  };
  const uint32_t prev_key = i0 > 0 ? keys[i0 - 1] : 0u;
  const bool has_prev = i0 > 0;
  const bool has_next = i0 + n < p.P;
  const uint32_t next_key = has_next ? keys[i0 + n] : 0u;
  int my_sd = ln + 2;  // no new node anywhere (past the chunk)
  if (tid < n) my_sd = tid == 0 ? 0 : shared_depths(s_key[tid - 1], my_key);
  s_sd[tid] = my_sd;
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int d = 0; d <= ln; ++d) {
    const uint32_t m = __ballot_sync(0xffffffffu, my_sd <= d);
    if (lane == 0) s_mask[warp * kMaxLev + d] = m;
  }
  __syncthreads();
  if (tid == 0) {
    int off = 0;
    for (int d = 0; d <= ln; ++d) {
      int r = 0;
      for (int w = 0; w < 4; ++w) r += __popc(s_mask[w * kMaxLev + d]);
      s_runs[d] = r;
      s_off[d] = off;
      off += r;
      if (d == ln - 1) off = 0;  // dV rows are numbered separately
    }
  }
  const int open_sd = has_prev ? shared_depths(prev_key, s_key[0]) : 0;  // levels < open_sd started earlier
  const int cont_sd = has_next ? shared_depths(s_key[n - 1], next_key) : 0;
  if (tid <= ln) {  // flags of this chunk
    flg[2 * tid] = 0;
    flg[2 * tid + 1] = 0;
  }
  __syncthreads();
  const int dk_rows = s_off[ln - 1] + s_runs[ln - 1];
  const int dv_rows = s_runs[ln];

  // 3. per pass (dK rows with q, then dV rows with dO), tiles of kMTile rows
  for (int pass = 0; pass < 2; ++pass) {
    const int rows = pass == 0 ? dk_rows : dv_rows;
    const T* s_b = pass == 0 ? s_q : s_g;
    for (int t0 = 0; t0 < rows; t0 += kMTile) {
      // G tile: zero, then scatter each path's coefficients (high | low)
      for (int idx = tid; idx < kMTile * kGStride / 8; idx += kMmaThreads)
        reinterpret_cast<uint4*>(s_G)[idx] = make_uint4(0, 0, 0, 0);
      __syncthreads();
      if (tid < n) {
        const int dlo = pass == 0 ? 0 : ln, dhi = pass == 0 ? ln : ln + 1;
        for (int d = dlo; d < dhi; ++d) {
          // run index of path tid at level d: set bits of level d up to and including it
          int r = __popc(s_mask[warp * kMaxLev + d] & (lt_mask | (1u << lane)));
          for (int w = 0; w < warp; ++w) r += __popc(s_mask[w * kMaxLev + d]);
          const int row = s_off[d] + r - 1 - t0;
          if (row >= 0 && row < kMTile) {
            if (s_sd[tid] <= d) {  // this path opens the run: its key names the row's node
              s_rkey[row] = my_key;
              s_rlev[row] = d;
            }
            const float c = s_co[d * kMmaChunk + tid];
            const T hi = __float2bfloat16_rn(c);
            const T lo = __float2bfloat16_rn(c - __bfloat162float(hi));
            s_G[row * kGStride + tid] = hi;
            s_G[row * kGStride + kMmaChunk + tid] = lo;
          }
        }
      }
      __syncthreads();
      // C[32 x D/4 slice] = G[32 x 256] * [B; B]
      float acc[2][NT][4];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[mt][nt][e] = 0.0f;
      const int n0 = warp * NT * 8;
#pragma unroll 4
      for (int ks = 0; ks < kGK / 16; ++ks) {
        uint32_t afr[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          const int row = mt * 16 + (lane & 15);
          const int col = ks * 16 + ((lane >> 4) << 3);
          ldsm_x4(afr[mt], s_G + row * kGStride + col);
        }
        const int kb = (ks * 16) & (kMmaChunk - 1);  // the low half reuses the same rows of B
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          uint32_t bfr[2];
          ldsm_x2_trans(bfr, s_b + (kb + (lane & 15)) * RS + n0 + nt * 8);
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) mma_bf16(acc[mt][nt], afr[mt], bfr);
        }
      }
      // epilogue: rows -> dk / dv, partials, flags
      const int g = lane >> 2, t = lane & 3;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int row = t0 + mt * 16 + g + half * 8;
          if (row >= rows) continue;
          const int d = s_rlev[row - t0];
          const int r = row - s_off[d];
          const uint32_t key = s_rkey[row - t0];
          const uint32_t pre = key >> (ln - d);
          const bool first = r == 0, last = r == s_runs[d] - 1;
          const bool before = first && d < open_sd;
          const bool cont = last && d < cont_sd;
          float* pdst = nullptr;
          if (before) pdst = part + (int64_t)(2 * d) * D;
          else if (cont) pdst = part + (int64_t)(2 * d + 1) * D;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const int c = n0 + nt * 8 + 2 * t;
            const float2 v = make_float2(acc[mt][nt][half * 2], acc[mt][nt][half * 2 + 1]);
            if (pdst != nullptr) {
              *reinterpret_cast<float2*>(pdst + c) = v;
            } else if (d < ln) {
              const int64_t node = ((int64_t)1 << d) - 1 + pre;
              char* rowp = dkb + node * p.dks * dk_es;
              if (p.dk_f32) *reinterpret_cast<float2*>(reinterpret_cast<float*>(rowp) + c) = v;
              else *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<T*>(rowp) + c) = __floats2bfloat162_rn(v.x, v.y);
            } else {
              const int64_t leaf = (int64_t)pre + base_node - K;
              if (p.dv_f32)
                *reinterpret_cast<float2*>(reinterpret_cast<float*>(dvb + leaf * p.dvs * 4) + c) = v;
              else
                *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<T*>(dvb + leaf * p.dvs * 2) + c) =
                    __floats2bfloat162_rn(v.x, v.y);
            }
          }
          if (warp == 0 && t == 0 && (before || cont)) {
            if (before) flg[2 * d] = (cont ? 2 : 1);
            else flg[2 * d + 1] = 1;
          }
        }
      }
      __syncthreads();  // G tile reused by the next pass
    }
  }

  // 4. unreached nodes: gaps between consecutive runs, and the head's two ends
  const int64_t zrow_dk = p.dks * dk_es, zrow_dv = p.dvs * dv_es;
  auto zero_node = [&](int d, int64_t pre) {
    if (d < ln) {
      char* rowp = dkb + (((int64_t)1 << d) - 1 + pre) * zrow_dk;
      for (int c = 0; c < D; c += 2) {
        if (p.dk_f32) *reinterpret_cast<float2*>(reinterpret_cast<float*>(rowp) + c) = make_float2(0.0f, 0.0f);
        else *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<T*>(rowp) + c) = __floats2bfloat162_rn(0.0f, 0.0f);
      }
    } else {
      char* rowp = dvb + (pre + base_node - K) * zrow_dv;
      for (int c = 0; c < D; c += 2) {
        if (p.dv_f32) *reinterpret_cast<float2*>(reinterpret_cast<float*>(rowp) + c) = make_float2(0.0f, 0.0f);
        else *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<T*>(rowp) + c) = __floats2bfloat162_rn(0.0f, 0.0f);
      }
    }
  };
  // path i (> 0) opening a run at level d leaves a gap after the previous run
  if (tid < n) {
    const uint32_t pk = tid > 0 ? s_key[tid - 1] : (has_prev ? prev_key : 0u);
    if (tid > 0 || has_prev) {
      if (my_key - pk > 1u) {
        const int sd = tid > 0 ? my_sd : shared_depths(pk, my_key);
        for (int d = sd; d <= ln; ++d) {
          const int64_t a = (int64_t)(pk >> (ln - d)), c = (int64_t)(my_key >> (ln - d));
          for (int64_t pf = a + 1; pf < c; ++pf) zero_node(d, pf);
        }
      }
    } else {  // the head's first path: everything to its left
      for (int d = 0; d <= ln; ++d)
        for (int64_t pf = 0; pf < (int64_t)(my_key >> (ln - d)); ++pf) zero_node(d, pf);
    }
    if (tid == n - 1 && !has_next) {  // the head's last path: everything to its right
      for (int d = 0; d <= ln; ++d) {
        const int64_t last = ((int64_t)1 << d) - 1;
        for (int64_t pf = (int64_t)(my_key >> (ln - d)) + 1; pf <= last; ++pf) zero_node(d, pf);
      }
    }
  }
}

template <int NT>
void launch_node_mma(const BwdParams& p, cudaStream_t st) {
  const size_t smem = mma_node_smem(p.D);
  cudaFuncSetAttribute(bwd_node_mma_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t chunks = (int64_t)p.B * p.H * p.chunks_per_seg;
  bwd_node_mma_kernel<NT><<<(unsigned)chunks, kMmaThreads, smem, st>>>(p);
}

}  // namespace ta
