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
// result is bitwise repeatable.
//
// One CTA walks a range of consecutive chunks of one head. A node still open at the end of
// a chunk is carried in shared memory (f32) into the next chunk's epilogue, so only nodes
// cut by a RANGE boundary go to the partial buffer and the fix-up kernel (whose "chunks"
// are then the ranges). The q rows of chunk j+1 are gathered (cp.async) while chunk j runs
// its dV product, and its dO rows while chunk j+1 runs its dK product.
#pragma once

#include "ta_common.cuh"

namespace ta {

constexpr int kMmaChunk = kChunkMma;  // paths per sub-chunk
// 8 warps: warp w computes G rows [16 (w / 4), +16) x columns [(w % 4) D/4, +D/4); threads
// 0..127 own one path each (the run masks are per warp of paths)
constexpr int kMmaThreads = 256;
// A CTA walks a range of consecutive chunks; ranges are sized for about this many CTAs
// (148 SMs x 2 resident CTAs x 4 waves), from the problem shape alone so that the
// summation order does not depend on the device.
constexpr int64_t kNodeTargetCtas = 1184;
constexpr int kMaxRangeChunks = 32;

// position of the n-th (0-based) set bit of a 32-bit mask
__device__ __forceinline__ int nth_set_bit(uint32_t m, int n) {
  for (int i = 0; i < n; ++i) m &= m - 1;
  return __ffs(m) - 1;
}


// NT = n8 tiles per warp (D / 32)
template <typename T, int NT>
__global__ void __launch_bounds__(kMmaThreads, 2) bwd_node_mma_kernel(const BwdParams p, int range_chunks,
                                                                      int ranges_per_seg) {
  extern __shared__ __align__(16) unsigned char s_mma[];
  const int D = p.D;
  const int RS = mma_row_stride(D);
  const int ln = p.log_n, lev = ln + 1;
  T* s_q = reinterpret_cast<T*>(s_mma);
  T* s_g = s_q + kMmaChunk * RS;
  T* s_G = s_g + kMmaChunk * RS;
  float* s_co = reinterpret_cast<float*>(s_G + kMTile * kGStride);   // [lev][path]
  float* s_carry = s_co + lev * kMmaChunk;                            // [2][lev][D]
  uint32_t* s_l = reinterpret_cast<uint32_t*>(s_carry + 2 * lev * D);  // [2][path] query rows
  uint32_t* s_rkey = s_l + 2 * kMmaChunk;                            // [kMTile] run keys of a tile
  int* s_rlev = reinterpret_cast<int*>(s_rkey + kMTile);             // [kMTile] levels of a tile
  uint32_t* s_mask = reinterpret_cast<uint32_t*>(s_rlev + kMTile);   // [4][kMaxLev]
  int* s_runs = reinterpret_cast<int*>(s_mask + 4 * kMaxLev);       // runs per level
  int* s_off = s_runs + kMaxLev;                                    // first row of level
  int* s_pre = s_off + kMaxLev;  // [2][kMaxLev]: the carried node began before the range
  int* s_wpre = s_pre + 2 * kMaxLev;  // [4][kMaxLev]: runs of level d in earlier path warps
  __shared__ uint32_t s_edge[4];  // keys of the head's first / last path, and their flags

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // path of this thread; the upper half (tid >= 128) writes the low coefficient halves
  const int pt = tid & (kMmaChunk - 1), upper = tid >> 7;
  const int64_t range = blockIdx.x;
  const int seg = (int)(range / ranges_per_seg);
  const int rr = (int)(range - (int64_t)seg * ranges_per_seg);
  const int c_first = rr * range_chunks;
  const int cnt = min(range_chunks, p.chunks_per_seg - c_first);
  const int b = seg / p.H, h = seg - (seg / p.H) * p.H;
  const uint32_t* keys = p.keys[p.sorted_buf] + (int64_t)seg * p.P;
  const uint32_t* vals = p.vals[p.sorted_buf] + (int64_t)seg * p.P;
  const int64_t base_node = ((int64_t)1 << ln) - 1;
  const int64_t K = (int64_t)p.N - 1;
  const int64_t dk_es = p.dk_f32 ? 4 : 2;
  char* dkb = p.dk + ((int64_t)b * p.dkb + (int64_t)h * p.dkh) * dk_es;
  const int64_t dv_es = p.dv_f32 ? 4 : 2;
  char* dvb = p.dv + ((int64_t)b * p.dvb + (int64_t)h * p.dvh) * dv_es;
  float* part = p.partial + range * (int64_t)lev * 2 * D;
  uint8_t* flg = p.flags + range * (int64_t)lev * 2;
  const char* qbase = p.q + ((int64_t)b * p.qb + (int64_t)h * p.qh) * 2;
  const char* gbase = p.dout + ((int64_t)b * p.gb + (int64_t)h * p.gh) * 2;
  const int cpr = D * 2 / 16;  // 16-byte pieces per row
  const int nsig4 = p.sig_stride / 4;
  const int h4 = (nsig4 + 1) / 2;  // the lower half stores levels [0, 4 h4), the upper the rest
  const int sig_lo = upper ? h4 : 0, sig_hi = upper ? nsig4 : h4;

  // gather the rows of a sub-chunk's n paths (query rows in sl) into dst; rows past n are zero
  // (each thread copies one 16-byte column piece of every rows_per_it-th row)
  const int rows_per_it = kMmaThreads / cpr, gc = tid % cpr, gr0 = tid / cpr;
  auto gather_rows = [&](T* dst, const uint32_t* sl, const char* src, int64_t stride_el, int n) {
    if (gr0 < rows_per_it) {
      for (int r = gr0; r < n; r += rows_per_it)
        cp_async16(reinterpret_cast<char*>(dst + r * RS) + gc * 16, src + (int64_t)sl[r] * stride_el * 2 + gc * 16);
      if (n < kMmaChunk)
        for (int r = gr0; r < kMmaChunk; r += rows_per_it)
          if (r >= n) *reinterpret_cast<uint4*>(reinterpret_cast<char*>(dst + r * RS) + gc * 16) = make_uint4(0, 0, 0, 0);
    }
    cp_async_commit();  // committed even when empty: the wait counts stay fixed
  };
  // a path's per-level coefficients (this half's levels): registers first, s_co later
  float4 sg[4];
  float c_dl = 0.0f, c_w = 0.0f;
  auto load_coef = [&](uint32_t pl) {
    const float4* sg4 = reinterpret_cast<const float4*>(p.sig + ((int64_t)seg * p.P + pl) * p.sig_stride);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (sig_lo + i < sig_hi) sg[i] = __ldg(sg4 + sig_lo + i);
    c_dl = p.dlp[(int64_t)seg * p.P + pl];
    if (!p.coef_mode && !upper) {
      const uint32_t l = pl / (uint32_t)p.S, s = pl - l * (uint32_t)p.S;
      c_w = p.weights[(((int64_t)l * p.B + b) * p.H + h) * p.S + s];
    }
  };
  auto store_coef = [&](uint32_t key) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (sig_lo + i >= sig_hi) break;
      const float vv[4] = {sg[i].x, sg[i].y, sg[i].z, sg[i].w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int d = 4 * (sig_lo + i) + u;
        if (d < ln)
          s_co[d * kMmaChunk + pt] = p.coef_mode ? vv[u] : (((key >> (ln - 1 - d)) & 1u) ? -vv[u] : vv[u]) * c_dl;
      }
    }
    if (!upper) s_co[ln * kMmaChunk + pt] = p.coef_mode ? c_dl : c_w;
  };
  auto shared_depths = [&](uint32_t a, uint32_t c) -> int {
    const uint32_t x = a ^ c;
    return x == 0 ? ln + 1 : ln - (32 - __clz(x)) + 1;
  };
  // the records one sub-chunk needs, loaded a sub-chunk ahead: this thread's path (key,
  // position), the key before a warp's first path, and the keys around the sub-chunk
  struct Rec {
    uint32_t key, pl, wprev, key0, keyl, prev, next;
  };
  auto load_rec = [&](int64_t i0, int n, Rec& r) {
    r.key = 0; r.pl = 0; r.wprev = 0;
    if (pt < n) {
      r.key = keys[i0 + pt];
      r.pl = vals[i0 + pt];
      if (lane == 0 && pt > 0) r.wprev = keys[i0 + pt - 1];
    }
    r.key0 = keys[i0];
    r.keyl = keys[i0 + n - 1];
    r.prev = i0 > 0 ? keys[i0 - 1] : 0u;
    r.next = i0 + n < p.P ? keys[i0 + n] : 0u;
  };

  // prologue: the first sub-chunk's records, rows and coefficients; a zero G tile
  const int64_t range_i0 = (int64_t)c_first * kMmaChunk;
  Rec cur;
  {
    const int n = (int)min((int64_t)kMmaChunk, p.P - range_i0);
    load_rec(range_i0, n, cur);
    if (tid < n) s_l[tid] = cur.pl / (uint32_t)p.S;
    if (tid < kMaxLev) s_pre[tid] = 1;  // at the range start, every open node began before it
    if (tid < 4) s_edge[tid] = 0;
    if (tid < 2 * lev) flg[tid] = 0;
    for (int idx = tid; idx < kMTile * kGStride / 8; idx += kMmaThreads)
      reinterpret_cast<uint4*>(s_G)[idx] = make_uint4(0, 0, 0, 0);
    __syncthreads();
    gather_rows(s_q, s_l, qbase, p.qs, n);
    gather_rows(s_g, s_l, gbase, p.gs, n);
    if (pt < n) {
      load_coef(cur.pl);
      store_coef(cur.key);
    }
  }

  for (int j = 0; j < cnt; ++j) {
    const int64_t i0 = range_i0 + (int64_t)j * kMmaChunk;
    const int n = (int)min((int64_t)kMmaChunk, p.P - i0);
    const int64_t i1 = i0 + kMmaChunk;
    const int n1 = j + 1 < cnt ? (int)min((int64_t)kMmaChunk, p.P - i1) : 0;
    Rec nxt;  // the next sub-chunk's records, consumed after this one's dK product
    if (n1 > 0) load_rec(i1, n1, nxt);
    const float* carry_in = s_carry + (j & 1) * lev * D;
    float* carry_out = s_carry + ((j + 1) & 1) * lev * D;
    const int* pre_in = s_pre + (j & 1) * kMaxLev;
    int* pre_out = s_pre + ((j + 1) & 1) * kMaxLev;
    uint32_t* sl_next = s_l + ((j + 1) & 1) * kMmaChunk;

    // run structure: path i opens a new node at level d iff d >= sd(i)
    const bool has_prev = i0 > 0, has_next = i0 + n < p.P;
    uint32_t pk = __shfl_up_sync(0xffffffffu, cur.key, 1);  // key of the path before pt
    if (lane == 0) pk = pt > 0 ? cur.wprev : cur.prev;
    int my_sd = ln + 2;  // no new node anywhere (past the chunk)
    if (pt < n) my_sd = pt == 0 ? 0 : shared_depths(pk, cur.key);
    if (tid < kMmaChunk) {
      for (int d = 0; d <= ln; ++d) {
        const uint32_t m = __ballot_sync(0xffffffffu, my_sd <= d);
        if (lane == 0) s_mask[warp * kMaxLev + d] = m;
      }
    }
    const int open_sd = has_prev ? shared_depths(cur.prev, cur.key0) : 0;  // levels < open_sd began earlier
    const int cont_sd = has_next ? shared_depths(cur.keyl, cur.next) : 0;
    const bool last_sub = j + 1 == cnt;
    __syncthreads();
    if (warp == 0) {  // lane d: runs of level d, per-warp prefixes, first row of the level
      int runs = 0;
      if (lane <= ln) {
        for (int w = 0; w < 4; ++w) {
          s_wpre[w * kMaxLev + lane] = runs;
          runs += __popc(s_mask[w * kMaxLev + lane]);
        }
        s_runs[lane] = runs;
      }
      const int x = lane < ln ? runs : 0;  // dK rows (levels < ln); dV rows are numbered apart
      int incl = x;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (lane < ln) s_off[lane] = incl - x;
      if (lane == ln) s_off[ln] = 0;
    }
    if (tid < n1) sl_next[tid] = nxt.pl / (uint32_t)p.S;
    cp_async_wait_1();  // this sub-chunk's q rows
    __syncthreads();
    const int dk_rows = s_off[ln - 1] + s_runs[ln - 1];
    const int dv_rows = s_runs[ln];
    const uint32_t le_mask = lane == 31 ? 0xffffffffu : ((2u << lane) - 1u);
    const int pw = pt >> 5;

    // per pass (dK rows with q, then dV rows with dO), tiles of kMTile rows
    for (int pass = 0; pass < 2; ++pass) {
      const int rows = pass == 0 ? dk_rows : dv_rows;
      const T* s_b = pass == 0 ? s_q : s_g;
      for (int t0 = 0; t0 < rows; t0 += kMTile) {
        // G tile: each thread writes its path's entries (high half: column pt, low half:
        // column 128 + pt) and clears the same entries after the product, so the tile is
        // zero again without a block-wide fill
        uint32_t wrote = 0;
        if (pt < n) {
          const int dlo = pass == 0 ? 0 : ln, dhi = pass == 0 ? ln : ln + 1;
          for (int d = dlo; d < dhi; ++d) {
            // run index of path pt at level d: set bits of level d up to and including it
            const int r = s_wpre[pw * kMaxLev + d] + __popc(s_mask[pw * kMaxLev + d] & le_mask);
            const int row = s_off[d] + r - 1 - t0;
            if (row >= 0 && row < kMTile) {
              if (!upper && my_sd <= d) {  // this path opens the run: its key names the row's node
                s_rkey[row] = cur.key;
                s_rlev[row] = d;
              }
              const float c = s_co[d * kMmaChunk + pt];
              const T hi = to_t<T>(c);
              s_G[row * kGStride + upper * kMmaChunk + pt] = upper ? to_t<T>(c - static_cast<float>(hi)) : hi;
              wrote |= 1u << row;
            }
          }
        }
        __syncthreads();
        // C[16 rows of mt x D/4 slice] = G[16 x 256] * [B; B]
        const int mt = warp >> 2;
        float acc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[nt][e] = 0.0f;
        const int n0 = (warp & 3) * NT * 8;
#pragma unroll 4
        for (int ks = 0; ks < kGK / 16; ++ks) {
          uint32_t afr[4];
          ldsm_x4(afr, s_G + (mt * 16 + (lane & 15)) * kGStride + ks * 16 + ((lane >> 4) << 3));
          const int kb = (ks * 16) & (kMmaChunk - 1);  // the low half reuses the same rows of B
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            uint32_t bfr[2];
            ldsm_x2_trans(bfr, s_b + (kb + (lane & 15)) * RS + n0 + nt * 8);
            Mma16<T>::mma(acc[nt], afr, bfr);
          }
        }
        // epilogue. A node open from the previous sub-chunk adds its carried row; a node
        // that continues into the next sub-chunk is carried; a node cut by the range's
        // boundary goes to the partial buffer (slot 2d: began before the range, slot 2d+1:
        // continues past it) for the fix-up; every other node is final.
        const int g = lane >> 2, t = lane & 3;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int row = t0 + mt * 16 + g + half * 8;
          if (row >= rows) continue;
          const int d = s_rlev[row - t0];
          const int r = row - s_off[d];
          const uint32_t key = s_rkey[row - t0];
          const uint32_t pre = key >> (ln - d);
          const bool open_in = r == 0 && d < open_sd;
          const bool cont = r == s_runs[d] - 1 && d < cont_sd;
          const bool before = open_in && pre_in[d] != 0;  // the node began before the range
          const bool add_carry = open_in && j > 0;
          const bool carry = cont && !last_sub;
          float* pdst = nullptr;
          if (!carry) {
            if (before) pdst = part + (int64_t)(2 * d) * D;
            else if (cont) pdst = part + (int64_t)(2 * d + 1) * D;
          }
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const int c = n0 + nt * 8 + 2 * t;
            float2 v = make_float2(acc[nt][half * 2], acc[nt][half * 2 + 1]);
            if (add_carry) {
              const float2 cv = *reinterpret_cast<const float2*>(carry_in + d * D + c);
              v.x = cv.x + v.x;
              v.y = cv.y + v.y;
            }
            if (carry) {
              *reinterpret_cast<float2*>(carry_out + d * D + c) = v;
            } else if (pdst != nullptr) {
              *reinterpret_cast<float2*>(pdst + c) = v;
            } else if (d < ln) {
              const int64_t node = ((int64_t)1 << d) - 1 + pre;
              char* rowp = dkb + node * p.dks * dk_es;
              if (p.dk_f32) *reinterpret_cast<float2*>(reinterpret_cast<float*>(rowp) + c) = v;
              else *reinterpret_cast<uint32_t*>(reinterpret_cast<T*>(rowp) + c) = Elem<T>::pack2(v.x, v.y);
            } else {
              const int64_t leaf = (int64_t)pre + base_node - K;
              if (p.dv_f32)
                *reinterpret_cast<float2*>(reinterpret_cast<float*>(dvb + leaf * p.dvs * 4) + c) = v;
              else
                *reinterpret_cast<uint32_t*>(reinterpret_cast<T*>(dvb + leaf * p.dvs * 2) + c) =
                    Elem<T>::pack2(v.x, v.y);
            }
          }
          if ((warp & 3) == 0 && t == 0) {
            if (carry) pre_out[d] = before ? 1 : 0;
            else if (before) flg[2 * d] = cont ? 2 : 1;
            else if (cont) flg[2 * d + 1] = 1;
          }
        }
        // the dO rows must have landed before the dV pass: wait with the last dK tile's barrier
        if (pass == 0 && t0 + kMTile >= rows) cp_async_wait_0();
        __syncthreads();  // G tile, run keys and levels reused by the next tile or pass
        while (wrote) {
          const int row = __ffs(wrote) - 1;
          wrote &= wrote - 1;
          s_G[row * kGStride + upper * kMmaChunk + pt] = to_t<T>(0.0f);
        }
      }
      if (pass == 0) {  // s_q is free: gather the next sub-chunk's q rows behind the dV product
        if (n1 > 0) gather_rows(s_q, sl_next, qbase, p.qs, n1);
        else cp_async_commit();
        if (pt < n1) load_coef(nxt.pl);
      }
    }

    // unreached nodes: gaps between consecutive runs, and the head's two ends
    if (tid < n) {
      const int64_t zrow_dk = p.dks * dk_es, zrow_dv = p.dvs * dv_es;
      auto zero_node = [&](int d, int64_t pf) {
        if (d < ln) {
          char* rowp = dkb + (((int64_t)1 << d) - 1 + pf) * zrow_dk;
          for (int c = 0; c < D; c += 2) {
            if (p.dk_f32) *reinterpret_cast<float2*>(reinterpret_cast<float*>(rowp) + c) = make_float2(0.0f, 0.0f);
            else *reinterpret_cast<uint32_t*>(reinterpret_cast<T*>(rowp) + c) = 0u;
          }
        } else {
          char* rowp = dvb + (pf + base_node - K) * zrow_dv;
          for (int c = 0; c < D; c += 2) {
            if (p.dv_f32) *reinterpret_cast<float2*>(reinterpret_cast<float*>(rowp) + c) = make_float2(0.0f, 0.0f);
            else *reinterpret_cast<uint32_t*>(reinterpret_cast<T*>(rowp) + c) = 0u;
          }
        }
      };
      const uint32_t my_key = cur.key;
      if (tid > 0 || has_prev) {  // path i opening a run at level d leaves a gap after the previous run
        if (my_key - pk > 1u) {
          const int sd = tid > 0 ? my_sd : shared_depths(pk, my_key);
          for (int d = sd; d <= ln; ++d) {
            const int64_t a = (int64_t)(pk >> (ln - d)), c = (int64_t)(my_key >> (ln - d));
            for (int64_t pf = a + 1; pf < c; ++pf) zero_node(d, pf);
          }
        }
      } else {  // the head's first path: everything to its left (zeroed by the whole CTA below)
        s_edge[0] = my_key;
        s_edge[2] = 1;
      }
      if (tid == n - 1 && !has_next) {  // the head's last path: everything to its right
        s_edge[1] = my_key;
        s_edge[3] = 1;
      }
    }
    __syncthreads();
    if (s_edge[2] | s_edge[3]) {
      // the head's two ends (every node left of its first path, right of its last): few
      // nodes for a head whose paths spread over its leaves, up to half the tree when they
      // cover only part of it (causal or sequence-parallel queries), so all threads share it
      for (int side = 0; side < 2; ++side) {
        if (!s_edge[2 + side]) continue;
        const uint32_t key = s_edge[side];
        for (int d = 0; d <= ln; ++d) {
          const int64_t at = (int64_t)(key >> (ln - d));
          const int64_t lo = side == 0 ? 0 : at + 1;
          const int64_t hi = side == 0 ? at : ((int64_t)1 << d);  // exclusive
          const int64_t pairs = (hi - lo) * (D / 2);
          for (int64_t i = tid; i < pairs; i += kMmaThreads) {
            const int64_t pf = lo + i / (D / 2);
            const int c = (int)(i % (D / 2)) * 2;
            if (d < ln) {
              char* rowp = dkb + (((int64_t)1 << d) - 1 + pf) * p.dks * dk_es;
              if (p.dk_f32) *reinterpret_cast<float2*>(reinterpret_cast<float*>(rowp) + c) = make_float2(0.0f, 0.0f);
              else *reinterpret_cast<uint32_t*>(reinterpret_cast<T*>(rowp) + c) = 0u;
            } else {
              char* rowp = dvb + (pf + base_node - K) * p.dvs * dv_es;
              if (p.dv_f32) *reinterpret_cast<float2*>(reinterpret_cast<float*>(rowp) + c) = make_float2(0.0f, 0.0f);
              else *reinterpret_cast<uint32_t*>(reinterpret_cast<T*>(rowp) + c) = 0u;
            }
          }
        }
      }
      __syncthreads();
      if (tid == 0) s_edge[2] = s_edge[3] = 0;
    }
    if (last_sub) break;
    // s_g is free: gather the next sub-chunk's dO rows behind its dK product. The s_co reads
    // of this sub-chunk ended before the last tile's barrier; the next run-structure barrier
    // publishes the new coefficients.
    gather_rows(s_g, sl_next, gbase, p.gs, n1);
    cur = nxt;
    if (pt < n1) store_coef(cur.key);
  }
}

// Range geometry of the tensor-core node pass: chunks per range and ranges per head.
inline void node_mma_ranges(const BwdParams& p, int& range_chunks, int& ranges_per_seg) {
  const int64_t total = (int64_t)p.B * p.H * p.chunks_per_seg;
  int64_t rc = p.node_range_chunks > 0 ? p.node_range_chunks : (total + kNodeTargetCtas - 1) / kNodeTargetCtas;
  rc = rc < 1 ? 1 : (rc > kMaxRangeChunks ? kMaxRangeChunks : rc);
  range_chunks = (int)rc;
  ranges_per_seg = (int)((p.chunks_per_seg + rc - 1) / rc);
}

template <typename T, int NT>
void launch_node_mma(const BwdParams& p, cudaStream_t st) {
  const size_t smem = mma_node_smem(p.D, p.log_n);
  cudaFuncSetAttribute(bwd_node_mma_kernel<T, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  int range_chunks, ranges_per_seg;
  node_mma_ranges(p, range_chunks, ranges_per_seg);
  const int64_t ranges = (int64_t)p.B * p.H * ranges_per_seg;
  bwd_node_mma_kernel<T, NT><<<(unsigned)ranges, kMmaThreads, smem, st>>>(p, range_chunks, ranges_per_seg);
}

}  // namespace ta
