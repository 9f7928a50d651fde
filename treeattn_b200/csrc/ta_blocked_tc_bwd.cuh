// Leaf-block attention backward of the generalised tree on the 5th-generation tensor cores
// (tcgen05 + TMEM), sm_100a, 16-bit inputs.
//
// One CTA of 512 threads per (batch*head, leaf block) walks the block's leaf-sorted
// (query, path) pairs in tiles of 128 (one pair per TMEM lane). Per tile:
//   1. S = Q_g K^T and dP = dO_g V^T: 2 * D/16 tcgen05.mma (M = 128 pairs, N = Lb) issued by
//      one thread into TMEM, committed to an mbarrier;
//   2. warp w reads TMEM lanes [32 (w % 4), +32) (its pairs) and part w / 4 of four column
//      parts:
//      P = exp2(scale log2(e) s - lse2) with the pair's base-2 log-sum-exp saved by the forward
//      (no row reduction), keys beyond the causal boundary masked, then w_s P and
//      dS = P (w_s dP - delta) as 16-bit K-major tiles in shared memory;
//   3. one thread issues dq = dS K (N = D, TMEM columns of its own), dV += (w P)^T dO and
//      dK += dS^T Q; dV / dK accumulate in TMEM over the block's tiles,
//      with the block's keys as the MMA rows when Lb = 128, else transposed (head_dim = 128
//      rows, keys as columns);
//   4. while those run, the warps issue every global read of the next tile (its query and dO
//      rows, its pairs' w_s, delta and log-sum-exp, its raw dz rows, and the paths of the tile
//      after it) as cp.async into the other buffers, so no thread waits on a global load, and
//      add this tile's summary gradients dc += dz^T Q on mma.sync (dz split into 16-bit high
//      and low parts; M = levels * fanout is too small for tcgen05);
//   5. each warp reads its dq rows back and stores them (input dtype) to the per-path buffer, while
//      the next tile's S and dP MMAs run.
// A block's pair range comes from a table built once per call (blk_block_ranges_kernel).
// Every operand tile is stored as 128-byte-swizzled atoms (8 rows x 64 16-bit columns, the
// 16-byte chunks of row i XOR-permuted by i % 8; sw128_off), which the tensor cores read
// without bank conflicts. The same physical tile serves as a K-major operand over its columns
// (SBO 1024, a 16-column step is 32 bytes into the atom) and as an MN-major operand over its
// rows (LBO = the atom-column stride, SBO 1024, a 16-row step is 2048 bytes), so K, Q, dO,
// w P and dS are each staged once. Every mbarrier wait is
// bounded as in the forward: the CTA agrees on a failure, waits once more for its issued MMAs,
// records the status word and frees its TMEM.
#pragma once

#include "ta_blocked_tc.cuh"

namespace ta {

constexpr int kTcBwdWarps = 16;                 // 4 TMEM lane quadrants x 4 column parts
constexpr int kTcBwdThreads = kTcBwdWarps * 32;
constexpr int kTcBwdParts = kTcBwdWarps / 4;
constexpr int kTcBwdDcItems = (16 + kTcBwdWarps - 1) / kTcBwdWarps;  // summary items per warp

template <int LB, int D>
struct BlkTcBwdGeom {
  static constexpr bool KEY_ROWS = LB == 128;           // dV / dK rows = keys (else head_dim)
  static constexpr int NV = KEY_ROWS ? D : LB;          // TMEM columns of dV, and of dK
  static constexpr int COLS_USED = 2 * LB + 2 * NV + D;  // S, dP, dV, dK, dq
  static constexpr int COLS = COLS_USED <= 256 ? 256 : 512;
  static constexpr size_t KT = (size_t)LB * D * 2;       // K_blk or V_blk
  static constexpr size_t QT = (size_t)kTcRows * D * 2;  // one Q or dO tile
  static constexpr size_t PT = (size_t)kTcRows * LB * 2; // the w P or dS tile
  static constexpr size_t ZT = (size_t)kTcRows * kZLd * 2;
  static constexpr size_t SCAL = (size_t)3 * kTcRows * 4;  // w_s, delta, lse2 of one tile
  static constexpr size_t oK = 0, oV = KT, oQ = 2 * KT, oG = oQ + 2 * QT, oWP = oG + 2 * QT,
                          oDS = oWP + PT, oZH = oDS + PT, oZL = oZH + ZT, oSC = oZL + ZT,
                          oPATH = oSC + 2 * SCAL, oBAR = oPATH + 3 * kTcRows * 4,
                          oZRAW = oBAR + 64;
  // shared memory with a raw dz staging tile of zw float32 columns
  static constexpr size_t smem(int zw) { return oZRAW + (size_t)kTcRows * zw * 4 + 1024; }
  static constexpr bool OK = (LB == 128 || D == 128) && LB >= 32 && LB % 16 == 0 && D % 16 == 0 &&
                             COLS_USED <= 512;
};

template <typename T, int LB, int D>
__global__ void __launch_bounds__(kTcBwdThreads, 1) blk_attn_bwd_tc_kernel(const BlkMmaParams p) {
  using G = BlkTcBwdGeom<LB, D>;
  static_assert(G::OK, "unsupported leaf block / head_dim for the tcgen05 backward");
  extern __shared__ __align__(1024) unsigned char sm_raw[];
  // the swizzled operand tiles need 1024-byte-aligned bases
  unsigned char* sm = sm_raw + ((1024u - (smem_u32(sm_raw) & 1023u)) & 1023u);
  unsigned char* sK = sm + G::oK;
  unsigned char* sV = sm + G::oV;
  unsigned char* sWP = sm + G::oWP;
  unsigned char* sDS = sm + G::oDS;
  uint16_t* s_zh = reinterpret_cast<uint16_t*>(sm + G::oZH);
  uint16_t* s_zl = reinterpret_cast<uint16_t*>(sm + G::oZL);
  uint32_t* s_path = reinterpret_cast<uint32_t*>(sm + G::oPATH);  // [3][128] ring of tiles
  float* s_zraw = reinterpret_cast<float*>(sm + G::oZRAW);        // [128][zw]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + G::oBAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 2);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int quad = warp & 3, part = warp >> 2;
  const int bh = blockIdx.x / p.nb;
  const int j = blockIdx.x - bh * p.nb;
  const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const uint32_t* vals = p.svals + (int64_t)bh * p.P;
  const uint32_t mS = smem_u32(bars), mD = smem_u32(bars + 1);
  const int64_t key0 = (int64_t)j * LB;
  const int64_t beg = p.ranges[(int64_t)bh * (p.nb + 1) + j];
  const int64_t end = p.ranges[(int64_t)bh * (p.nb + 1) + j + 1];
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(mS) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(mD) : "memory");
  }
  __syncwarp();  // tcgen05.alloc is .sync.aligned: warp 0 must be converged
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s_tmem)),
                 "r"(G::COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  const int DF = p.DF;
  const int zsh = DF <= 16 ? 4 : 5;  // log2 of the dz tile width
  const int zmt = (DF + 15) >> 4;
  constexpr int NPAIR = D / 16;
  // the paths of tile x (at t0) into ring slot x % 3
  auto fetch_paths = [&](int64_t t0, int slot) {
    if (tid < kTcRows) {
      uint32_t* dst = s_path + slot * kTcRows + tid;
      if (t0 + tid < end) cp_async4(dst, vals + t0 + tid);
      else *dst = 0u;
    }
  };
  // K_blk and V_blk, both in the core-matrix layout over (key, d); the first tile's paths
  constexpr int CPR = D * 2 / 16;
  for (int i = tid; i < LB * CPR; i += blockDim.x) {
    const int r = i / CPR, c = i - r * CPR;
    const int64_t key = key0 + r;
    cp_async16(sK + sw128_off(r, c, LB), p.k + (key * p.ks + (int64_t)b * p.kb + (int64_t)h * p.kh) * 2 + c * 16);
    cp_async16(sV + sw128_off(r, c, LB), p.v + (key * p.vs + (int64_t)b * p.vb + (int64_t)h * p.vh) * 2 + c * 16);
  }
  if (beg < end) fetch_paths(beg, 0);
  cp_async_commit();
  for (int i = tid; i < (kTcRows << zsh); i += blockDim.x) s_zraw[i] = 0.0f;

  // every global read of tile x (at t0, buffer `buf`), issued one tile ahead with cp.async:
  // threads 0-127 the query rows and the pair scalars, threads 128-255 the dO rows; all
  // threads the raw dz rows; and the paths of tile x + 1. Rows past the tile are zero.
  auto gather = [&](int64_t t0, int buf, int slot) {
    const int n = (int)min((int64_t)kTcRows, end - t0);
    const int r = tid & (kTcRows - 1);
    const int role = tid >> 7;                     // which tensor and which of its chunks
    const bool dout = role >= kTcBwdParts / 2;
    constexpr int CPP = CPR / (kTcBwdParts / 2);   // 16-byte chunks of a row per thread
    const int cfirst = (role % (kTcBwdParts / 2)) * CPP;
    unsigned char* dst = sm + (dout ? G::oG : G::oQ) + buf * G::QT;
    const uint32_t path = s_path[slot * kTcRows + r];
    const int64_t l = (int64_t)(path / (uint32_t)p.S);
    const char* src = dout ? p.dout + (l * p.gs + (int64_t)b * p.gb + (int64_t)h * p.gh) * 2
                           : p.q + (l * p.qs + (int64_t)b * p.qb + (int64_t)h * p.qh) * 2;
#pragma unroll
    for (int c = cfirst; c < cfirst + CPP; ++c) {
      unsigned char* d_ = dst + sw128_off(r, c, kTcRows);
      if (r < n) cp_async16(d_, src + c * 16);
      else *reinterpret_cast<uint4*>(d_) = make_uint4(0, 0, 0, 0);
    }
    if (role == 0) {
      float* sc = reinterpret_cast<float*>(sm + G::oSC + buf * G::SCAL);
      if (r < n) {
        const int64_t s = (int64_t)path - l * p.S;
        cp_async4(sc + r, p.weights + ((l * p.B + b) * p.H + h) * p.S + s);
        cp_async4(sc + kTcRows + r, p.delta + (int64_t)bh * p.P + path);
        cp_async4(sc + 2 * kTcRows + r, p.lse + (int64_t)bh * p.P + path);
      } else {
        sc[r] = sc[kTcRows + r] = sc[2 * kTcRows + r] = 0.0f;
      }
    }
    if ((DF & 3) == 0) {
      // whole 16-byte pieces of the dz rows (the pad columns stay zero from the prologue)
      const int cpr = DF >> 2;
      for (int i = tid; i < kTcRows * cpr; i += blockDim.x) {
        const int rr = i / cpr, c = i - rr * cpr;
        float* d_ = s_zraw + (rr << zsh) + c * 4;
        if (rr < n)
          cp_async16(d_, p.dz_rows + ((int64_t)bh * p.P + s_path[slot * kTcRows + rr]) * DF + c * 4);
        else
          *reinterpret_cast<float4*>(d_) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
    } else {
      for (int i = tid; i < (kTcRows << zsh); i += blockDim.x) {
        const int rr = i >> zsh, c = i & ((1 << zsh) - 1);
        if (rr < n && c < DF)
          cp_async4(s_zraw + i, p.dz_rows + ((int64_t)bh * p.P + s_path[slot * kTcRows + rr]) * DF + c);
        else
          s_zraw[i] = 0.0f;
      }
    }
    if (t0 + kTcRows < end) fetch_paths(t0 + kTcRows, slot == 2 ? 0 : slot + 1);
    cp_async_commit();
  };

  float acc_dc[kTcBwdDcItems][2][4];
#pragma unroll
  for (int i = 0; i < kTcBwdDcItems; ++i)
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc_dc[i][t][e] = 0.0f;

  cp_async_wait_0();  // K_blk, V_blk, the first tile's paths
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const uint32_t tS = tmem, tP = tmem + LB, tV = tmem + 2 * LB, tK = tmem + 2 * LB + G::NV,
                 tQ = tmem + 2 * LB + 2 * G::NV;
  const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
  if (beg < end) gather(beg, 0, 0);
  constexpr uint32_t idS = tc_idesc<T>(kTcRows, LB, 0, 0);
  constexpr uint32_t idDQ = tc_idesc<T>(kTcRows, D, 0, 1);
  constexpr uint32_t idKV = G::KEY_ROWS ? tc_idesc<T>(LB, D, 1, 1) : tc_idesc<T>(D, LB, 1, 1);
  const float sl2 = p.scale * kLog2e;
  const int r = quad * 32 + lane;  // this thread's pair row (TMEM lane)
  uint32_t phS = 0, phD = 0;
  int failed = 0;  // 1: a wait in the tile loop expired (the last commit was mS), 2: the final
                   // dq / dV / dK wait expired (the last commit was mD)
  int buf = 0, slot = 0;
  // dq rows of the tile in ring slot `sl` with `n` pairs (this thread's pair, its part of the
  // columns), once its MMAs completed
  auto dq_out = [&](int sl, int n) {
    const uint32_t path = s_path[sl * kTcRows + r];
    T* dst = r < n ? reinterpret_cast<T*>(p.dq_path) + ((int64_t)bh * p.P + path) * D : nullptr;
#pragma unroll
    for (int c0 = part * (D / kTcBwdParts); c0 < (part + 1) * (D / kTcBwdParts); c0 += 16) {
      float x[16];
      tc_ld16(tQ + lane_addr + c0, x);
      if (dst != nullptr) {
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 16; i += 2) pk[i >> 1] = Mma<T>::pack(x[i] * p.scale, x[i + 1] * p.scale);
        uint4* d4 = reinterpret_cast<uint4*>(dst + c0);
        d4[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        d4[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      }
    }
  };
  int prev_slot = -1, prev_n = 0;  // the tile whose dq MMAs are in flight
  for (int64_t t0 = beg; t0 < end; t0 += kTcRows, buf ^= 1, slot = slot == 2 ? 0 : slot + 1) {
    const int n = (int)min((int64_t)kTcRows, end - t0);
    const unsigned char* sQ = sm + G::oQ + buf * G::QT;
    const unsigned char* sG = sm + G::oG + buf * G::QT;
    cp_async_wait_0();  // everything of this tile, and the next tile's paths
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        // K-major over d: 16-column step kk is 32 bytes into atom column kk / 4
        const uint32_t qo = (kk >> 2) * (kTcRows * 128) + (kk & 3) * 32, ko = (kk >> 2) * (LB * 128) + (kk & 3) * 32;
        tc_mma(tS, tc_desc_sw(smem_u32(sQ) + qo, 16, 1024), tc_desc_sw(smem_u32(sK) + ko, 16, 1024), idS,
               kk > 0 ? 1u : 0u);
        tc_mma(tP, tc_desc_sw(smem_u32(sG) + qo, 16, 1024), tc_desc_sw(smem_u32(sV) + ko, 16, 1024), idS,
               kk > 0 ? 1u : 0u);
      }
      tc_commit(mS);
    }
    // while S and dP run: this tile's dz rows as 16-bit high / low parts, and the previous
    // tile's dq rows
    for (int i = tid; i < (kTcRows << zsh); i += blockDim.x) {
      const int rr = i >> zsh, c = i & ((1 << zsh) - 1);
      const float z = s_zraw[i];
      const uint16_t hi = Mma<T>::half_bits(z);
      s_zh[rr * kZLd + c] = hi;
      s_zl[rr * kZLd + c] = Mma<T>::half_bits(z - raw_to_float<T>(hi));
    }
    if (prev_slot >= 0) {
      // (an expired wait here leaves this tile's S / dP in flight too: failed = 1 drains them,
      // and with them everything issued before)
      if (__syncthreads_or(!tc_wait(mD, phD, p.wait_ns))) { failed = 1; break; }
      phD ^= 1u;
      tc_fence_after();
      dq_out(prev_slot, prev_n);
    }
    if (__syncthreads_or(!tc_wait(mS, phS, p.wait_ns))) { failed = 1; break; }
    phS ^= 1u;
    tc_fence_after();
    {
      // w P and dS of this thread's pair over its part of the keys
      const float* sc = reinterpret_cast<const float*>(sm + G::oSC + buf * G::SCAL);
      const uint32_t path = s_path[slot * kTcRows + r];
      int vis = 0;
      if (r < n) {
        const int64_t bnd = p.causal ? (p.row0 + (int64_t)(path / (uint32_t)p.S)) + p.N - p.row_total
                                     : INT64_MAX;
        vis = visible_keys<LB>(bnd, key0);
      }
      const float w = sc[r], dl = sc[kTcRows + r], nlse2 = -sc[2 * kTcRows + r];
#pragma unroll
      for (int c0 = part * (LB / kTcBwdParts); c0 < (part + 1) * (LB / kTcBwdParts); c0 += 16) {
        float sv[16], dv[16];
        tc_ld16x2(tS + lane_addr + c0, tP + lane_addr + c0, sv, dv);
        uint32_t pw[8], pd[8];
        if (c0 + 16 <= vis) {
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            const float p0 = ex2_approx(fmaf(sv[i], sl2, nlse2));
            const float p1 = ex2_approx(fmaf(sv[i + 1], sl2, nlse2));
            pw[i >> 1] = Mma<T>::pack(w * p0, w * p1);
            pd[i >> 1] = Mma<T>::pack(p0 * fmaf(w, dv[i], -dl), p1 * fmaf(w, dv[i + 1], -dl));
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            const float p0 = c0 + i < vis ? ex2_approx(fmaf(sv[i], sl2, nlse2)) : 0.0f;
            const float p1 = c0 + i + 1 < vis ? ex2_approx(fmaf(sv[i + 1], sl2, nlse2)) : 0.0f;
            pw[i >> 1] = Mma<T>::pack(w * p0, w * p1);
            pd[i >> 1] = Mma<T>::pack(p0 * fmaf(w, dv[i], -dl), p1 * fmaf(w, dv[i + 1], -dl));
          }
        }
        const uint32_t o0 = sw128_off(r, c0 >> 3, kTcRows), o1 = sw128_off(r, (c0 >> 3) + 1, kTcRows);
        *reinterpret_cast<uint4*>(sWP + o0) = make_uint4(pw[0], pw[1], pw[2], pw[3]);
        *reinterpret_cast<uint4*>(sWP + o1) = make_uint4(pw[4], pw[5], pw[6], pw[7]);
        *reinterpret_cast<uint4*>(sDS + o0) = make_uint4(pd[0], pd[1], pd[2], pd[3]);
        *reinterpret_cast<uint4*>(sDS + o1) = make_uint4(pd[4], pd[5], pd[6], pd[7]);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      // dq = dS K (K_blk as the MN-major B operand over its key rows)
#pragma unroll
      for (int kk = 0; kk < LB / 16; ++kk)
        tc_mma(tQ, tc_desc_sw(smem_u32(sDS) + (kk >> 2) * (kTcRows * 128) + (kk & 3) * 32, 16, 1024),
               tc_desc_sw(smem_u32(sK) + kk * 2048, LB * 128, 1024), idDQ, kk > 0 ? 1u : 0u);
      // dV += (w P)^T dO, dK += dS^T Q over the tile's pairs (the MMA's K), both operands
      // MN-major over their pair rows
      const int kend = (n + 15) >> 4;
      for (int kk = 0; kk < kend; ++kk) {
        const uint32_t acc = (t0 > beg || kk > 0) ? 1u : 0u;
        // MN-major over the pair rows: 16-row step kk is two 8-row groups (2048 bytes)
        const uint64_t dwp = tc_desc_sw(smem_u32(sWP) + kk * 2048, kTcRows * 128, 1024);
        const uint64_t dds = tc_desc_sw(smem_u32(sDS) + kk * 2048, kTcRows * 128, 1024);
        const uint64_t dgo = tc_desc_sw(smem_u32(sG) + kk * 2048, kTcRows * 128, 1024);
        const uint64_t dq_ = tc_desc_sw(smem_u32(sQ) + kk * 2048, kTcRows * 128, 1024);
        if constexpr (G::KEY_ROWS) {
          tc_mma(tV, dwp, dgo, idKV, acc);
          tc_mma(tK, dds, dq_, idKV, acc);
        } else {
          tc_mma(tV, dgo, dwp, idKV, acc);
          tc_mma(tK, dq_, dds, idKV, acc);
        }
      }
      tc_commit(mD);
    }
    prev_slot = slot;
    prev_n = n;
    // while the tensor cores run: the next tile's reads (its buffers were last read by the
    // previous tile's MMAs, complete), then this tile's summary gradients
    if (t0 + kTcRows < end) gather(t0 + kTcRows, buf ^ 1, slot == 2 ? 0 : slot + 1);
    {
      const int kend = (n + 15) & ~15;
#pragma unroll
      for (int i = 0; i < kTcBwdDcItems; ++i) {
        const int item = warp + kTcBwdWarps * i;
        if (item < zmt * NPAIR) {
          const int zm = (item / NPAIR) * 16, zn = (item % NPAIR) * 16;
          for (int kc = 0; kc < kend; kc += 16) {
            uint32_t ah[4], al[4], bb[4];
            frag_a_t(ah, s_zh, kZLd, zm, kc, lane);
            frag_a_t(al, s_zl, kZLd, zm, kc, lane);
            frag_b_kn_sw(bb, sQ, zn, kc, lane);
            Mma<T>::run(acc_dc[i][0], ah, bb);
            Mma<T>::run(acc_dc[i][0], al, bb);
            Mma<T>::run(acc_dc[i][1], ah, bb + 2);
            Mma<T>::run(acc_dc[i][1], al, bb + 2);
          }
        }
      }
    }
    tc_fence_before();
  }
  if (!failed && prev_slot >= 0) {
    if (__syncthreads_or(!tc_wait(mD, phD, p.wait_ns))) {
      failed = 2;
    } else {
      phD ^= 1u;
      tc_fence_after();
      dq_out(prev_slot, prev_n);
    }
  }
  cp_async_wait_0();
  if (failed) {
    // let the MMAs issued before the expired wait finish before their TMEM is freed
    if (failed == 1) tc_wait(mS, phS, kTcWaitNs);
    else tc_wait(mD, phD, kTcWaitNs);
    if (tid == 0) {
      *p.status = 1;
      __threadfence_system();
    }
  } else {
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // summary partials of this block
    {
      const int g = lane >> 2, tq = lane & 3;
      float* dcp = p.dc_part + ((int64_t)bh * p.nb + j) * DF * D;
#pragma unroll
      for (int i = 0; i < kTcBwdDcItems; ++i) {
        const int item = warp + kTcBwdWarps * i;
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
    // dV (input dtype) and the attention part of dK (float32); zeros for a block no pair reached
    T* dvb = reinterpret_cast<T*>(p.dv) + (int64_t)b * p.dvb + (int64_t)h * p.dvh;
    float* dkb = p.dk_attn + (int64_t)bh * p.N * D;
    const bool any = beg < end;
    if constexpr (G::KEY_ROWS) {
      // lane = key row, columns = head_dim (this warp's part)
      const int64_t key = key0 + r;
#pragma unroll
      for (int c0 = part * (D / kTcBwdParts); c0 < (part + 1) * (D / kTcBwdParts); c0 += 16) {
        float x[16], y[16];
        tc_ld16x2(tV + lane_addr + c0, tK + lane_addr + c0, x, y);
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 16; i += 2) pk[i >> 1] = any ? Mma<T>::pack(x[i], x[i + 1]) : 0u;
        uint4* vd = reinterpret_cast<uint4*>(dvb + key * p.dvs + c0);
        vd[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        vd[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        float4* kd = reinterpret_cast<float4*>(dkb + key * D + c0);
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          kd[i >> 2] = any ? make_float4(y[i] * p.scale, y[i + 1] * p.scale, y[i + 2] * p.scale, y[i + 3] * p.scale)
                           : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
    } else {
      // lane = head_dim column d, TMEM columns = keys (this warp's part)
      const int d = r;
#pragma unroll
      for (int c0 = part * (LB / kTcBwdParts); c0 < (part + 1) * (LB / kTcBwdParts); c0 += 16) {
        float x[16], y[16];
        tc_ld16x2(tV + lane_addr + c0, tK + lane_addr + c0, x, y);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int64_t key = key0 + c0 + i;
          dvb[key * p.dvs + d] = static_cast<T>(any ? x[i] : 0.0f);
          dkb[key * D + d] = any ? y[i] * p.scale : 0.0f;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  __syncwarp();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(G::COLS) : "memory");
}

}  // namespace ta
