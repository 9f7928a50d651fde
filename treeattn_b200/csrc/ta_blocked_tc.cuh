// Leaf-block attention forward of the generalised tree on the 5th-generation tensor cores
// (tcgen05 + TMEM), sm_100a, 16-bit inputs.
//
// One CTA of 256 threads per (batch*head, leaf block) walks the block's leaf-sorted
// (query, path) pairs in tiles of 128 -- one pair per TMEM lane; warp w reads lanes
// [32 (w % 4), +32) and column half w / 4. Per tile:
//   1. one elected thread issues S = Q_g K^T as D/16 tcgen05.mma (M = 128, N = Lb, float32
//      accumulator in TMEM) and commits them to an mbarrier;
//   2. while S runs, the previous tile's O rows are read back from TMEM, scaled by
//      w_s / rowsum and stored (input dtype) with the pair's base-2 log-sum-exp;
//   3. the next tile's query rows, w_s and the paths of the tile after it are gathered with
//      cp.async into the other buffers (so no thread waits on a global load);
//   4. the row max of S (the two column halves exchanged through shared memory), then
//      P = 2^(s scale log2(e) - max) as a 16-bit tile in shared memory and its row sums;
//   5. one thread issues O = P V (Lb/16 tcgen05.mma, N = D) into a second TMEM range.
// Operand tiles are 128-byte-swizzled atoms (sw128_off): K-major for Q, K and P, and V_blk
// read as the MN-major operand over its key rows. The pair range of a block comes from the
// per-call table of blk_block_ranges_kernel.
// Descriptor and instruction-descriptor fields follow the sm100 UMMA layout (shared-memory
// descriptor: start >> 4 in [0,14), leading-byte offset >> 4 in [16,30), stride-byte offset
// >> 4 in [32,46), version 1 in [46,48), layout type in [61,64) = 0 for no swizzle; instruction
// descriptor: D format [4,6), A / B format [7,10) / [10,13), A / B major [15] / [16],
// N >> 3 [17,23), M >> 4 [24,29)). Every mbarrier wait is bounded: the CTA agrees on a
// failure (__syncthreads_or), records it in the host-visible status word, waits once more
// (bounded by kTcWaitNs) for the MMA it had issued, frees its TMEM and returns.
#pragma once

#include "ta_blocked_mma.cuh"

namespace ta {

constexpr int kTcRows = 128;         // pairs per tile = MMA M = TMEM lanes
constexpr int kTcCols = 256;         // TMEM columns allocated per CTA (S: Lb, O: D)
constexpr uint64_t kTcWaitNs = 1000000000ull;  // default bound of one mbarrier wait: 1 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// No-swizzle shared-memory matrix descriptor.
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

template <typename T>
__host__ __device__ constexpr uint32_t tc_idesc(int M, int N, int a_mn_major, int b_mn_major) {
  const uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)a_mn_major << 15) |
         ((uint32_t)b_mn_major << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
      :
      : "r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__device__ __forceinline__ void tc_commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar)
               : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait for the mbarrier phase `parity`, at most `limit_ns`; false if it never completed. The
// warp is reconverged on return (the next tcgen05.ld is .sync.aligned).
__device__ __forceinline__ bool tc_wait(uint32_t mbar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t t0 = global_ns();
  bool done = false;
  while (!done) {
    uint32_t ok;
    if (limit_ns >= 1000) {  // try_wait may suspend the thread for a while before it answers
      asm volatile(
          "{\n\t.reg .pred P1;\n\tmbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
          "selp.b32 %0, 1, 0, P1;\n\t}\n"
          : "=r"(ok)
          : "r"(mbar), "r"(parity)
          : "memory");
    } else {  // sub-microsecond bounds (tests of the status path) poll without suspending
      asm volatile(
          "{\n\t.reg .pred P1;\n\tmbarrier.test_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
          "selp.b32 %0, 1, 0, P1;\n\t}\n"
          : "=r"(ok)
          : "r"(mbar), "r"(parity)
          : "memory");
    }
    done = ok != 0;
    if (!done && global_ns() - t0 > limit_ns) break;
  }
  __syncwarp();
  return __all_sync(0xffffffffu, done);
}

// 16 consecutive float32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Two 16-column TMEM reads of this thread's lane and their completion wait in one asm
// statement, so no use of the registers can be scheduled before the wait.
__device__ __forceinline__ void tc_ld16x2(uint32_t a0, uint32_t a1, float* x, float* y) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%32];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%33];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(a0), "r"(a1)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    x[i] = __uint_as_float(r[i]);
    y[i] = __uint_as_float(r[16 + i]);
  }
}

// 2^x with the hardware approximation (inputs are <= 0 up to rounding; -inf gives 0)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Byte offset of 16-byte chunk `c` (columns 8c .. 8c + 7) of row `r` in a 16-bit tile of `rows`
// rows stored as 128-byte-swizzled atoms: atom column c / 8 (64 columns) at (c / 8) * rows * 128,
// 8-row group r / 8 at (r / 8) * 1024, and within an atom chunk c % 8 of row r % 8 at
// (r % 8) * 128 + ((c % 8) ^ (r % 8)) * 16 (the tile base is 1024-byte aligned).
__device__ __forceinline__ uint32_t sw128_off(int r, int c, int rows) {
  return (uint32_t)((c >> 3) * (rows * 128) + (r >> 3) * 1024 + (r & 7) * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// Shared-memory descriptor of a 128-byte-swizzled operand (layout type 2).
__device__ __forceinline__ uint64_t tc_desc_sw(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return tc_desc(saddr, lbo, sbo) | (2ull << 61);
}

// B fragments of two n8 tiles (n0, n0 + 8), k16, from a [k][n] tile of kTcRows rows in the
// swizzled layout above: the same rows and columns as frag_b_kn.
__device__ __forceinline__ void frag_b_kn_sw(uint32_t* r, const unsigned char* base, int n0, int k0, int lane) {
  ldsm4t(r, base + sw128_off(k0 + ((lane >> 3) & 1) * 8 + (lane & 7), (n0 >> 3) + (lane >> 4), kTcRows));
}

// First sorted (query, path) pair of every leaf block of every head: out[bh][j] for j in
// [0, nb], out[bh][nb] = P (one thread per sorted position; each boundary writes the blocks it
// opens, so empty blocks get their successor's start).
static __global__ void __launch_bounds__(256) blk_block_ranges_kernel(const uint32_t* skeys, int64_t P, int nb,
                                                               int64_t HB, uint32_t* out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= HB * (P + 1)) return;
  const int64_t bh = i / (P + 1), x = i - bh * (P + 1);
  const uint32_t* keys = skeys + bh * P;
  const int64_t prev = x > 0 ? (int64_t)keys[x - 1] : -1;
  const int64_t cur = x < P ? (int64_t)keys[x] : (int64_t)nb;
  for (int64_t kk = prev + 1; kk <= cur && kk <= nb; ++kk) out[bh * (nb + 1) + kk] = (uint32_t)x;
}

// Smem geometry of the forward: K_blk and V_blk, two query tiles, the P tile (at least one
// 64-column atom wide), per-tile scalars, the row-max / row-sum exchange between the two
// column halves, the path ring and the barriers; at least 80 KB, so that no more than two CTAs
// share an SM: their two 256-column TMEM allocations then always fit the SM's 512 columns and
// tcgen05.alloc never has to wait for another CTA.
template <int LB, int D>
struct BlkTcFwdGeom {
  static constexpr int PC = LB < 64 ? 64 : LB;            // stored columns of the P tile
  static constexpr size_t KT = (size_t)LB * D * 2;
  static constexpr size_t QT = (size_t)kTcRows * D * 2;
  static constexpr size_t PT = (size_t)kTcRows * PC * 2;
  static constexpr size_t oK = 0, oV = ((KT + 1023) / 1024) * 1024, oQ = 2 * oV, oP = oQ + 2 * QT,
                          oW = oP + PT,                     // [2][128] w_s per tile buffer
                          oMX = oW + 2 * kTcRows * 4,       // [2 halves][128] row max partials
                          oSM = oMX + 2 * kTcRows * 4,      // [2 bufs][2 halves][128] row sums
                          oLM = oSM + 4 * kTcRows * 4,      // [2 bufs][128] row max (base 2)
                          oPATH = oLM + 2 * kTcRows * 4,    // [3][128] path ring
                          oBAR = oPATH + 3 * kTcRows * 4;
  static constexpr size_t NEED = oBAR + 64 + 1024;
  static constexpr size_t SMEM = NEED > (size_t)80 * 1024 ? NEED : (size_t)80 * 1024;
  static constexpr bool OK = LB % 16 == 0 && LB >= 16 && LB <= 128 && (D == 64 || D == 128) &&
                             LB + D <= kTcCols;
};

template <typename T, int LB, int D>
__global__ void __launch_bounds__(256) blk_attn_fwd_tc_kernel(const BlkMmaParams p) {
  using G = BlkTcFwdGeom<LB, D>;
  static_assert(G::OK, "tile shape");
  extern __shared__ __align__(1024) unsigned char tc_raw[];
  unsigned char* sm = tc_raw + ((1024u - (smem_u32(tc_raw) & 1023u)) & 1023u);
  unsigned char* sK = sm + G::oK;
  unsigned char* sV = sm + G::oV;
  unsigned char* sP = sm + G::oP;
  float* s_w = reinterpret_cast<float*>(sm + G::oW);
  float* s_mx = reinterpret_cast<float*>(sm + G::oMX);
  float* s_sum = reinterpret_cast<float*>(sm + G::oSM);
  float* s_lm = reinterpret_cast<float*>(sm + G::oLM);
  uint32_t* s_path = reinterpret_cast<uint32_t*>(sm + G::oPATH);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + G::oBAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 2);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int quad = warp & 3, half = warp >> 2;
  const int bh = blockIdx.x / p.nb;
  const int j = blockIdx.x - bh * p.nb;
  const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const uint32_t* vals = p.svals + (int64_t)bh * p.P;
  const uint32_t mS = smem_u32(bars), mO = smem_u32(bars + 1);
  const int64_t key0 = (int64_t)j * LB;
  const int64_t beg = p.ranges[(int64_t)bh * (p.nb + 1) + j];
  const int64_t end = p.ranges[(int64_t)bh * (p.nb + 1) + j + 1];
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(mS) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(mO) : "memory");
  }
  __syncwarp();  // tcgen05.alloc is .sync.aligned: warp 0 must be converged
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s_tmem)),
                 "r"(kTcCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  auto fetch_paths = [&](int64_t t0, int slot) {
    if (tid < kTcRows) {
      uint32_t* dst = s_path + slot * kTcRows + tid;
      if (t0 + tid < end) cp_async4(dst, vals + t0 + tid);
      else *dst = 0u;
    }
  };
  // K_blk and V_blk in the swizzled layout over (key, d); the first tile's paths
  constexpr int CPR = D * 2 / 16;
  for (int i = tid; i < LB * CPR; i += blockDim.x) {
    const int r = i / CPR, c = i - r * CPR;
    const int64_t key = key0 + r;
    cp_async16(sK + sw128_off(r, c, LB), p.k + (key * p.ks + (int64_t)b * p.kb + (int64_t)h * p.kh) * 2 + c * 16);
    cp_async16(sV + sw128_off(r, c, LB), p.v + (key * p.vs + (int64_t)b * p.vb + (int64_t)h * p.vh) * 2 + c * 16);
  }
  if (beg < end) fetch_paths(beg, 0);
  cp_async_commit();
  // query rows (threads 0-127: chunks [0, CPR/2), 128-255: the rest) and w_s of the tile at t0
  // into buffer `buf`, and the paths of the tile after it; rows past the tile are zero
  auto gather = [&](int64_t t0, int buf, int slot) {
    const int n = (int)min((int64_t)kTcRows, end - t0);
    const int r = tid & (kTcRows - 1), part = tid >> 7;
    unsigned char* dst = sm + G::oQ + buf * G::QT;
    const uint32_t path = s_path[slot * kTcRows + r];
    const int64_t l = (int64_t)(path / (uint32_t)p.S);
    const char* src = p.q + (l * p.qs + (int64_t)b * p.qb + (int64_t)h * p.qh) * 2;
#pragma unroll
    for (int c = part * (CPR / 2); c < (part + 1) * (CPR / 2); ++c) {
      unsigned char* d_ = dst + sw128_off(r, c, kTcRows);
      if (r < n) cp_async16(d_, src + c * 16);
      else *reinterpret_cast<uint4*>(d_) = make_uint4(0, 0, 0, 0);
    }
    if (part == 0) {
      float* w = s_w + buf * kTcRows + r;
      if (r < n) cp_async4(w, p.weights + ((l * p.B + b) * p.H + h) * p.S + ((int64_t)path - l * p.S));
      else *w = 0.0f;
    }
    if (t0 + kTcRows < end) fetch_paths(t0 + kTcRows, slot == 2 ? 0 : slot + 1);
    cp_async_commit();
  };
  cp_async_wait_0();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const uint32_t tS = tmem, tO = tmem + LB;
  const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
  if (beg < end) gather(beg, 0, 0);
  constexpr uint32_t idS = tc_idesc<T>(kTcRows, LB, 0, 0);
  constexpr uint32_t idO = tc_idesc<T>(kTcRows, D, 0, 1);
  constexpr int SC = LB >= 32 ? LB / 2 : LB;  // S columns per half (half 1 idles at Lb = 16)
  const bool s_part = LB >= 32 || half == 0;
  const float sl2 = p.scale * kLog2e;
  const int r = quad * 32 + lane;  // this thread's pair row (TMEM lane)
  uint32_t phS = 0, phO = 0;
  int failed = 0;  // 1: a wait in the tile loop expired (last commit mS), 2: the final O wait
  // O rows of the tile in buffer `pb` / ring slot `sl` with `n` pairs: w_s o_s / rowsum
  // (16-bit) and the pair's base-2 log-sum-exp
  auto o_out = [&](int pb, int sl, int n) {
    const float sum = s_sum[(pb * 2) * kTcRows + r] + s_sum[(pb * 2 + 1) * kTcRows + r];
    const float sc = sum > 0.0f ? s_w[pb * kTcRows + r] / sum : 0.0f;
    const uint32_t path = s_path[sl * kTcRows + r];
    T* dst = r < n ? reinterpret_cast<T*>(p.path_out) + ((int64_t)bh * p.P + path) * D : nullptr;
    if (dst != nullptr && half == 0 && p.lse != nullptr)
      p.lse[(int64_t)bh * p.P + path] = s_lm[pb * kTcRows + r] + __log2f(sum);
#pragma unroll
    for (int c0 = half * (D / 2); c0 < (half + 1) * (D / 2); c0 += 32) {
      float x[16], y[16];
      tc_ld16x2(tO + lane_addr + c0, tO + lane_addr + c0 + 16, x, y);
      if (dst != nullptr) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          pk[i >> 1] = Mma<T>::pack(x[i] * sc, x[i + 1] * sc);
          pk[8 + (i >> 1)] = Mma<T>::pack(y[i] * sc, y[i + 1] * sc);
        }
        uint4* d4 = reinterpret_cast<uint4*>(dst + c0);
        d4[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        d4[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        d4[2] = make_uint4(pk[8], pk[9], pk[10], pk[11]);
        d4[3] = make_uint4(pk[12], pk[13], pk[14], pk[15]);
      }
    }
  };
  int buf = 0, slot = 0, prev_buf = -1, prev_slot = 0, prev_n = 0;
  for (int64_t t0 = beg; t0 < end; t0 += kTcRows, buf ^= 1, slot = slot == 2 ? 0 : slot + 1) {
    const int n = (int)min((int64_t)kTcRows, end - t0);
    const unsigned char* sQ = sm + G::oQ + buf * G::QT;
    cp_async_wait_0();  // this tile's rows and w_s, the next tile's paths
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t qo = (kk >> 2) * (kTcRows * 128) + (kk & 3) * 32, ko = (kk >> 2) * (LB * 128) + (kk & 3) * 32;
        tc_mma(tS, tc_desc_sw(smem_u32(sQ) + qo, 16, 1024), tc_desc_sw(smem_u32(sK) + ko, 16, 1024), idS,
               kk > 0 ? 1u : 0u);
      }
      tc_commit(mS);
    }
    // while S runs: the previous tile's O rows
    if (prev_buf >= 0) {
      if (__syncthreads_or(!tc_wait(mO, phO, p.wait_ns))) { failed = 1; break; }
      phO ^= 1u;
      tc_fence_after();
      o_out(prev_buf, prev_slot, prev_n);
    }
    if (__syncthreads_or(!tc_wait(mS, phS, p.wait_ns))) { failed = 1; break; }
    phS ^= 1u;
    tc_fence_after();
    // the next tile's reads (its buffers and ring slot were last used by the previous tile,
    // read back above)
    if (t0 + kTcRows < end) gather(t0 + kTcRows, buf ^ 1, slot == 2 ? 0 : slot + 1);
    int vis = 0;
    if (r < n) {
      const uint32_t path = s_path[slot * kTcRows + r];
      const int64_t bnd = p.causal ? (p.row0 + (int64_t)(path / (uint32_t)p.S)) + p.N - p.row_total : INT64_MAX;
      vis = visible_keys<LB>(bnd, key0);
    }
    // pass 1: row max over this half of the keys
    float mx = -INFINITY;
    if (s_part) {
#pragma unroll
      for (int c0 = half * SC; c0 < half * SC + SC; c0 += 16) {
        float v[16];
        tc_ld16(tS + lane_addr + c0, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) mx = c0 + i < vis ? fmaxf(mx, v[i]) : mx;
      }
    }
    s_mx[half * kTcRows + r] = mx;
    __syncthreads();
    mx = fmaxf(s_mx[r], s_mx[kTcRows + r]);
    const float nm2 = mx > -INFINITY ? -mx * sl2 : 0.0f;
    // pass 2: P = 2^(s sl2 - max), its row sum, P to the swizzled tile
    float sum = 0.0f;
    if (s_part) {
#pragma unroll
      for (int c0 = half * SC; c0 < half * SC + SC; c0 += 16) {
        float v[16];
        tc_ld16(tS + lane_addr + c0, v);
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          const float e0 = c0 + i < vis ? ex2_approx(fmaf(v[i], sl2, nm2)) : 0.0f;
          const float e1 = c0 + i + 1 < vis ? ex2_approx(fmaf(v[i + 1], sl2, nm2)) : 0.0f;
          sum += e0 + e1;
          pk[i >> 1] = Mma<T>::pack(e0, e1);
        }
        *reinterpret_cast<uint4*>(sP + sw128_off(r, c0 >> 3, kTcRows)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        *reinterpret_cast<uint4*>(sP + sw128_off(r, (c0 >> 3) + 1, kTcRows)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      }
    }
    s_sum[(buf * 2 + half) * kTcRows + r] = sum;
    if (half == 0) s_lm[buf * kTcRows + r] = -nm2;
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      // O = P V (V_blk as the MN-major B operand over its key rows)
#pragma unroll
      for (int kk = 0; kk < LB / 16; ++kk)
        tc_mma(tO, tc_desc_sw(smem_u32(sP) + (kk >> 2) * (kTcRows * 128) + (kk & 3) * 32, 16, 1024),
               tc_desc_sw(smem_u32(sV) + kk * 2048, LB * 128, 1024), idO, kk > 0 ? 1u : 0u);
      tc_commit(mO);
    }
    prev_buf = buf;
    prev_slot = slot;
    prev_n = n;
    tc_fence_before();
  }
  if (!failed && prev_buf >= 0) {
    if (__syncthreads_or(!tc_wait(mO, phO, p.wait_ns))) {
      failed = 2;
    } else {
      phO ^= 1u;
      tc_fence_after();
      o_out(prev_buf, prev_slot, prev_n);
    }
  }
  cp_async_wait_0();
  if (failed) {
    // let the MMAs issued before the expired wait finish before their TMEM is freed
    if (failed == 1) tc_wait(mS, phS, kTcWaitNs);
    else tc_wait(mO, phO, kTcWaitNs);
    if (tid == 0) {
      *p.status = 1;
      __threadfence_system();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  __syncwarp();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcCols) : "memory");
}

}  // namespace ta
