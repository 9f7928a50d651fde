// Leaf-block attention forward of the generalised tree on the 5th-generation tensor cores
// (tcgen05 + TMEM), sm_100a, 16-bit inputs.
//
// One CTA of 128 threads per (batch*head, leaf block) walks the block's leaf-sorted
// (query, path) pairs in tiles of 128 -- one pair per thread and per TMEM lane:
//   1. the tile's query rows are gathered into shared memory (cp.async) in the canonical
//      no-swizzle K-major layout (8-row x 16-byte core matrices); K_blk (K-major) and V_blk
//      (MN-major) were staged once the same way;
//   2. one elected thread issues S = Q_g K^T as D/16 tcgen05.mma (M = 128, N = Lb, float32
//      accumulator in TMEM) and commits them to an mbarrier;
//   3. every thread loads its own S row from TMEM (tcgen05.ld 32x32b), applies the scale and
//      its causal mask, and writes exp(s - max) as 16-bit P into shared memory (K-major);
//   4. O = P V as Lb/16 tcgen05.mma (N = D) into a second TMEM range; every thread reads its O
//      row, scales it by w_s / rowsum and stores w_s o_s (input dtype) to the per-path buffer.
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

// Shared memory per CTA, at least 80 KB so that no more than two CTAs share an SM: their two
// 256-column TMEM allocations then always fit the SM's 512 columns and tcgen05.alloc never
// has to wait for another CTA.
template <int LB, int D>
__host__ __device__ constexpr size_t blk_tc_fwd_smem() {
  constexpr size_t need = (size_t)2 * kTcRows * D * 2  // Q tiles (double-buffered)
                          + (size_t)LB * D * 2 * 2     // K_blk, V_blk
                          + (size_t)kTcRows * LB * 2   // P tile
                          + 64;                        // mbarrier, TMEM address, pair range
  return need > (size_t)80 * 1024 ? need : (size_t)80 * 1024;
}

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

// byte offset of element (r, c) of a K-major no-swizzle tile with `cols` columns
__device__ __forceinline__ uint32_t kmaj_off(int r, int c, int cols) {
  return (uint32_t)((r >> 3) * (cols * 16) + (c >> 3) * 128 + (r & 7) * 16 + (c & 7) * 2);
}

template <typename T, int LB, int D>
__global__ void __launch_bounds__(kTcRows) blk_attn_fwd_tc_kernel(const BlkMmaParams p) {
  static_assert(LB % 16 == 0 && D % 16 == 0 && LB + D <= kTcCols, "tile shape");
  extern __shared__ __align__(128) unsigned char tc_smem[];
  unsigned char* s_q0 = tc_smem;                      // 2 x [128 x D] K-major
  unsigned char* s_k = s_q0 + 2 * kTcRows * D * 2;   // [LB x D] K-major
  unsigned char* s_v = s_k + LB * D * 2;             // [LB x D] MN-major (n = d)
  unsigned char* s_p = s_v + LB * D * 2;             // [128 x LB] K-major
  uint64_t* s_bar = reinterpret_cast<uint64_t*>(s_p + kTcRows * LB * 2);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(s_bar + 1);
  int64_t* s_range = reinterpret_cast<int64_t*>(s_bar + 2);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int bh = blockIdx.x / p.nb;
  const int j = blockIdx.x - bh * p.nb;
  const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const uint32_t* keys = p.skeys + (int64_t)bh * p.P;
  const uint32_t* vals = p.svals + (int64_t)bh * p.P;
  const uint32_t mbar = smem_u32(s_bar);
  if (tid < 2) {
    const uint32_t target = (uint32_t)j + tid;
    int64_t lo = 0, hi = p.P;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if (keys[mid] < target) lo = mid + 1; else hi = mid;
    }
    s_range[tid] = lo;
  }
  if (tid == 0) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(mbar) : "memory");
  __syncwarp();  // tcgen05.alloc is .sync.aligned: warp 0 must be converged
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s_tmem)),
                 "r"(kTcCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // K_blk (K-major) and V_blk (MN-major: 16-byte chunk (key k, d-group g) at g*LB*16 + k*16)
  constexpr int CPR = D * 2 / 16;
  for (int i = tid; i < LB * CPR; i += blockDim.x) {
    const int r = i / CPR, c = i - r * CPR;
    const int64_t key = (int64_t)j * LB + r;
    cp_async16(s_k + kmaj_off(r, c * 8, D), p.k + (key * p.ks + (int64_t)b * p.kb + (int64_t)h * p.kh) * 2 + c * 16);
    cp_async16(s_v + c * (LB * 16) + r * 16, p.v + (key * p.vs + (int64_t)b * p.vb + (int64_t)h * p.vh) * 2 + c * 16);
  }
  cp_async_commit();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const uint32_t tS = tmem, tO = tmem + LB;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
  const int64_t beg = s_range[0], end = s_range[1];
  constexpr uint32_t idS = tc_idesc<T>(kTcRows, LB, 0, 0);
  constexpr uint32_t idO = tc_idesc<T>(kTcRows, D, 0, 1);
  uint32_t phase = 0;
  bool failed = false;
  // the query rows of tile t0 go to buffer `buf` (rows past the tile are zero)
  auto gather = [&](int64_t t0, int buf) {
    const int n = (int)min((int64_t)kTcRows, end - t0);
    const int r = tid;
    unsigned char* sq = s_q0 + buf * (kTcRows * D * 2);
    int64_t l = 0;
    if (r < n) l = (int64_t)(vals[t0 + r] / p.S);
    for (int c = 0; c < CPR; ++c) {
      unsigned char* dst = sq + kmaj_off(r, c * 8, D);
      if (r < n) cp_async16(dst, p.q + (l * p.qs + (int64_t)b * p.qb + (int64_t)h * p.qh) * 2 + c * 16);
      else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
    cp_async_commit();
  };
  if (beg < end) gather(beg, 0);
  int buf = 0;
  for (int64_t t0 = beg; t0 < end && !failed; t0 += kTcRows, buf ^= 1) {
    const int n = (int)min((int64_t)kTcRows, end - t0);
    // this thread's pair row
    const int r = tid;
    int64_t path = 0, bnd = INT64_MAX;
    if (r < n) {
      path = vals[t0 + r];
      if (p.causal) bnd = (p.row0 + path / p.S) + p.N - p.row_total;
    }
    const unsigned char* s_q = s_q0 + buf * (kTcRows * D * 2);
    // next tile's rows stream in while this one computes (its buffer was freed by the
    // previous iteration's closing barrier)
    if (t0 + kTcRows < end) {
      gather(t0 + kTcRows, buf ^ 1);
      cp_async_wait_1();
    } else {
      cp_async_wait_0();
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk)
        tc_mma(tS, tc_desc(smem_u32(s_q) + kk * 256, 128, D * 16), tc_desc(smem_u32(s_k) + kk * 256, 128, D * 16),
               idS, kk > 0 ? 1u : 0u);
      tc_commit(mbar);
    }
    // the whole CTA leaves together when any warp's wait expired
    if (__syncthreads_or(!tc_wait(mbar, phase, p.wait_ns))) { failed = true; break; }
    phase ^= 1u;
    tc_fence_after();
    // row max, then P = exp(s - max) (16-bit, K-major) and the row sum; the S row is read from
    // TMEM once when it fits in registers (Lb <= 64), else twice
    const int64_t key0 = (int64_t)j * LB;
    float sum = 0.0f, row_max = -INFINITY;
    if constexpr (LB <= 64) {
      float sv[LB];
#pragma unroll
      for (int c0 = 0; c0 < LB; c0 += 16) tc_ld16(tS + lane_base + c0, sv + c0);
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < LB; ++i) {
        sv[i] = key0 + i > bnd ? -INFINITY : sv[i] * p.scale;
        mx = fmaxf(mx, sv[i]);
      }
      row_max = mx;
#pragma unroll
      for (int c0 = 0; c0 < LB; c0 += 8) {
        uint32_t pk[4];
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const float e0 = (r < n && sv[c0 + i] > -INFINITY) ? expf(sv[c0 + i] - mx) : 0.0f;
          const float e1 = (r < n && sv[c0 + i + 1] > -INFINITY) ? expf(sv[c0 + i + 1] - mx) : 0.0f;
          sum += e0 + e1;
          pk[i >> 1] = Mma<T>::pack(e0, e1);
        }
        *reinterpret_cast<uint4*>(s_p + kmaj_off(r, c0, LB)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
    } else {
      float mx = -INFINITY;
#pragma unroll
      for (int c0 = 0; c0 < LB; c0 += 16) {
        float v[16];
        tc_ld16(tS + lane_base + c0, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float sc = key0 + c0 + i > bnd ? -INFINITY : v[i] * p.scale;
          mx = fmaxf(mx, sc);
        }
      }
      row_max = mx;
#pragma unroll
      for (int c0 = 0; c0 < LB; c0 += 16) {
        float v[16];
        tc_ld16(tS + lane_base + c0, v);
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          const float e0 = (r < n && key0 + c0 + i <= bnd) ? expf(v[i] * p.scale - mx) : 0.0f;
          const float e1 = (r < n && key0 + c0 + i + 1 <= bnd) ? expf(v[i + 1] * p.scale - mx) : 0.0f;
          sum += e0 + e1;
          pk[i >> 1] = Mma<T>::pack(e0, e1);
        }
        *reinterpret_cast<uint4*>(s_p + kmaj_off(r, c0, LB)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        *reinterpret_cast<uint4*>(s_p + kmaj_off(r, c0 + 8, LB)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
#pragma unroll
      for (int kk = 0; kk < LB / 16; ++kk)
        tc_mma(tO, tc_desc(smem_u32(s_p) + kk * 256, 128, LB * 16), tc_desc(smem_u32(s_v) + kk * 256, 128, LB * 16),
               idO, kk > 0 ? 1u : 0u);
      tc_commit(mbar);
    }
    if (__syncthreads_or(!tc_wait(mbar, phase, p.wait_ns))) { failed = true; break; }
    phase ^= 1u;
    tc_fence_after();
    // O row: every lane executes the same tcgen05.ld; only valid rows store
    float w = 0.0f;
    uint4* dst = nullptr;
    if (r < n) {
      const int64_t l = path / p.S, s = path - l * p.S;
      w = p.weights[(((int64_t)l * p.B + b) * p.H + h) * p.S + s] / sum;
      dst = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.path_out) + ((int64_t)bh * p.P + path) * D);
      if (p.lse != nullptr) p.lse[(int64_t)bh * p.P + path] = (row_max + logf(sum)) * kLog2e;
    }
    __syncwarp();
#pragma unroll
    for (int c0 = 0; c0 < D; c0 += 16) {
      float v[16];
      tc_ld16(tO + lane_base + c0, v);
      if (dst != nullptr) {
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 16; i += 2) pk[i >> 1] = Mma<T>::pack(v[i] * w, v[i + 1] * w);
        dst[c0 >> 3] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        dst[(c0 >> 3) + 1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      }
    }
    tc_fence_before();
    __syncthreads();  // TMEM and shared tiles are free for the next tile
    tc_fence_after();
  }
  cp_async_wait_0();
  if (failed) {
    // let the MMA issued before the expired wait finish before its TMEM is freed
    tc_wait(mbar, phase, kTcWaitNs);
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
