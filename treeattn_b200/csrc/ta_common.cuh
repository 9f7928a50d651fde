// Shared device/host helpers for the treeattn_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/treeattn_b200.h"

namespace ta {

// ---------------------------------------------------------------------------------------
// error reporting (host)
// ---------------------------------------------------------------------------------------
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int check_launch(const char* what);
int check_view(const char* name, const void* ptr, ta_layout lay, int esize, bool allow_null);
int check_shape(const ta_shape* s, bool need_pow2);
int causal_tail(const ta_shape* shape, const void* q, ta_layout ql, const void* k, ta_layout kl,
                const void* v, ta_layout vl, void* out, ta_layout ol, const ta_rng* rng,
                const float* gumbels, const int32_t* corrected, int32_t* leaf, float* weights,
                float* branch_prob, cudaStream_t st);
int pick_cpl(int nchunks);

// Per-launch CUDA-event timing, enabled by ta_profile_enable(1): a scope records an event
// pair around the launches it encloses on `stream`; ta_profile_collect() aggregates them.
struct ProfScope {
  ProfScope(const char* name, cudaStream_t stream);
  ~ProfScope();
  int slot;
  cudaStream_t stream;
};
#define TA_PROFILE(name, stream) ::ta::ProfScope _ta_prof_##__LINE__(name, stream)

// ---------------------------------------------------------------------------------------
// element types
// ---------------------------------------------------------------------------------------
inline int dtype_size(int32_t dt) { return dt == TA_F32 ? 4 : 2; }

// Rows are moved in 16-byte chunks; a chunk holds EPC elements.
template <typename T> struct Elem;
template <> struct Elem<float> {
  static constexpr int EPC = 4;
  __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
  }
  __device__ __forceinline__ static float round(float x) { return x; }
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr int EPC = 8;
  __device__ __forceinline__ static void unpack2(uint32_t w, float* f) {
    f[0] = __uint_as_float(w << 16);
    f[1] = __uint_as_float(w & 0xffff0000u);
  }
  __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
    unpack2(u.x, f); unpack2(u.y, f + 2); unpack2(u.z, f + 4); unpack2(u.w, f + 6);
  }
  __device__ __forceinline__ static uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
  }
  __device__ __forceinline__ static float round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
};
template <> struct Elem<__half> {
  static constexpr int EPC = 8;
  __device__ __forceinline__ static void unpack2(uint32_t w, float* f) {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    float2 t = __half22float2(h);
    f[0] = t.x; f[1] = t.y;
  }
  __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
    unpack2(u.x, f); unpack2(u.y, f + 2); unpack2(u.z, f + 4); unpack2(u.w, f + 6);
  }
  __device__ __forceinline__ static uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
  }
  __device__ __forceinline__ static float round(float x) {
    return __half2float(__float2half_rn(x));
  }
};

// float -> element type, round to nearest even
template <typename T> __device__ __forceinline__ T to_t(float x);
template <> __device__ __forceinline__ __nv_bfloat16 to_t<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half to_t<__half>(float x) { return __float2half_rn(x); }

// Dot-product step over one 16-byte chunk: acc += sum_e a[e] * b[e] in element order, with
// float32 accumulation. 16-bit types use the sm_100 mixed-precision FMA (bf16/f16 operands,
// f32 accumulate), which is exactly the f32 FMA of the widened operands.
template <typename T> struct Dot;
template <> struct Dot<float> {
  __device__ __forceinline__ static float chunk(const uint4& a, const uint4& b, float acc) {
    acc = fmaf(__uint_as_float(a.x), __uint_as_float(b.x), acc);
    acc = fmaf(__uint_as_float(a.y), __uint_as_float(b.y), acc);
    acc = fmaf(__uint_as_float(a.z), __uint_as_float(b.z), acc);
    acc = fmaf(__uint_as_float(a.w), __uint_as_float(b.w), acc);
    return acc;
  }
};
#define TA_MIXED_FMA2(TYPE)                                                              \
  __device__ __forceinline__ static float fma2(uint32_t a, uint32_t b, float acc) {    \
    asm("{\n .reg .b16 al, ah, bl, bh;\n mov.b32 {al, ah}, %1;\n mov.b32 {bl, bh}, %2;\n" \
        " fma.rn.f32." TYPE " %0, al, bl, %0;\n fma.rn.f32." TYPE " %0, ah, bh, %0;\n}"  \
        : "+f"(acc) : "r"(a), "r"(b));                                                     \
    return acc;                                                                            \
  }                                                                                        \
  __device__ __forceinline__ static float chunk(const uint4& a, const uint4& b, float acc) { \
    acc = fma2(a.x, b.x, acc);                                                             \
    acc = fma2(a.y, b.y, acc);                                                             \
    acc = fma2(a.z, b.z, acc);                                                             \
    acc = fma2(a.w, b.w, acc);                                                             \
    return acc;                                                                            \
  }
template <> struct Dot<__nv_bfloat16> { TA_MIXED_FMA2("bf16") };
template <> struct Dot<__half> { TA_MIXED_FMA2("f16") };
#undef TA_MIXED_FMA2

// (a0, a1) += s * (b0, b1) as one packed float32x2 FMA: the same two correctly rounded
// FMAs as fmaf on each half, in half the instructions.
__device__ __forceinline__ void ffma2(float& a0, float& a1, float s, float b0, float b1) {
  asm("{\n\t.reg .b64 A, B, S;\n\tmov.b64 A, {%0, %1};\n\tmov.b64 B, {%3, %4};\n\t"
      "mov.b64 S, {%2, %2};\n\tfma.rn.f32x2 A, S, B, A;\n\tmov.b64 {%0, %1}, A;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(s), "f"(b0), "f"(b1));
}

// ldmatrix / mma.sync m16n8k16 (bf16 operands, f32 accumulate)
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

__device__ __forceinline__ void mma_f16(float* c, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
template <typename T> struct Mma16;
template <> struct Mma16<__nv_bfloat16> {
  __device__ __forceinline__ static void mma(float* c, const uint32_t* a, const uint32_t* b) { mma_bf16(c, a, b); }
};
template <> struct Mma16<__half> {
  __device__ __forceinline__ static void mma(float* c, const uint32_t* a, const uint32_t* b) { mma_f16(c, a, b); }
};

__device__ __forceinline__ uint32_t word_of(const uint4& u, int j) {
  return j == 0 ? u.x : (j == 1 ? u.y : (j == 2 ? u.z : u.w));
}

// Four dot products per query on the tensor cores, for a warp of eight 4-lane groups (one
// query per group). Lane t of group g holds 16-byte chunks t, t+4, ... of its query's row
// (`qv`) and of the four node rows its query's four paths visit (`kv[path]`). One m16n8k16
// product per 16 features and pair of paths: A rows = (path pair, query) node rows, B columns
// = the eight queries, both taking their k positions from the same (chunk, word) of each lane,
// so row (query g, path t) times column g is the wanted dot (the other 7 columns are unused).
// The wanted entries of group g sit on lane g/2 of that group; four shuffles hand path t's
// logit to lane t. Products of 16-bit values are exact; sums accumulate in float32.
template <typename T, int CPL>
__device__ __forceinline__ float mma_path_dots(const uint4 (&qv)[CPL], const uint4 (&kv)[4][CPL],
                                               int t4, unsigned gmask) {
  // two accumulator sets (even / odd 16-feature steps) halve the dependent MMA chain
  float d01[2][4] = {}, d23[2][4] = {};
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint32_t b[2] = {word_of(qv[i], 2 * half), word_of(qv[i], 2 * half + 1)};
      const uint32_t a01[4] = {word_of(kv[0][i], 2 * half), word_of(kv[1][i], 2 * half),
                               word_of(kv[0][i], 2 * half + 1), word_of(kv[1][i], 2 * half + 1)};
      const uint32_t a23[4] = {word_of(kv[2][i], 2 * half), word_of(kv[3][i], 2 * half),
                               word_of(kv[2][i], 2 * half + 1), word_of(kv[3][i], 2 * half + 1)};
      Mma16<T>::mma(d01[half], a01, b);
      Mma16<T>::mma(d23[half], a23, b);
    }
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    d01[0][e] += d01[1][e];
    d23[0][e] += d23[1][e];
  }
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;
  const int odd = g & 1;
  const int src = (lane & ~3) | (g >> 1);
  const float p0 = __shfl_sync(gmask, odd ? d01[0][1] : d01[0][0], src, 32);
  const float p1 = __shfl_sync(gmask, odd ? d01[0][3] : d01[0][2], src, 32);
  const float p2 = __shfl_sync(gmask, odd ? d23[0][1] : d23[0][0], src, 32);
  const float p3 = __shfl_sync(gmask, odd ? d23[0][3] : d23[0][2], src, 32);
  return t4 == 0 ? p0 : (t4 == 1 ? p1 : (t4 == 2 ? p2 : p3));
}

__device__ __forceinline__ uint4 ldg16(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}
// Streaming load that is not kept in L1 (rows read once).
__device__ __forceinline__ uint4 ld16_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
// Bring the line holding `p` into L1 ahead of its load (no register is written).
__device__ __forceinline__ void prefetch_l1(const void* p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}
// 16-byte load from a shared-memory address (explicit state space, so it always issues as a
// shared-memory load).
__device__ __forceinline__ uint4 lds16_sa(uint32_t saddr) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(saddr));
  return r;
}
__device__ __forceinline__ uint4 lds16(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem));
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(sa), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Levels of a head's tree kept in shared memory by the path-walking kernels: the largest
// T <= log_n whose 2^T - 1 node rows fit in `budget` bytes.
__host__ __device__ inline int smem_tree_levels(int log_n, int row_bytes, int budget) {
  int t = 0;
  while (t < log_n && (((1ll << (t + 1)) - 1) * row_bytes) <= budget) ++t;
  return t;
}
constexpr int kTreeSmemBudget = 64 * 1024;

// Cooperative copy of tree rows [0, rows) of one head into shared memory (all threads of
// the block; completes with the caller's cp_async_wait_0 + __syncthreads).
__device__ __forceinline__ void stage_tree_rows(char* dst, const char* kbase, uint32_t kstride,
                                                int rows, int row_bytes) {
  const int pieces_per_row = row_bytes >> 4;
  const int total = rows * pieces_per_row;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int r = i / pieces_per_row, c = i - r * pieces_per_row;
    cp_async16(dst + (size_t)r * row_bytes + c * 16, kbase + (uint64_t)r * kstride + c * 16);
  }
  cp_async_commit();
}

__device__ __forceinline__ void st16(void* p, const uint4& v) {
  *reinterpret_cast<uint4*>(p) = v;
}

// ---------------------------------------------------------------------------------------
// math shared by forward and backward (accurate libm calls; no fast-math anywhere)
// ---------------------------------------------------------------------------------------
// (logsigmoid(x), logsigmoid(-x)) = (min(0,x) - t, min(0,-x) - t), t = log1p(exp(-|x|)):
// the same expression torch's log_sigmoid kernel evaluates.
__device__ __forceinline__ void log_sigmoid_pair(float x, float& left, float& right) {
  const float t = log1pf(expf(-fabsf(x)));
  left = fminf(0.0f, x) - t;
  right = fminf(0.0f, -x) - t;
}

// The same pair, also returning e = exp(-|x|).
__device__ __forceinline__ void log_sigmoid_pair_e(float x, float& left, float& right, float& e) {
  e = expf(-fabsf(x));
  const float t = log1pf(e);
  left = fminf(0.0f, x) - t;
  right = fminf(0.0f, -x) - t;
}

// σ(-sgn x) for the direction taken (sgn = +1 for direction 0): the probability of the branch
// not taken, exp(min(0, ±x)) / (1 + e) with e = exp(-|x|), i.e. 1 / (1 + e) when the branch not
// taken has the non-negative argument and e / (1 + e) otherwise.
__device__ __forceinline__ float branch_not_taken_prob(float x, int dir, float e) {
  const bool big = dir ? (x >= 0.0f) : (x <= 0.0f);  // argument of the branch not taken >= 0
  return (big ? 1.0f : e) / (1.0f + e);
}

__device__ __forceinline__ float clamp_logit(float x, float m) {
  return x > m ? m : (x < -m ? -m : x);
}

// Path position of a leaf: heap node of the final step is (1 << log_n) - 1 + bits, with
// the direction taken at depth d in bit (log_n - 1 - d) of `bits`.
__device__ __forceinline__ int64_t heap_node(int depth, uint32_t bits, int log_n) {
  return ((int64_t)1 << depth) - 1 + (int64_t)(bits >> (log_n - depth));
}

__host__ __device__ inline int floor_log2(int64_t n) {
  int r = 0;
  while (n > 1) { n >>= 1; ++r; }
  return r;
}

}  // namespace ta
