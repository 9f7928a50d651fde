// Tree build (sequence-axis Haar transform) and its transpose, sm_100a.
//
// Reference: haar_internal_node_keys (attn_bench/baselines/_treeattn_common.py:54-86).
// Level l pairs positions (i, i + 2^l), i a multiple of 2^(l+1), and writes
// avg = (a + b) / 2 at i and diff = (a - b) / 2 at i + 2^l, every op rounded to the input
// dtype. Position p >= 1 ends up holding the diff of level ctz(p); position 0 (the global
// mean) is dropped, so internal node n is position n + 1.
//
// HBM-streaming design: a thread owns one 16-byte column slice of one (batch, head) and a
// run of 2^lv consecutive positions. It streams the run in position order and keeps a
// carry stack of partial averages (one per level) in registers, emitting each diff as
// soon as its pair completes. Each pass covers 5 levels; the run's average goes to a small
// scratch array that the next pass treats as its input sequence (32x shorter), so the
// whole build is ceil(log2(S) / 5) launches that read the keys once and write the nodes
// once. Consecutive threads own consecutive 16-byte slices of a (position, head) row, so
// every warp access is a contiguous 512-byte span in the bshd layout.
//
// The backward pass runs the same schedule top-down: g_a = (g_avg + g_diff) / 2 and
// g_b = (g_avg - g_diff) / 2, exact in float32, rounded once to the output dtype.

#include "ta_common.cuh"

namespace ta {

constexpr int kRunLog = 5;  // levels per pass
constexpr int kTreeThreads = 256;

__host__ __device__ constexpr int ctz_const(int x) { return (x & 1) ? 0 : 1 + ctz_const(x >> 1); }

struct TreeParams {
  const char* src;  // pass input (dtype for forward, float32 for backward)
  char* dst;        // pass output (forward: scratch dtype averages; backward: next-level grads)
  char* nodes;      // forward: k_int (dtype, written); backward: dk_int (float32, read)
  int64_t ss, sb, sh;  // src strides (elements): position, batch, head
  int64_t ds, db, dh;  // dst strides
  int64_t ns, nb, nh;  // node strides
  int32_t B, H, vecs;  // vecs = 16-byte slices per row
  int64_t count;       // entries of the pass input sequence
  int64_t pos_scale;   // global position of input entry c is c * pos_scale
  int32_t write_dst;   // forward: store run averages (0 on the last pass)
  int32_t tree_layout; // node rows in tree order (TA_LAYOUT_TREE) instead of position order
  int32_t log_s;       // log2 of the sequence length
};

// Row of the node that holds the Haar coefficient at position pos >= 1. Reference layout:
// row pos - 1 (the array attn-bench's build returns, which the samplers read as a heap).
// Tree layout: the coefficient of level l = ctz(pos) pairs the two halves of the block of
// 2^(l+1) positions starting at pos - 2^l, i.e. heap node (depth log_s - 1 - l, index
// pos >> (l + 1)), so every heap node holds (mean(left half) - mean(right half)) / 2 of its
// own subtree.
__device__ __forceinline__ int64_t node_row(const TreeParams& p, int64_t pos) {
  if (!p.tree_layout) return pos - 1;
  const int l = __ffsll(pos) - 1;
  const int d = p.log_s - 1 - l;
  return ((int64_t)1 << d) - 1 + (pos >> (l + 1));
}

// forward: one run of 2^LV entries
template <typename T, int LV>
__global__ void __launch_bounds__(kTreeThreads) haar_fwd_kernel(const TreeParams p) {
  using E = Elem<T>;
  constexpr int EPC = E::EPC;
  constexpr int RUN = 1 << LV;
  const int64_t runs = p.count >> LV;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)p.B * runs * p.H * p.vecs;
  if (tid >= total) return;
  int64_t t = tid;
  const int v = (int)(t % p.vecs); t /= p.vecs;
  const int h = (int)(t % p.H); t /= p.H;
  const int64_t run = t % runs;
  const int b = (int)(t / runs);

  const char* src = p.src + ((int64_t)b * p.sb + (int64_t)h * p.sh) * sizeof(T) + v * 16;
  char* nodes = p.nodes + ((int64_t)b * p.nb + (int64_t)h * p.nh) * sizeof(T) + v * 16;
  const int64_t c0 = run << LV;

  float stack[LV][EPC];
  float cur[EPC];
  // rows are loaded a batch at a time, all loads of a batch issued before its math
  constexpr int BATCH = RUN < 16 ? RUN : 16;
#pragma unroll
  for (int i0 = 0; i0 < RUN; i0 += BATCH) {
  uint4 rows[BATCH];
#pragma unroll
  for (int u = 0; u < BATCH; ++u) rows[u] = ld16_stream(src + (c0 + i0 + u) * p.ss * (int64_t)sizeof(T));
#pragma unroll
  for (int u = 0; u < BATCH; ++u) {
    const int i = i0 + u;
    E::unpack(rows[u], cur);
#pragma unroll
    for (int l = 0; l < LV; ++l) {
      if (((i >> l) & 1) == 0) {
#pragma unroll
        for (int e = 0; e < EPC; ++e) stack[l][e] = cur[e];
        break;
      }
      float diff[EPC];
#pragma unroll
      for (int e = 0; e < EPC; ++e) {
        const float a = stack[l][e], bb = cur[e];
        diff[e] = E::round(E::round(a - bb) * 0.5f);
        cur[e] = E::round(E::round(a + bb) * 0.5f);
      }
      // pair (i - 2^(l+1) + 1, i - 2^l + 1): diff lands on the right block's start
      const int64_t pos = (c0 + i + 1 - (1 << l)) * p.pos_scale;
      st16(nodes + node_row(p, pos) * p.ns * (int64_t)sizeof(T), E::pack(diff));
    }
  }
  }
  if (p.write_dst) {
    char* dst = p.dst + ((int64_t)b * p.db + (int64_t)h * p.dh) * sizeof(T) + v * 16;
    st16(dst + run * p.ds * (int64_t)sizeof(T), E::pack(cur));
  }
}

// backward: expand one run of 2^LV entries from the gradient of its average.
// src = float32 gradients of run averages (NULL on the top pass: zero), dst = float32
// gradients of the pass input entries (or dtype dk_leaf on pass 0 when OUT_T != float).
constexpr int kTreeBwdThreads = 128;
template <typename OUT_T, int LV>
__global__ void __launch_bounds__(kTreeBwdThreads) haar_bwd_kernel(const TreeParams p) {
  using E = Elem<OUT_T>;
  constexpr int RUN = 1 << LV;
  const int64_t runs = p.count >> LV;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  // 16-byte slices of float32 (4 elements); vecs counts float32 slices here
  const int64_t total = (int64_t)p.B * runs * p.H * p.vecs;
  if (tid >= total) return;
  int64_t t = tid;
  const int v = (int)(t % p.vecs); t /= p.vecs;
  const int h = (int)(t % p.H); t /= p.H;
  const int64_t run = t % runs;
  const int b = (int)(t / runs);
  const int64_t c0 = run << LV;

  const char* nodes = p.nodes + ((int64_t)b * p.nb + (int64_t)h * p.nh) * 4 + v * 16;
  float g[LV + 1][4];
  // the diff at position c0 + m (m = 1 .. RUN-1) is used once, by the left child at level
  // ctz(m): load all of them before any math
  float dpre[RUN][4];
#pragma unroll
  for (int m = 1; m < RUN; ++m)
    Elem<float>::unpack(ld16_stream(nodes + node_row(p, (c0 + m) * p.pos_scale) * p.ns * 4), dpre[m]);
  if (p.src != nullptr) {
    const char* src = p.src + ((int64_t)b * p.sb + (int64_t)h * p.sh) * 4 + v * 16;
    Elem<float>::unpack(ld16_stream(src + run * p.ss * 4), g[LV]);
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) g[LV][e] = 0.0f;
  }
  char* dst = p.dst + ((int64_t)b * p.db + (int64_t)h * p.dh) * sizeof(OUT_T) +
              (int64_t)v * 4 * sizeof(OUT_T);
#pragma unroll
  for (int i = 0; i < RUN; ++i) {
    const int top = (i == 0) ? LV - 1 : ctz_const(i);
#pragma unroll
    for (int l = LV - 1; l >= 0; --l) {
      if (l > top) continue;
      if ((i >> l) & 1) {  // right child: the parent's diff sits at position i
#pragma unroll
        for (int e = 0; e < 4; ++e) g[l][e] = (g[l + 1][e] - dpre[i][e]) * 0.5f;
      } else {  // left child: the parent's diff sits at position i + 2^l
#pragma unroll
        for (int e = 0; e < 4; ++e) g[l][e] = (g[l + 1][e] + dpre[i + (1 << l)][e]) * 0.5f;
      }
    }
    char* out = dst + (c0 + i) * p.ds * (int64_t)sizeof(OUT_T);
    if constexpr (sizeof(OUT_T) == 4) {
      st16(out, Elem<float>::pack(g[0]));
    } else {
      uint2 w;
      w.x = E::pack2(g[0][0], g[0][1]);
      w.y = E::pack2(g[0][2], g[0][3]);
      *reinterpret_cast<uint2*>(out) = w;
    }
  }
}

template <typename T>
static void launch_haar_fwd(int lv, const TreeParams& p, cudaStream_t st) {
  TA_PROFILE("tree_build", st);
  const int64_t total = (int64_t)p.B * (p.count >> lv) * p.H * p.vecs;
  const unsigned grid = (unsigned)((total + kTreeThreads - 1) / kTreeThreads);
  switch (lv) {
    case 1: haar_fwd_kernel<T, 1><<<grid, kTreeThreads, 0, st>>>(p); break;
    case 2: haar_fwd_kernel<T, 2><<<grid, kTreeThreads, 0, st>>>(p); break;
    case 3: haar_fwd_kernel<T, 3><<<grid, kTreeThreads, 0, st>>>(p); break;
    case 4: haar_fwd_kernel<T, 4><<<grid, kTreeThreads, 0, st>>>(p); break;
    default: haar_fwd_kernel<T, 5><<<grid, kTreeThreads, 0, st>>>(p); break;
  }
}

template <typename OUT_T>
static void launch_haar_bwd(int lv, const TreeParams& p, cudaStream_t st) {
  TA_PROFILE("tree_build_bwd", st);
  const int64_t total = (int64_t)p.B * (p.count >> lv) * p.H * p.vecs;
  const unsigned grid = (unsigned)((total + kTreeBwdThreads - 1) / kTreeBwdThreads);
  switch (lv) {
    case 1: haar_bwd_kernel<OUT_T, 1><<<grid, kTreeBwdThreads, 0, st>>>(p); break;
    case 2: haar_bwd_kernel<OUT_T, 2><<<grid, kTreeBwdThreads, 0, st>>>(p); break;
    case 3: haar_bwd_kernel<OUT_T, 3><<<grid, kTreeBwdThreads, 0, st>>>(p); break;
    case 4: haar_bwd_kernel<OUT_T, 4><<<grid, kTreeBwdThreads, 0, st>>>(p); break;
    default: haar_bwd_kernel<OUT_T, 5><<<grid, kTreeBwdThreads, 0, st>>>(p); break;
  }
}

// Scratch: run averages (forward, dtype) or their gradients (backward, float32) of every
// pass but the last, each stored [B][H][count][D].
static size_t scratch_bytes(int64_t B, int64_t S, int64_t H, int64_t D) {
  size_t total = 0;
  int64_t count = S;
  while (count > (1 << kRunLog)) {
    count >>= kRunLog;
    total += (size_t)(B * H * count * D) * 4 + 256;
  }
  return total;
}

static int check_tree_args(int32_t dtype, int64_t B, int64_t S, int64_t H, int64_t D) {
  if (dtype != TA_F32 && dtype != TA_F16 && dtype != TA_BF16)
    return fail(TA_ERR_INVALID, "unknown dtype %d", dtype);
  if (B <= 0 || H <= 0 || D <= 0) return fail(TA_ERR_INVALID, "batch, heads and head_dim must be > 0");
  if (S < 2 || (S & (S - 1))) return fail(TA_ERR_INVALID, "seq_len must be a power of two >= 2 (got %lld)", (long long)S);
  if ((D * dtype_size(dtype)) % 16 || D % 4)
    return fail(TA_ERR_UNSUPPORTED, "head_dim * element size must be a multiple of 16 bytes");
  return TA_OK;
}

}  // namespace ta

using namespace ta;

extern "C" size_t ta_tree_build_workspace_size(int64_t B, int64_t S, int64_t H, int64_t D,
                                               int32_t dtype) {
  (void)dtype;
  return scratch_bytes(B, S, H, D);
}

extern "C" size_t ta_tree_build_backward_workspace_size(int64_t B, int64_t S, int64_t H,
                                                        int64_t D) {
  return scratch_bytes(B, S, H, D);
}

extern "C" int ta_tree_build_ex(int32_t dtype, int64_t B, int64_t S, int64_t H, int64_t D,
                                const void* k_leaf, ta_layout kl, void* k_int, ta_layout nl,
                                int32_t node_layout, void* ws, size_t ws_bytes,
                                ta_stream_t stream) {
  int rc = check_tree_args(dtype, B, S, H, D);
  if (rc) return rc;
  if (node_layout != TA_LAYOUT_REFERENCE && node_layout != TA_LAYOUT_TREE)
    return fail(TA_ERR_INVALID, "unknown node layout %d", node_layout);
  const int es = dtype_size(dtype);
  if ((rc = check_view("k_leaf", k_leaf, kl, es, false)) ||
      (rc = check_view("k_int", k_int, nl, es, false)))
    return rc;
  if (ws_bytes < scratch_bytes(B, S, H, D) || (scratch_bytes(B, S, H, D) && !ws))
    return fail(TA_ERR_WORKSPACE, "tree build workspace too small (%zu < %zu)", ws_bytes,
                scratch_bytes(B, S, H, D));
  cudaStream_t st = (cudaStream_t)stream;
  TreeParams p{};
  p.B = (int32_t)B; p.H = (int32_t)H; p.vecs = (int32_t)(D * es / 16);
  p.nodes = (char*)k_int; p.ns = nl.seq; p.nb = nl.batch; p.nh = nl.head;
  p.src = (const char*)k_leaf; p.ss = kl.seq; p.sb = kl.batch; p.sh = kl.head;
  p.count = S;
  p.pos_scale = 1;
  p.tree_layout = node_layout == TA_LAYOUT_TREE;
  p.log_s = floor_log2(S);
  char* scratch = (char*)ws;
  while (true) {
    const int lv = p.count > (1 << kRunLog) ? kRunLog : floor_log2(p.count);
    const int64_t next = p.count >> lv;
    p.write_dst = next > 1;
    if (p.write_dst) {
      p.dst = scratch;
      p.ds = D; p.dh = next * D; p.db = H * next * D;
    }
    switch (dtype) {
      case TA_F32: launch_haar_fwd<float>(lv, p, st); break;
      case TA_F16: launch_haar_fwd<__half>(lv, p, st); break;
      default: launch_haar_fwd<__nv_bfloat16>(lv, p, st); break;
    }
    if ((rc = check_launch("tree build"))) return rc;
    if (!p.write_dst) break;
    scratch += (size_t)(B * H * next * D) * 4 + 256;
    p.src = p.dst; p.ss = p.ds; p.sb = p.db; p.sh = p.dh;
    p.count = next;
    p.pos_scale <<= lv;
  }
  return TA_OK;
}

extern "C" int ta_tree_build(int32_t dtype, int64_t B, int64_t S, int64_t H, int64_t D,
                             const void* k_leaf, ta_layout kl, void* k_int, ta_layout nl,
                             void* ws, size_t ws_bytes, ta_stream_t stream) {
  return ta_tree_build_ex(dtype, B, S, H, D, k_leaf, kl, k_int, nl, TA_LAYOUT_REFERENCE, ws,
                          ws_bytes, stream);
}

extern "C" int ta_tree_build_backward_ex(int32_t dtype, int64_t B, int64_t S, int64_t H,
                                         int64_t D, const float* dk_int, ta_layout nl,
                                         void* dk_leaf, ta_layout ol, int32_t node_layout,
                                         void* ws, size_t ws_bytes, ta_stream_t stream) {
  int rc = check_tree_args(dtype, B, S, H, D);
  if (rc) return rc;
  if (node_layout != TA_LAYOUT_REFERENCE && node_layout != TA_LAYOUT_TREE)
    return fail(TA_ERR_INVALID, "unknown node layout %d", node_layout);
  const int es = dtype_size(dtype);
  if ((rc = check_view("dk_int", dk_int, nl, 4, false)) ||
      (rc = check_view("dk_leaf", dk_leaf, ol, es, false)))
    return rc;
  if (((D * es) % 8) != 0) return fail(TA_ERR_UNSUPPORTED, "head_dim not supported");
  if (ws_bytes < scratch_bytes(B, S, H, D) || (scratch_bytes(B, S, H, D) && !ws))
    return fail(TA_ERR_WORKSPACE, "tree build backward workspace too small");
  cudaStream_t st = (cudaStream_t)stream;
  // pass geometry, bottom-up, so the launches can run top-down
  int64_t counts[16];
  int lvs[16];
  int64_t scales[16];
  size_t offs[16];
  int np = 0;
  {
    int64_t count = S, scale = 1;
    while (true) {
      const int lv = count > (1 << kRunLog) ? kRunLog : floor_log2(count);
      counts[np] = count; lvs[np] = lv; scales[np] = scale;
      ++np;
      const int64_t next = count >> lv;
      if (next <= 1) break;
      count = next;
      scale <<= lv;
    }
    // pass j >= 1 keeps the gradients of its counts[j] input entries at offs[j]
    offs[0] = 0;
    size_t off = 0;
    for (int j = 1; j < np; ++j) {
      offs[j] = off;
      off += (size_t)(B * H * counts[j] * D) * 4 + 256;
    }
  }
  for (int j = np - 1; j >= 0; --j) {
    TreeParams p{};
    p.B = (int32_t)B; p.H = (int32_t)H; p.vecs = (int32_t)(D / 4);
    p.nodes = (char*)dk_int; p.ns = nl.seq; p.nb = nl.batch; p.nh = nl.head;
    p.count = counts[j];
    p.pos_scale = scales[j];
    p.tree_layout = node_layout == TA_LAYOUT_TREE;
    p.log_s = floor_log2(S);
    // gradients of this pass's run averages: produced by pass j+1 (none on the top pass)
    if (j + 1 < np) {
      const int64_t n = counts[j + 1];
      p.src = (const char*)ws + offs[j + 1];
      p.ss = D; p.sh = n * D; p.sb = H * n * D;
    }
    if (j > 0) {  // gradients of this pass's input entries, float32 scratch
      const int64_t n = counts[j];
      p.dst = (char*)ws + offs[j];
      p.ds = D; p.dh = n * D; p.db = H * n * D;
      launch_haar_bwd<float>(lvs[j], p, st);
    } else {
      p.dst = (char*)dk_leaf; p.ds = ol.seq; p.db = ol.batch; p.dh = ol.head;
      switch (dtype) {
        case TA_F32: launch_haar_bwd<float>(lvs[j], p, st); break;
        case TA_F16: launch_haar_bwd<__half>(lvs[j], p, st); break;
        default: launch_haar_bwd<__nv_bfloat16>(lvs[j], p, st); break;
      }
    }
    if ((rc = check_launch("tree build backward"))) return rc;
  }
  return TA_OK;
}

extern "C" int ta_tree_build_backward(int32_t dtype, int64_t B, int64_t S, int64_t H, int64_t D,
                                      const float* dk_int, ta_layout nl, void* dk_leaf,
                                      ta_layout ol, void* ws, size_t ws_bytes,
                                      ta_stream_t stream) {
  return ta_tree_build_backward_ex(dtype, B, S, H, D, dk_int, nl, dk_leaf, ol,
                                   TA_LAYOUT_REFERENCE, ws, ws_bytes, stream);
}
