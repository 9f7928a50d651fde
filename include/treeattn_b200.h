/*
 * treeattn_b200 -- C ABI of the B200-native stochastic tree-attention kernels.
 *
 * Plain pointers, sizes and a CUDA stream; no torch types. Every entry point returns
 * TA_OK (0) or a TA_ERR_* code and never throws; ta_last_error() gives the message of the
 * last failure on the calling thread. The caller owns every buffer (inputs, outputs and
 * workspace). Kernels are enqueued on `stream` (a cudaStream_t / CUstream; NULL = the
 * legacy default stream) and nothing synchronises the host.
 *
 * Tensor arguments are strided views of a (seq, batch, head, dim) tensor whose `dim` axis
 * is contiguous; ta_layout gives the other three strides in ELEMENTS. Row starts must be
 * 16-byte aligned (dim * element size and every stride * element size multiples of 16).
 * That covers the reference layouts (L,B,H,D) / (K,B,H,D) / (N,B,H,D), the packed-head
 * (L,B,E) views of hierarchical_attention, and the attn-bench bshd layout (B,S,H,D).
 *
 * Per-sample outputs (leaf indices, weights, log-probabilities) are contiguous
 * (L, B, H, S) arrays in the reference's C order; packed path bits are (L, B, H, S, P)
 * bytes with P = ceil(log2(N) / 8) and bit d of the path in byte d/8, bit d%8.
 *
 * Reference interfaces cited as file:line inside the TreeAttention project.
 */
#ifndef TREEATTN_B200_H
#define TREEATTN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TA_ABI_VERSION 1

typedef void* ta_stream_t; /* cudaStream_t */

enum ta_status {
  TA_OK = 0,
  TA_ERR_INVALID = 1,     /* bad shape, pointer, stride or alignment */
  TA_ERR_UNSUPPORTED = 2, /* valid but not implemented (e.g. head_dim too large) */
  TA_ERR_CUDA = 3,        /* a CUDA runtime call or launch failed */
  TA_ERR_WORKSPACE = 4    /* workspace missing or smaller than *_workspace_size() */
};

enum ta_dtype { TA_F32 = 0, TA_F16 = 1, TA_BF16 = 2 };

/* Element strides of a (seq, batch, head, dim) view; dim has stride 1. */
typedef struct ta_layout {
  int64_t seq;
  int64_t batch;
  int64_t head;
} ta_layout;

/* Problem geometry of one tree-attention call (reference names in brackets). */
typedef struct ta_shape {
  int64_t batch;       /* B */
  int64_t num_queries; /* L */
  int64_t num_leaves;  /* N: values are leaves; N-1 internal node keys in heap order */
  int64_t num_heads;   /* H */
  int64_t head_dim;    /* D */
  int64_t num_samples; /* S: sampled root-to-leaf paths per query */
  int32_t dtype;       /* ta_dtype of q, k, v, out and the input-typed gradients */
  float max_logit;     /* node logits are clamped to +-max_logit (_autograd.py:14) */
} ta_shape;

/*
 * The Gumbel stream: torch's CUDA generator as consumed by one exponential_() call per
 * tree depth over numel = L*B*H*S*2 (_autograd.py:188-195; _tree_mha.py:109).
 * Depth d uses philox (seed, offset + d * offset_step); element e of that draw comes from
 * subsequence e % draw_stride, draw (e / draw_stride) / 4, component (e / draw_stride) % 4.
 */
typedef struct ta_rng {
  uint64_t seed;
  uint64_t offset;
  uint64_t offset_step;
  int64_t draw_stride;
} ta_rng;

/* ---- runtime ------------------------------------------------------------------------ */

/* Message of the last failed call on this thread ("" if none). */
const char* ta_last_error(void);

/* TA_ABI_VERSION of the loaded library. */
int32_t ta_abi_version(void);

/*
 * Per-launch timing: while enabled, every kernel the library launches is bracketed by a
 * CUDA event pair on its stream. ta_profile_collect() waits for the recorded launches,
 * writes one "kernel_name launches total_ms" line per kernel into buf (truncated to len),
 * clears the records and returns the full text length. No reference counterpart (the
 * reference's harness times whole calls only, harness.py:207-221).
 */
int ta_profile_enable(int32_t on);
int64_t ta_profile_collect(char* buf, size_t len);

/*
 * SM count and max resident threads per SM of CUDA device `device`: the two numbers
 * torch's distribution kernels size their grid from (inputs of ta_philox_plan).
 */
int ta_device_rng_geometry(int32_t device, int32_t* sm_count, int32_t* max_threads_per_sm);

/*
 * torch's distribution-kernel execution policy for `numel` draws on a device with
 * `sm_count` SMs and `max_threads_per_sm` threads per SM: the philox offset increment of
 * one exponential_() call and its grid stride.
 * Replaces compute_full_draw_rng_config (sample_non_causal_paths.cu:139-156).
 */
int ta_philox_plan(int64_t numel, int32_t sm_count, int32_t max_threads_per_sm,
                   uint64_t* offset_step, int64_t* draw_stride);

/*
 * The Gumbel noise of tree depths depth0 .. depth0+depths-1: out[d * numel + e] is
 * bit-identical to torch.empty(numel, dtype=float32, device=cuda).exponential_().log_().neg_()
 * drawn at generator state (rng->seed, rng->offset + (depth0 + d) * rng->offset_step) -- the
 * per-depth draws of the reference (_autograd.py:188-195). Each philox 4-vector is computed
 * once and feeds the four elements torch's grid-stride loop assigns to it. The result is the
 * `gumbels` input of ta_forward / ta_sample_paths.
 */
int ta_gumbel_fill(float* out, int64_t numel, const ta_rng* rng, int32_t depth0,
                   int32_t depths, ta_stream_t stream);

/*
 * One shard of the draw ta_gumbel_fill makes for a (row_total, batch_total, head_total,
 * row_elems) tensor (rows = queries, row_elems = 2 * samples): out[d][r][b][h][i] (float32,
 * (depths, row_count, batch_count, head_count, row_elems)) is the full draw's element
 * (row0 + r, batch0 + b, head0 + h, i). rng is the plan of the FULL numel, so ranks that
 * each fill their own (query, batch, head) block see exactly the noise of one unsharded call:
 * head/batch sharding with no collective, and the query split of sequence parallelism. The
 * full draw must stay below 2^31 elements. No counterpart in the reference (it is
 * single-GPU); extends the per-depth draws of _autograd.py:188-195.
 */
typedef struct ta_shard {
  int64_t row_total, row0, row_count;
  int64_t batch_total, batch0, batch_count;
  int64_t head_total, head0, head_count;
} ta_shard;
int ta_gumbel_fill_shard(float* out, const ta_rng* rng, const ta_shard* shard, int64_t row_elems,
                         int32_t depth0, int32_t depths, ta_stream_t stream);

/* ---- tree build (A1) ---------------------------------------------------------------- */

/*
 * Internal-node keys from leaf keys: the sequence-axis Haar transform of the attn-bench
 * adapters, op-by-op in the input dtype, global mean dropped, written in the reference's
 * position order (node n <- position n+1). seq_len must be a power of two >= 2.
 * k_leaf: (S, B, H, D) view; k_int: (S-1, B, H, D) view, same dtype.
 * Replaces haar_internal_node_keys (attn_bench/baselines/_treeattn_common.py:54-86).
 */
size_t ta_tree_build_workspace_size(int64_t batch, int64_t seq_len, int64_t num_heads,
                                    int64_t head_dim, int32_t dtype);
int ta_tree_build(int32_t dtype, int64_t batch, int64_t seq_len, int64_t num_heads,
                  int64_t head_dim, const void* k_leaf, ta_layout k_leaf_layout, void* k_int,
                  ta_layout k_int_layout, void* workspace, size_t workspace_bytes,
                  ta_stream_t stream);

/*
 * ta_tree_build / ta_tree_build_backward with a choice of node order. TA_LAYOUT_REFERENCE is
 * the reference's: attn-bench's build returns its coefficients in position order (node n =
 * position n + 1) and the samplers read that array as a heap, so a heap node does not hold
 * its own subtree's summary (_treeattn_common.py:54-86 read by _tree_mha.py:99-121).
 * TA_LAYOUT_TREE puts each coefficient on the heap node of the subtree it summarises:
 * node (depth d, index i) = (mean(left half) - mean(right half)) / 2 of leaves
 * [i * 2^(log2 S - d), (i + 1) * 2^(log2 S - d)), each op rounded to the input dtype. No
 * counterpart in the reference (a semantic fix behind a flag).
 */
enum { TA_LAYOUT_REFERENCE = 0, TA_LAYOUT_TREE = 1 };
int ta_tree_build_ex(int32_t dtype, int64_t batch, int64_t seq_len, int64_t num_heads,
                     int64_t head_dim, const void* k_leaf, ta_layout k_leaf_layout, void* k_int,
                     ta_layout k_int_layout, int32_t node_layout, void* workspace,
                     size_t workspace_bytes, ta_stream_t stream);
int ta_tree_build_backward_ex(int32_t dtype, int64_t batch, int64_t seq_len, int64_t num_heads,
                              int64_t head_dim, const float* dk_int, ta_layout dk_int_layout,
                              void* dk_leaf, ta_layout dk_leaf_layout, int32_t node_layout,
                              void* workspace, size_t workspace_bytes, ta_stream_t stream);

/*
 * ta_tree_build without a workspace, for callers that cannot allocate device memory (a host
 * whose runtime owns all HBM in its own pool, or a C/FFI caller with no device allocator).
 * It has no counterpart in the reference. The scratch is a fixed per-device array of
 * TA_NOALLOC_SCRATCH_BYTES; shapes needing more (ta_tree_build_workspace_size) return
 * TA_ERR_WORKSPACE. It needs no zeroing. The first call on a device does the set-up
 * (looks up the array's address), so make it before any stream capture. Calls that
 * overlap on one device race on the shared scratch: serialise them.
 */
#define TA_NOALLOC_SCRATCH_BYTES ((size_t)8 << 20)
int ta_tree_build_noalloc(int32_t dtype, int64_t batch, int64_t seq_len, int64_t num_heads,
                          int64_t head_dim, const void* k_leaf, ta_layout k_leaf_layout,
                          void* k_int, ta_layout k_int_layout, ta_stream_t stream);

/*
 * Gradient of ta_tree_build: dk_leaf = transpose(Haar) dk_int, computed in float32 and
 * written once in `dtype`. dk_int is float32, (S-1, B, H, D) view.
 * Replaces autograd through haar_internal_node_keys (_treeattn_common.py:54-86).
 */
size_t ta_tree_build_backward_workspace_size(int64_t batch, int64_t seq_len,
                                             int64_t num_heads, int64_t head_dim);
int ta_tree_build_backward(int32_t dtype, int64_t batch, int64_t seq_len, int64_t num_heads,
                           int64_t head_dim, const float* dk_int, ta_layout dk_int_layout,
                           void* dk_leaf, ta_layout dk_leaf_layout, void* workspace,
                           size_t workspace_bytes, ta_stream_t stream);

/* ---- fused forward (A3-A7) ------------------------------------------------------------ */

/*
 * Stochastic non-causal tree attention forward, one launch: per (query, sample) walk the
 * tree drawing the Gumbel noise in-kernel (or reading `gumbels` when it is not NULL:
 * float32 (log2 N, L, B, H, S, 2), e.g. from ta_gumbel_fill), softmax the path
 * log-probabilities over the S samples, and write out[l,b,h] = sum_s w_s v[leaf_s]. Writes
 * leaf (int32, may be NULL), weights (float32, may be NULL), packed path bits (may be NULL)
 * and, when branch_prob is not NULL, the probability of the branch NOT taken at every
 * depth of every path, sigmoid(-sgn s) (float32, 16-byte aligned,
 * [B*H][L*S][ta_branch_prob_stride(N)], head-major), which ta_backward consumes so it never
 * recomputes a node logit. num_leaves must be a power of two >= 2.
 * Replaces _StochasticNonCausalTreeAttention.forward (_autograd.py:647-704), i.e.
 * sample_non_causal_paths_forward + softmax + weighted_value_sum_forward
 * (treeattn_cuda.cpp:479-488).
 */
int ta_forward(const ta_shape* shape, const void* q, ta_layout q_layout, const void* k_int,
               ta_layout k_layout, const void* v, ta_layout v_layout, void* out,
               ta_layout out_layout, const ta_rng* rng, const float* gumbels, int32_t* leaf,
               float* weights, uint8_t* packed_paths, float* branch_prob, ta_stream_t stream);

/* Floats per path row of branch_prob: log2(N) rounded up to a multiple of 4. */
int32_t ta_branch_prob_stride(int64_t num_leaves);

/* ---- fused deterministic backward (A8) -------------------------------------------- */

/*
 * Gradients of ta_forward given its leaf, weights and branch_prob outputs. dq is written in
 * shape->dtype; dk in `dk_dtype` and dv in `dv_dtype` (each TA_F32 for a float32 buffer, e.g.
 * partial gradients that are reduced across ranks afterwards, or shape->dtype). No float atomics: dK/dV are reduced by sorting paths by leaf and summing
 * each node's contributions in a fixed order, so results are bitwise repeatable.
 * The sort of the paths by leaf needs only `leaf`, so it runs on an internal side stream of the
 * calling thread (created on its first call on a device) beside the query pass; `stream` waits
 * for it through an event before the node pass, so all the call's work is ordered before
 * anything enqueued on `stream` afterwards, and the call never blocks the host.
 * Replaces _StochasticNonCausalTreeAttention.backward (_autograd.py:707-860):
 * prepare_non_causal_backward, scatter_weighted_grad_v_forward and
 * accumulate_qk_non_causal_all_depths_prepared_inplace (treeattn_cuda.cpp:479-488).
 */
size_t ta_backward_workspace_size(const ta_shape* shape);
int ta_backward(const ta_shape* shape, const void* q, ta_layout q_layout, const void* k_int,
                ta_layout k_layout, const void* v, ta_layout v_layout, const void* grad_out,
                ta_layout grad_out_layout, const int32_t* leaf, const float* weights,
                const float* branch_prob, void* dq, ta_layout dq_layout, void* dk,
                ta_layout dk_layout, int32_t dk_dtype, void* dv, ta_layout dv_layout,
                int32_t dv_dtype, void* workspace, size_t workspace_bytes, ta_stream_t stream);

/*
 * Coefficient form of the deterministic backward, for callers that form their own per-level
 * coefficients (the causal sampler). `shape->num_samples` is the number of paths per query
 * P/L. For every path p of a head (head-major [b*H+h][l*P/L + j]): keys[p] = path bits (leaf
 * index), vals[p] = l*P/L + j, coef[p][ta_branch_prob_stride(N)] = dLoss/d(q . k[node]) at
 * each level, value_weight[p] = weight of the path's leaf in out. Computes
 *   dq[l] = sum_{p of l, d} coef k[node],  dk[n] = sum_{(p,d) through n} coef q[l(p)],
 *   dv[leaf] = sum_{p ending there} value_weight dO[l(p)]
 * with the same sorted, atomics-free reduction as ta_backward. dk / dv in TA_F32 or the input
 * dtype; workspace: ta_backward_workspace_size(shape).
 */
int ta_backward_coef(const ta_shape* shape, const void* q, ta_layout q_layout, const void* k_int,
                     ta_layout k_layout, const void* grad_out, ta_layout grad_out_layout,
                     const float* coef, const float* value_weight, const uint32_t* keys,
                     const uint32_t* vals, void* dq, ta_layout dq_layout, void* dk,
                     ta_layout dk_layout, int32_t dk_dtype, void* dv, ta_layout dv_layout,
                     int32_t dv_dtype, void* workspace, size_t workspace_bytes,
                     ta_stream_t stream);

/*
 * Process-wide size of the tensor-core node pass's ranges (bf16, head_dim % 32 == 0): each CTA
 * reduces `chunks` consecutive 128-path chunks of a head, carrying open nodes between them, and
 * only nodes cut by a range boundary go through the fix-up. 0 (default) derives it from the
 * shape (about 1184 ranges, at most 32 chunks each); values above 32 are clamped. The
 * summation order, and so the low bits of dK / dV, depend on it. Returns the previous setting.
 */
int32_t ta_backward_set_node_range(int32_t chunks);

/*
 * Process-wide choice of how the non-causal samplers (ta_forward, ta_sample_paths,
 * ta_replay_paths) form the per-level logits q . k_node for 16-bit inputs with head_dim a
 * multiple of 32: 1 (default) = m16n8k16 tensor-core products over a warp's eight queries
 * (exact 16-bit products, float32 sums), 0 = float32 FMA chains on the CUDA cores. The two
 * sum in different orders, so a decision whose scores tie to within float32 rounding may
 * differ. Returns the previous setting. (No reference counterpart: the reference's kernels are
 * scalar.)
 */
int32_t ta_forward_set_tensor_dots(int32_t enable);

/* ---- causal mode (A9) ------------------------------------------------------------- */

/*
 * Causal stochastic sampling for queries [0, L), query t's causal boundary leaf being
 * t + query_offset: pass 1 computes the boundary-path log-masses M[d] and boundary logits
 * s_b[d] of every (b, h) (float32 masses, (L, B, H, 2 log2 N + 1): M[0..log2 N] then
 * s_b[0..log2 N - 1]); pass 2 samples S paths per (b, h), correcting
 * level d's branch log-probabilities to m_child + lp - M[d] when every sample of the query
 * sits on the boundary node. Gumbel draws: one exponential_() of numel B*H*S*2 per (query,
 * level) at rng->offset + (t * log2 N + d) * rng->offset_step (ta_philox_plan of that
 * numel), or `gumbels` (L, log2 N, B, H, S, 2). Writes leaf, weights (softmax over the S
 * paths), out = sum w v[leaf], corrected[t] = number of leading corrected levels, and
 * branch_prob (16-byte aligned) as ta_forward. The corrected prefix runs one CTA per query
 * (B*H*S*8 + B*H*(2 log2 N + 1)*4 bytes of shared memory, at most 200 KiB); the levels after
 * it run per (batch, head) like ta_forward.
 * Replaces _sample_paths_causal (treeattn_torch/_tree_mha.py:125-268) and the stochastic
 * branch of hierarchical_attention (:379-412).
 */
int ta_causal_forward(const ta_shape* shape, int64_t query_offset, const void* q,
                      ta_layout q_layout, const void* k_int, ta_layout k_layout, const void* v,
                      ta_layout v_layout, void* out, ta_layout out_layout, const ta_rng* rng,
                      const float* gumbels, int32_t* leaf, float* weights, float* branch_prob,
                      int32_t* corrected, float* masses, ta_stream_t stream);

/*
 * Backward coefficients of ta_causal_forward for L*(S+1) paths per head (each query's S
 * samples, then its boundary path carrying the gradient of the corrected levels' masses),
 * in the layout ta_backward_coef takes (num_samples = S + 1).
 * Replaces autograd through _sample_paths_causal (treeattn_torch/_tree_mha.py:125-268).
 */
int ta_causal_coefficients(const ta_shape* shape, int64_t query_offset, const void* q,
                           ta_layout q_layout, const void* k_int, ta_layout k_layout,
                           const void* v, ta_layout v_layout, const void* grad_out,
                           ta_layout grad_out_layout, const int32_t* leaf, const float* weights,
                           const float* branch_prob, const int32_t* corrected,
                           const float* masses, float* coef, float* value_weight,
                           uint32_t* keys, uint32_t* vals, ta_stream_t stream);

/* ---- exact mode (A10) ------------------------------------------------------------- */

/*
 * Exact tree attention over all N leaves: log p(leaf) = sum over its path of
 * logsigmoid(+-q . k[node]); non-causal weights exp(log p); causal weights mask leaves
 * n > l + query_offset and softmax over the rest. out[l] = sum_n w_n v_n, optional weights
 * (L, B, H, N) float32. shape->num_samples is ignored; workspace of
 * ta_exact_workspace_size(shape) bytes (queries are processed in blocks that fit it).
 * Replaces _deterministic_attention (treeattn_torch/_tree_mha.py:271-321).
 */
size_t ta_exact_workspace_size(const ta_shape* shape);
int ta_exact_forward(const ta_shape* shape, int32_t causal, int64_t query_offset,
                     const void* q, ta_layout q_layout, const void* k_int, ta_layout k_layout,
                     const void* v, ta_layout v_layout, void* out, ta_layout out_layout,
                     float* weights, void* workspace, size_t workspace_bytes,
                     ta_stream_t stream);

/*
 * Gradients of ta_exact_forward: dq (input dtype) is written; dk and dv are float32 and are
 * written, or added to when `accumulate` is nonzero (so a causal call can add the exact
 * prefix's share). Deterministic: per-query coefficient rows and fixed-order GEMMs.
 * Replaces autograd through _deterministic_attention (_tree_mha.py:271-321).
 */
int ta_exact_backward(const ta_shape* shape, int32_t causal, int64_t query_offset,
                      const void* q, ta_layout q_layout, const void* k_int, ta_layout k_layout,
                      const void* v, ta_layout v_layout, const void* grad_out,
                      ta_layout grad_out_layout, void* dq, ta_layout dq_layout, float* dk,
                      ta_layout dk_layout, float* dv, ta_layout dv_layout, int32_t accumulate,
                      void* workspace, size_t workspace_bytes, ta_stream_t stream);

/* ---- generalised tree: fanout f, leaf blocks of Lb keys -------------------------------- */

/*
 * No counterpart in the reference (its tree is binary with one key per leaf); the benchmark
 * configurations name a fanout and a leaf block. N = leaf_block * fanout^Dp keys; node
 * (d, j) summarises the keys of blocks [j f^(Dp-d), (j+1) f^(Dp-d)) as mean / 2 (float32,
 * levels 1..Dp, ta_blocked_summary_rows rows per head, [B*H][rows][D]). Each of the S paths of
 * a query draws one child per level by Gumbel-max over log_softmax(q . c_children) (causal:
 * children starting beyond the query's bottom-right-aligned boundary row0 + l + N - row_total
 * masked), then attends softmax(softmax_scale q . K_blk^T) V_blk over its leaf block (causal:
 * keys beyond the boundary masked); out = sum_s softmax_s(path log-prob) o_s. At fanout 2,
 * leaf block 1 this is the reference sampler on the TA_LAYOUT_TREE node keys.
 * Noise: philox keyed by the GLOBAL (batch, head, query) of the (row/batch/head)_total problem,
 * element offset + (level * S + s) * f + child, so shards draw exactly what the full call draws;
 * a call consumes Dp * S * f offsets (rounded up to 4). `gumbels` (Dp, L, B, H, S, f) replaces
 * it. The backward is deterministic (sorted per leaf block, no float atomics).
 */
typedef struct ta_blocked {
  int32_t fanout;      /* power of two, 2 .. 16 */
  int32_t leaf_block;  /* power of two, 1 .. 256 */
  int32_t causal;
  float softmax_scale; /* leaf-block attention scale (> 0) */
  int64_t row0, row_total, batch0, batch_total, head0, head_total; /* this call's block */
} ta_blocked;
int64_t ta_blocked_summary_rows(int64_t num_leaves, int32_t fanout, int32_t leaf_block);
int ta_blocked_build(const ta_shape* shape, const ta_blocked* cfg, const void* k,
                     ta_layout k_layout, float* summaries, ta_stream_t stream);
int ta_blocked_gumbel_fill(const ta_shape* shape, const ta_blocked* cfg, const ta_rng* rng,
                           float* out, ta_stream_t stream);
/*
 * Leaf-block attention on the tensor cores (16-bit inputs, head_dim 64 or 128, leaf block 16..128;
 * the backward also needs leaf_block >= 32 and leaf_block * head_dim <= 8192): the forward then
 * takes `path_out` ([B*H][L*S][D] rows of w_s * o_s per path in the input dtype followed by
 * [B*H][L*S] float32 base-2 log-sum-exps of each path's scaled leaf-block scores,
 * B*H*L*S*(D/2+1) floats in all, kept for the backward) and a workspace of
 * ta_blocked_forward_workspace_size bytes; with
 * path_out NULL (or for other shapes) everything runs on the CUDA cores.
 * ta_blocked_uses_tensor_cores tells which.
 */
int32_t ta_blocked_uses_tensor_cores(const ta_shape* shape, const ta_blocked* cfg,
                                     int32_t backward);
/*
 * Process-wide choice of the tensor-core forward: 1 = tcgen05 with TMEM accumulators, 0 =
 * mma.sync, -1 = by shape (the default: tcgen05 at leaf_block 128, mma.sync below, as measured
 * at the benchmark configurations). Returns the previous setting.
 */
int32_t ta_blocked_set_tcgen05(int32_t enable);
/*
 * Process-wide choice of the tensor-core backward for (leaf_block, head_dim) = (128, 64) and
 * (64, 128): 1 = tcgen05 with TMEM accumulators (default), 0 = mma.sync. Other shapes always
 * use mma.sync. Returns the previous setting. (No reference counterpart.)
 */
int32_t ta_blocked_set_tcgen05_backward(int32_t enable);
/*
 * Every mbarrier wait of the tcgen05 kernels is bounded (default 1 s). A CTA whose wait
 * expires records it in a process-wide status word in mapped host memory, waits for its
 * issued MMA, frees its TMEM and returns; that call's results are invalid. The word is read
 * without a device synchronisation: ta_blocked_status returns it (1 = an expired wait since
 * it was last cleared; `clear` != 0 resets it), and the next ta_blocked_forward /
 * ta_blocked_backward returns TA_ERR_CUDA (clearing it) instead of running. The word is set
 * once the failing kernel has run: synchronise its stream first for a definite answer.
 * ta_blocked_set_tc_wait_ns sets the bound in nanoseconds (0 = the 1 s default; returns the
 * previous bound); short bounds exist for testing the status path.
 * (No reference counterpart: the reference has no tensor-core kernels.)
 */
int32_t ta_blocked_status(int32_t clear);
uint64_t ta_blocked_set_tc_wait_ns(uint64_t ns);
size_t ta_blocked_forward_workspace_size(const ta_shape* shape, const ta_blocked* cfg);
int ta_blocked_forward(const ta_shape* shape, const ta_blocked* cfg, const void* q,
                       ta_layout q_layout, const void* k, ta_layout k_layout, const void* v,
                       ta_layout v_layout, const float* summaries, void* out,
                       ta_layout out_layout, const ta_rng* rng, const float* gumbels,
                       int32_t* block, float* weights, float* path_out, void* workspace,
                       size_t workspace_bytes, ta_stream_t stream);
size_t ta_blocked_backward_workspace_size(const ta_shape* shape, const ta_blocked* cfg);
int ta_blocked_backward(const ta_shape* shape, const ta_blocked* cfg, const void* q,
                        ta_layout q_layout, const void* k, ta_layout k_layout, const void* v,
                        ta_layout v_layout, const float* summaries, const void* grad_out,
                        ta_layout grad_out_layout, const int32_t* block, const float* weights,
                        const float* path_out, void* dq, ta_layout dq_layout, void* dk,
                        ta_layout dk_layout, void* dv, ta_layout dv_layout, void* workspace,
                        size_t workspace_bytes, ta_stream_t stream);

/* ---- reference-granularity entry points (treeattn_cuda.cpp:479-488) ---------------- */

/*
 * Sampler only: leaf (int32), raw accumulated log-probabilities (float32) and packed bits.
 * Replaces sample_non_causal_paths_forward (sample_non_causal_paths.cu:160-241).
 */
int ta_sample_paths(const ta_shape* shape, const void* q, ta_layout q_layout,
                    const void* k_int, ta_layout k_layout, const ta_rng* rng,
                    const float* gumbels, int32_t* leaf, float* log_prob,
                    uint8_t* packed_paths, ta_stream_t stream);

/*
 * Replay packed path bits: leaf (int32) and log-probabilities (float32), or, when
 * `softmax` is nonzero, the normalised weights instead of the log-probabilities.
 * Replaces replay_non_causal_paths_forward (replay_non_causal_paths.cu:20-81) and
 * prepare_non_causal_backward (backward_prepare_non_causal.cu:41-124).
 */
int ta_replay_paths(const ta_shape* shape, const void* q, ta_layout q_layout,
                    const void* k_int, ta_layout k_layout, const uint8_t* packed_paths,
                    int32_t softmax, int32_t* leaf, float* log_prob_or_weights,
                    ta_stream_t stream);

/*
 * out[l,b,h] = sum_s w[l,b,h,s] v[clamp(leaf[l,b,h,s], 0, N-1), b, h].
 * Replaces weighted_value_sum_forward (weighted_value_sum.cu:8-143).
 */
int ta_weighted_value_sum(const ta_shape* shape, const void* v, ta_layout v_layout,
                          const int32_t* leaf, const float* weights, void* out,
                          ta_layout out_layout, ta_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* TREEATTN_B200_H */
