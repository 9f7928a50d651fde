"""CPU restatement of the reference's stochastic tree attention (TEST INFRASTRUCTURE ONLY).

This module is the parity oracle. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it, and only as the
checker or the timed CPU baseline -- never as a product code path.

Everything here is plain numpy in float32 (the accumulation type of the reference's CUDA
path for every input dtype), with the Gumbel noise passed in explicitly so the same
function can be driven by

* Gumbels recorded from the reference itself (golden fixtures, ``tests/golden``), and
* Gumbels drawn from torch's CUDA generator on the GPU box (bit-exact path parity).

Pinned against the reference: ``tests/test_oracle_golden.py`` checks every function below
against fixtures produced by running the reference implementation
(``tests/golden/make_golden.py``).

Reference files (paths inside the TreeAttention project):

* ``packages/treeattn-torch/src/treeattn_torch/_tree_mha.py`` -- the pure-torch op
* ``packages/treeattn-cuda/src/treeattn_cuda/_autograd.py`` -- the autograd op being replaced
* ``packages/attn-bench/src/attn_bench/baselines/_treeattn_common.py`` -- Haar tree build
"""

from __future__ import annotations

import numpy as np

MAX_LOGIT = 1e3


# --------------------------------------------------------------------------------------
# dtype emulation (the Haar build runs op-by-op in the input dtype)
# --------------------------------------------------------------------------------------

def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even); returned as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounding = 0x7FFF + ((u >> 16) & 1)
    r = ((u + rounding) >> 16) << 16
    nan = np.isnan(x)
    out = r.astype(np.uint32).view(np.float32).copy()
    out[nan] = np.nan
    return out


def round_to_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 ``x`` to ``dtype`` ('f32', 'f16', 'bf16') and return float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f32":
        return x
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        return round_to_bf16(x)
    raise ValueError(dtype)


# --------------------------------------------------------------------------------------
# A1: Haar tree build  (_treeattn_common.py:54-86)
# --------------------------------------------------------------------------------------

def haar_internal_node_keys(k_sbhd: np.ndarray, dtype: str = "f32") -> np.ndarray:
    """Restates ``haar_internal_node_keys`` (_treeattn_common.py:54-86).

    ``k_sbhd``: (S, B, H, D) leaf keys (float32 holding values of ``dtype``).
    Per level l: pairs (i, i + 2^l) with i a multiple of 2^(l+1) become
    ``avg = (a + b) / 2`` at i and ``diff = (a - b) / 2`` at i + 2^l, each op rounded to
    ``dtype``. Index 0 (the global mean) is dropped; the result has S-1 rows in the
    reference's in-order position layout (node n <- position n + 1).
    """
    S = k_sbhd.shape[0]
    if S <= 0 or (S & (S - 1)) != 0:
        raise ValueError(f"treeattn requires power-of-two seqlen, got {S}")
    out = np.array(k_sbhd, dtype=np.float32, copy=True)
    levels = S.bit_length() - 1
    for level in range(levels):
        step = 1 << level
        idx1 = np.arange(S >> (level + 1)) * (2 * step)
        idx2 = idx1 + step
        a = out[idx1]
        b = out[idx2]
        avg = round_to_dtype(round_to_dtype(a + b, dtype) / np.float32(2), dtype)
        diff = round_to_dtype(round_to_dtype(a - b, dtype) / np.float32(2), dtype)
        out[idx1] = avg
        out[idx2] = diff
    return out[1:].copy()


def tree_layout_rows(num_leaves: int) -> np.ndarray:
    """Heap row of every position-order coefficient (tree-correct layout, no reference
    counterpart): position p >= 1 with l = ctz(p) holds the level-l pair of the block of
    2^(l+1) leaves starting at p - 2^l, i.e. heap node (depth log2 N - 1 - l, index
    p >> (l + 1)). Returns rows[p - 1] for p = 1 .. N-1."""
    ln = num_leaves.bit_length() - 1
    rows = np.empty(num_leaves - 1, dtype=np.int64)
    for pos in range(1, num_leaves):
        lvl = (pos & -pos).bit_length() - 1
        d = ln - 1 - lvl
        rows[pos - 1] = (1 << d) - 1 + (pos >> (lvl + 1))
    return rows


def tree_layout_node_keys(k_sbhd: np.ndarray, dtype: str = "f32") -> np.ndarray:
    """The Haar build with each coefficient moved to its subtree's heap node."""
    ref = haar_internal_node_keys(k_sbhd, dtype)
    out = np.empty_like(ref)
    out[tree_layout_rows(k_sbhd.shape[0])] = ref
    return out


def haar_internal_node_keys_backward(grad_internal: np.ndarray) -> np.ndarray:
    """Exact (float32) transpose of the Haar build: grad wrt leaf keys.

    avg = (a+b)/2, diff = (a-b)/2  =>  g_a = (g_avg + g_diff)/2, g_b = (g_avg - g_diff)/2,
    applied top-down from the dropped global mean (gradient 0).
    """
    K = grad_internal.shape[0]
    S = K + 1
    g = np.zeros((S,) + grad_internal.shape[1:], dtype=np.float32)
    g[1:] = grad_internal
    levels = S.bit_length() - 1
    for level in reversed(range(levels)):
        step = 1 << level
        idx1 = np.arange(S >> (level + 1)) * (2 * step)
        idx2 = idx1 + step
        g_avg = g[idx1].copy()
        g_diff = g[idx2].copy()
        g[idx1] = (g_avg + g_diff) * np.float32(0.5)
        g[idx2] = (g_avg - g_diff) * np.float32(0.5)
    return g


# --------------------------------------------------------------------------------------
# A3/A4: path sampling with injected Gumbels  (_tree_mha.py:78-122, _autograd.py:141-220)
# --------------------------------------------------------------------------------------

def log_n_of(num_leaves: int) -> int:
    """Tree depth used by the CUDA op: floor(log2 N) (_autograd.py:171)."""
    return max(num_leaves.bit_length() - 1, 0)


def path_bytes(num_leaves: int) -> int:
    """Bytes of packed direction bits per sample (_autograd.py:68-70)."""
    return (log_n_of(num_leaves) + 7) // 8


def log_sigmoid_pair(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(logsigmoid(x), logsigmoid(-x)) as min(0, +-x) - log1p(exp(-|x|)), in float32."""
    x = x.astype(np.float32)
    t = np.log1p(np.exp(-np.abs(x))).astype(np.float32)
    left = (np.minimum(np.float32(0), x) - t).astype(np.float32)
    right = (np.minimum(np.float32(0), -x) - t).astype(np.float32)
    return left, right


def _gather_rows(tree: np.ndarray, nodes: np.ndarray) -> np.ndarray:
    """tree (T,B,H,D), nodes (L,B,H,S) -> (L,B,H,S,D) with tree[nodes[l,b,h,s], b, h]."""
    T, B, H, D = tree.shape
    bidx = np.arange(B)[None, :, None, None]
    hidx = np.arange(H)[None, None, :, None]
    return tree[np.clip(nodes, 0, T - 1), bidx, hidx]


def sample_paths(q: np.ndarray, k: np.ndarray, gumbels: np.ndarray, num_samples: int,
                 max_logit: float = MAX_LOGIT):
    """Gumbel-max path sampling (non-causal).

    q (L,B,H,D) float32, k (K,B,H,D) float32 in heap order, gumbels
    (log_n, L, B, H, S, 2) float32 (index 0 = left / direction 0, 1 = right).
    Per depth: s = clamp(q . k[node], +-max_logit); lp = [logsig(s), logsig(-s)];
    dir = 1 iff lp_R + G_R > lp_L + G_L (argmax ties resolve left); lp_acc += lp[dir];
    node = 2 node + 1 + dir.  Returns (leaf int64, log_prob float32, packed uint8).
    """
    L, B, H, D = q.shape
    K = k.shape[0]
    N = K + 1
    log_n = log_n_of(N)
    node = np.zeros((L, B, H, num_samples), dtype=np.int64)
    lp = np.zeros((L, B, H, num_samples), dtype=np.float32)
    packed = np.zeros((L, B, H, num_samples, path_bytes(N)), dtype=np.uint8)
    q32 = q.astype(np.float32)
    k32 = k.astype(np.float32)
    for depth in range(log_n):
        kn = _gather_rows(k32, node)
        dots = np.einsum("lbhd,lbhsd->lbhs", q32, kn, dtype=np.float32)
        dots = np.clip(dots, -max_logit, max_logit).astype(np.float32)
        left, right = log_sigmoid_pair(dots)
        g = gumbels[depth]
        sl = (left + g[..., 0]).astype(np.float32)
        sr = (right + g[..., 1]).astype(np.float32)
        direction = (sr > sl).astype(np.int64)
        lp = (lp + np.where(direction == 1, right, left)).astype(np.float32)
        packed[..., depth >> 3] |= (direction << (depth & 7)).astype(np.uint8)
        node = 2 * node + 1 + direction
    return node - K, lp, packed


def replay_paths(q: np.ndarray, k: np.ndarray, packed: np.ndarray, max_logit: float = MAX_LOGIT):
    """Rebuild (leaf, log_prob) from packed direction bits (_autograd.py:260-314)."""
    L, B, H, S, _ = packed.shape
    K = k.shape[0]
    log_n = log_n_of(K + 1)
    node = np.zeros((L, B, H, S), dtype=np.int64)
    lp = np.zeros((L, B, H, S), dtype=np.float32)
    for depth in range(log_n):
        kn = _gather_rows(k.astype(np.float32), node)
        dots = np.clip(np.einsum("lbhd,lbhsd->lbhs", q.astype(np.float32), kn, dtype=np.float32),
                       -max_logit, max_logit)
        left, right = log_sigmoid_pair(dots)
        direction = ((packed[..., depth >> 3] >> (depth & 7)) & 1).astype(np.int64)
        lp = (lp + np.where(direction == 1, right, left)).astype(np.float32)
        node = 2 * node + 1 + direction
    return node - K, lp


def softmax_log_probs(lp: np.ndarray) -> np.ndarray:
    """lp - logsumexp(lp) then exp, over the sample axis (_autograd.py:495-498)."""
    m = lp.max(axis=-1, keepdims=True)
    lse = m + np.log(np.exp(lp - m).sum(axis=-1, keepdims=True))
    return np.exp(lp - lse).astype(np.float32)


def weighted_value_sum(v: np.ndarray, leaf: np.ndarray, w: np.ndarray) -> np.ndarray:
    """out[l,b,h] = sum_s w[l,b,h,s] v[clamp(leaf), b, h] (weighted_value_sum.cu:8-47)."""
    N = v.shape[0]
    gathered = _gather_rows(v.astype(np.float32), np.clip(leaf, 0, N - 1))
    return np.einsum("lbhs,lbhsd->lbhd", w.astype(np.float32), gathered, dtype=np.float32)


# --------------------------------------------------------------------------------------
# A7: forward  (_autograd.py:647-704)
# --------------------------------------------------------------------------------------

def forward(q, k, v, gumbels, num_samples, max_logit=MAX_LOGIT):
    """Stochastic non-causal forward on (L,B,H,D) arrays.

    Returns dict(out (L,B,H,D) f32, weights (L,B,H,S) f32, leaf, log_prob, packed).
    """
    leaf, lp, packed = sample_paths(q, k, gumbels, num_samples, max_logit)
    w = softmax_log_probs(lp)
    out = weighted_value_sum(v, leaf, w)
    return dict(out=out, weights=w, leaf=leaf, log_prob=lp, packed=packed)


# --------------------------------------------------------------------------------------
# A8: analytic backward  (_autograd.py:707-860)
# --------------------------------------------------------------------------------------

def _scatter_rows(dst: np.ndarray, rows: np.ndarray, coef: np.ndarray, src: np.ndarray) -> None:
    """dst[rows[l,b,h,s], b, h] += coef[l,b,h,s] * src[l,b,h] (repeated rows summed, float64).

    Per (b, h) this is a sparse (rows x L) matrix times src, so scipy's sparse product does the
    scatter: the same totals as np.add.at up to summation order, fast at 10^6 paths.
    """
    from scipy import sparse

    L, B, H, S = rows.shape
    T = dst.shape[0]
    lidx = np.broadcast_to(np.arange(L)[:, None], (L, S)).ravel()
    for b in range(B):
        for h in range(H):
            m = sparse.csr_matrix((coef[:, b, h].astype(np.float64).ravel(),
                                   (rows[:, b, h].ravel(), lidx)), shape=(T, L))
            dst[:, b, h] += m @ src[:, b, h].astype(np.float64)


def backward(q, k, v, grad_out, leaf, w, max_logit=MAX_LOGIT):
    """Analytic gradients of the stochastic forward (Gumbels are constants).

    g_s = dO . v[leaf_s];  dlp_s = w_s (g_s - sum_t w_t g_t);  dV[leaf_s] += w_s dO;
    per depth: gl = sgn * sigmoid(-sgn * s) * dlp (sgn = +1 for direction 0),
    dq += gl k[node], dk[node] += gl q.  Returns (dq, dk, dv) float32.
    """
    L, B, H, D = q.shape
    K = k.shape[0]
    N = K + 1
    log_n = log_n_of(N)
    q32, k32, v32 = (x.astype(np.float32) for x in (q, k, v))
    do32 = grad_out.astype(np.float32)
    S = leaf.shape[-1]
    leaf_c = np.clip(leaf, 0, N - 1)
    vg = _gather_rows(v32, leaf_c)
    g = np.einsum("lbhd,lbhsd->lbhs", do32, vg, dtype=np.float32)
    dlp = (w * (g - (w * g).sum(-1, keepdims=True))).astype(np.float32)

    dv = np.zeros((N, B, H, D), dtype=np.float64)
    _scatter_rows(dv, leaf_c, w, do32)

    dq = np.zeros((L, B, H, D), dtype=np.float64)
    dk = np.zeros((max(K, 1), B, H, D), dtype=np.float64)
    node_final = leaf + K
    node = np.zeros_like(leaf)
    for depth in range(log_n):
        bit = (node_final + 1) >> (log_n - 1 - depth) & 1
        kn = _gather_rows(k32, node)
        s = np.clip(np.einsum("lbhd,lbhsd->lbhs", q32, kn, dtype=np.float32), -max_logit, max_logit)
        sgn = np.where(bit == 0, 1.0, -1.0)
        gl = sgn * (1.0 / (1.0 + np.exp(sgn * s.astype(np.float64)))) * dlp
        dq += (gl[..., None] * kn).sum(axis=-2)
        _scatter_rows(dk, node, gl, q32)
        node = 2 * node + 1 + bit
    return dq.astype(np.float32), dk[:K].astype(np.float32), dv.astype(np.float32)


def path_bits_from_leaf(leaf: np.ndarray, num_leaves: int) -> np.ndarray:
    """Packed direction bytes recovered from a leaf index (power-of-two N)."""
    log_n = log_n_of(num_leaves)
    out = np.zeros(leaf.shape + (path_bytes(num_leaves),), dtype=np.uint8)
    for depth in range(log_n):
        bit = (leaf >> (log_n - 1 - depth)) & 1
        out[..., depth >> 3] |= (bit << (depth & 7)).astype(np.uint8)
    return out


# --------------------------------------------------------------------------------------
# Drop-in adapter level (bshd): Haar build + attention  (baselines/treeattn_torch.py:48-90)
# --------------------------------------------------------------------------------------

def adapter_forward_backward(q_bshd, k_bshd, v_bshd, grad_out_bshd, gumbels, num_samples,
                             dtype="f32", max_logit=MAX_LOGIT, node_layout="reference"):
    """fn(q,k,v) of the attn-bench adapter, with its backward.

    Inputs are float32 arrays holding ``dtype`` values, layout (B,S,H,D).
    Returns dict(out, dq, dk, dv, weights, leaf) in bshd (out rounded to ``dtype``).
    ``node_layout="tree"`` uses the tree-correct node order (no reference counterpart).
    """
    q = np.transpose(q_bshd, (1, 0, 2, 3))
    k = np.transpose(k_bshd, (1, 0, 2, 3))
    v = np.transpose(v_bshd, (1, 0, 2, 3))
    k_int = haar_internal_node_keys(k, dtype)
    rows = tree_layout_rows(k.shape[0]) if node_layout == "tree" else None
    if rows is not None:
        k_int = k_int[np.argsort(rows)]
    fw = forward(q, k_int, v, gumbels, num_samples, max_logit)
    do = np.transpose(grad_out_bshd, (1, 0, 2, 3))
    dq, dk_int, dv = backward(q, k_int, v, do, fw["leaf"], fw["weights"], max_logit)
    if rows is not None:
        dk_int = dk_int[rows]
    dk = haar_internal_node_keys_backward(dk_int)
    t = lambda x: np.ascontiguousarray(np.transpose(x, (1, 0, 2, 3)))  # noqa: E731
    return dict(out=t(round_to_dtype(fw["out"], dtype)), dq=t(dq), dk=t(dk), dv=t(dv),
                weights=fw["weights"], leaf=fw["leaf"])


def adapter_forward_backward_given_leaves(q_bshd, k_bshd, v_bshd, grad_out_bshd, leaf, dtype="f32",
                                          max_logit=MAX_LOGIT):
    """``adapter_forward_backward`` along given sampled leaves (L,B,H,S) instead of noise.

    The path log-probabilities are replayed from the leaves' direction bits
    (_autograd.py:260-314), so out and dq/dk/dv are the reference's values for exactly those
    paths. Used to check values independently of near-tie decisions at large sizes.
    """
    q = np.transpose(q_bshd, (1, 0, 2, 3))
    k = np.transpose(k_bshd, (1, 0, 2, 3))
    v = np.transpose(v_bshd, (1, 0, 2, 3))
    k_int = haar_internal_node_keys(k, dtype)
    leaf = np.asarray(leaf, np.int64)
    rl, lp = replay_paths(q, k_int, path_bits_from_leaf(leaf, v.shape[0]), max_logit)
    assert np.array_equal(rl, leaf)
    w = softmax_log_probs(lp)
    out = weighted_value_sum(v, leaf, w)
    do = np.transpose(grad_out_bshd, (1, 0, 2, 3))
    dq, dk_int, dv = backward(q, k_int, v, do, leaf, w, max_logit)
    dk = haar_internal_node_keys_backward(dk_int)
    t = lambda x: np.ascontiguousarray(np.transpose(x, (1, 0, 2, 3)))  # noqa: E731
    return dict(out=t(round_to_dtype(out, dtype)), dq=t(dq), dk=t(dk), dv=t(dv), weights=w,
                k_int=k_int)


# --------------------------------------------------------------------------------------
# A10: deterministic (exact) tree attention  (_tree_mha.py:271-321)
# --------------------------------------------------------------------------------------

def leaf_log_probs(q, k):
    """log p(leaf n | q) = sum over the path's levels of logsigmoid(+-q.k[node]) (power-of-two N).

    q (L,B,H,D), k (K,B,H,D) -> (L,B,H,N) float32, leaves in index order (_tree_mha.py:285-306).
    """
    L, B, H, D = q.shape
    K = k.shape[0]
    N = K + 1
    log_n = log_n_of(N)
    dots = np.einsum("lbhd,kbhd->lbhk", q.astype(np.float32), k.astype(np.float32),
                     dtype=np.float32)
    lp = np.zeros((L, B, H, 1), dtype=np.float32)
    for d in range(log_n):
        s = dots[..., (1 << d) - 1:(1 << (d + 1)) - 1]          # nodes of level d in order
        left, right = log_sigmoid_pair(s)
        lp = np.stack([lp + left, lp + right], axis=-1).reshape(L, B, H, -1).astype(np.float32)
    return lp


def deterministic_attention(q, k, v, is_causal, query_offset=0):
    """Exact attention over all N root-to-leaf paths (_tree_mha.py:271-321).

    Non-causal: weights = exp(log p(leaf)); causal: leaves n > l + query_offset masked, then
    softmax over the leaves. Returns (out (L,B,H,D) f32, weights (L,B,H,N) f32).
    """
    lp = leaf_log_probs(q, k)
    L = q.shape[0]
    N = lp.shape[-1]
    if is_causal:
        mask = np.arange(N)[None, :] > (np.arange(L)[:, None] + query_offset)
        lp = np.where(mask[:, None, None, :], -np.inf, lp)
        m = lp.max(-1, keepdims=True)
        e = np.exp(lp - m)
        w = (e / e.sum(-1, keepdims=True)).astype(np.float32)
    else:
        w = np.exp(lp).astype(np.float32)
    out = np.einsum("lbhn,nbhd->lbhd", w, v.astype(np.float32), dtype=np.float32)
    return out, w


# --------------------------------------------------------------------------------------
# A9: causal sampler  (_tree_mha.py:125-268)
# --------------------------------------------------------------------------------------

def _lse2(a, b):
    m = np.maximum(a, b)
    m_safe = np.where(np.isfinite(m), m, 0.0)
    return (m_safe + np.log(np.exp(a - m_safe) + np.exp(b - m_safe))).astype(np.float32)


def boundary_log_masses(q_t, k, boundary, log_n):
    """Pass 1 of the causal sampler for one query: masses M[d] along the boundary path.

    q_t (B,H,D); returns (nodes [log_n], M (B,H,log_n+1) with M[log_n] = 0, dots (B,H,log_n)).
    M[d] = logsumexp(M[d+1] + lp_on, off_mass + lp_off) where the off-path child is masked
    (-inf) when the boundary goes left, and counts log(#leaves of the left subtree) when it
    goes right (_tree_mha.py:145-196).
    """
    nodes = []
    node = 0
    for d in range(log_n):
        nodes.append(node)
        node = 2 * node + 1 + ((boundary >> (log_n - 1 - d)) & 1)
    kb = k[nodes].astype(np.float32)                       # (log_n, B, H, D)
    dots = np.einsum("bhd,pbhd->bhp", q_t.astype(np.float32), kb, dtype=np.float32)
    B, H = q_t.shape[:2]
    M = np.zeros((B, H, log_n + 1), dtype=np.float32)
    for d in range(log_n - 1, -1, -1):
        direction = (boundary >> (log_n - 1 - d)) & 1
        left, right = log_sigmoid_pair(dots[..., d])
        if direction == 0:
            on, off, off_mass = left, right, np.float32(-np.inf)
        else:
            on, off = right, left
            off_mass = np.float32(np.log(np.float32(1 << (log_n - 1 - d))))
        M[..., d] = _lse2(M[..., d + 1] + on, off_mass + off)
    return nodes, M, dots


def sample_paths_causal(q, k, gumbels, num_samples, causal_offset=0):
    """Causal Gumbel-max sampling with the reference's two-pass boundary correction.

    q (L,B,H,D), k (K,B,H,D); gumbels (L, log_n, B, H, S, 2) float32 -- one draw per (query,
    level) as the reference draws them (_tree_mha.py:255). The correction of level d applies
    only when EVERY (b, h, s) sample sits on the boundary node (_tree_mha.py:204-207).
    Returns (leaf (L,B,H,S), log_prob (L,B,H,S), corrected_levels (L,) int).
    """
    L, B, H, D = q.shape
    K = k.shape[0]
    N = K + 1
    log_n = log_n_of(N)
    S = num_samples
    bidx = np.arange(B)[:, None, None]
    hidx = np.arange(H)[None, :, None]
    leaves = np.zeros((L, B, H, S), dtype=np.int64)
    lps = np.zeros((L, B, H, S), dtype=np.float32)
    ncorr = np.zeros(L, dtype=np.int64)
    k32 = k.astype(np.float32)
    for t in range(L):
        boundary = t + causal_offset
        bnodes, M, _ = boundary_log_masses(q[t], k, boundary, log_n)
        node = np.zeros((B, H, S), dtype=np.int64)
        acc = np.zeros((B, H, S), dtype=np.float32)
        corr = 0
        for d in range(log_n):
            on_path = bool(np.all(node == bnodes[d]))
            kn = k32[node, bidx, hidx]                           # (B,H,S,D)
            s = np.einsum("bhd,bhsd->bhs", q[t].astype(np.float32), kn, dtype=np.float32)
            left, right = log_sigmoid_pair(s)
            if on_path:
                corr = d + 1
                bdir = (boundary >> (log_n - 1 - d)) & 1
                parent = M[..., d][..., None]
                child = M[..., d + 1][..., None]
                if bdir == 0:
                    m_left, m_right = child, np.float32(-np.inf)
                else:
                    m_left = np.float32(np.log(np.float32(1 << (log_n - 1 - d))))
                    m_right = child
                left = (m_left + left - parent).astype(np.float32)
                right = (m_right + right - parent).astype(np.float32)
            g = gumbels[t, d]
            direction = ((right + g[..., 1]) > (left + g[..., 0])).astype(np.int64)
            acc = (acc + np.where(direction == 1, right, left)).astype(np.float32)
            node = 2 * node + 1 + direction
        leaves[t] = node - K
        lps[t] = acc
        ncorr[t] = corr
    return leaves, lps, ncorr


def causal_attention(q, k, v, gumbels, num_samples):
    """hierarchical_attention(..., is_causal=True, mode='stochastic') (_tree_mha.py:379-412).

    L > S: the first S queries take exact causal attention, the rest are sampled with causal
    offset S (gumbels then cover only those L - S queries). Returns dict(out, weights, leaf).
    """
    L = q.shape[0]
    S = num_samples
    hybrid = L > S
    if hybrid:
        out_det, _ = deterministic_attention(q[:S], k, v, True)
        leaf, lp, _ = sample_paths_causal(q[S:], k, gumbels, S, causal_offset=S)
    else:
        leaf, lp, _ = sample_paths_causal(q, k, gumbels, S, causal_offset=0)
    N = v.shape[0]
    lp = np.where((leaf >= 0) & (leaf < N), lp, -np.inf)
    m = lp.max(-1, keepdims=True)
    e = np.exp(lp - m)
    w = (e / e.sum(-1, keepdims=True)).astype(np.float32)
    out_sto = weighted_value_sum(v, leaf, w)
    out = np.concatenate([out_det, out_sto], axis=0) if hybrid else out_sto
    return dict(out=out, weights=w, leaf=leaf)
