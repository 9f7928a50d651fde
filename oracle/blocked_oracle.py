"""CPU restatement of the generalised (fanout f, leaf block Lb) tree attention.

TEST INFRASTRUCTURE ONLY (same rules as ``oracle/tree_oracle.py``): tests import it as the
checker; no product path calls it.

PARITY UNPINNED: the reference has no fanout or leaf-block knob (its tree is binary with one
token per leaf), so nothing in the reference pins this mode. What does pin it: at f = 2,
Lb = 1 it is the reference's sampler on the tree-correct node layout (child logits differ by
q . (mean_L - mean_R) / 2, so the softmax over two children is the reference's
(logsigmoid(q.k), logsigmoid(-q.k)) pair, _tree_mha.py:99-121), and a one-key leaf block returns
that key's value; ``tests/test_blocked_oracle.py`` checks that reduction against
``tree_oracle``.

Semantics (N keys, Lb keys per leaf block, nb = N / Lb blocks = f^Dp):

* node (d, j), d = 0..Dp, covers blocks [j f^(Dp-d), (j+1) f^(Dp-d)); its summary is
  c(d, j) = mean of its keys / 2 (float32);
* per sampled path, from the root: children logits z_i = q . c(d+1, f j + i); causal queries
  mask children whose first key lies beyond the boundary; lsm = log_softmax(z over unmasked);
  dir = argmax(lsm + G) (first maximum); lp += lsm[dir]; j = f j + dir;
* at the leaf block: a_k = softmax_scale * q . k_k over its keys (causal: keys beyond the
  boundary masked), o = softmax(a) @ V_block;
* out = sum_s softmax_s(lp)_s o_s.

The causal boundary of query l of L (bottom-right aligned) is l + N - L.
"""

from __future__ import annotations

import numpy as np


def depth_of(num_keys: int, fanout: int, leaf_block: int) -> int:
    """Dp with num_keys = leaf_block * fanout^Dp (ValueError otherwise)."""
    if fanout < 2 or fanout & (fanout - 1):
        raise ValueError("fanout must be a power of two >= 2")
    if leaf_block < 1 or leaf_block & (leaf_block - 1):
        raise ValueError("leaf_block must be a power of two >= 1")
    if num_keys % leaf_block:
        raise ValueError("num_keys must be a multiple of leaf_block")
    nb = num_keys // leaf_block
    dp = 0
    while fanout ** dp < nb:
        dp += 1
    if fanout ** dp != nb:
        raise ValueError(f"num_keys / leaf_block = {nb} is not a power of the fanout {fanout}")
    return dp


def summaries(k: np.ndarray, fanout: int, leaf_block: int) -> list[np.ndarray]:
    """Node summaries per level d = 1..Dp: array (f^d, B, H, D), float32 (index 0 = level 1)."""
    N = k.shape[0]
    dp = depth_of(N, fanout, leaf_block)
    kk = k.astype(np.float64)
    out = []
    for d in range(1, dp + 1):
        n = fanout ** d
        span = N // n
        out.append((kk.reshape(n, span, *k.shape[1:]).mean(axis=1) / 2).astype(np.float32))
    return out


def _log_softmax_masked(z: np.ndarray, valid: np.ndarray) -> np.ndarray:
    zz = np.where(valid, z, -np.inf)
    m = zz.max(-1, keepdims=True)
    return (zz - m - np.log(np.exp(zz - m).sum(-1, keepdims=True))).astype(np.float32)


def _boundary(L, num_keys, query_start, total_queries):
    """Causal boundary of queries [query_start, query_start + L) of ``total_queries``."""
    total = L if total_queries is None else total_queries
    return query_start + np.arange(L) + num_keys - total


def sample_blocks(q, summ, gumbels, num_samples, fanout, leaf_block, num_keys, causal,
                  query_start=0, total_queries=None):
    """Sampled leaf block (L, B, H, S) and path log-probability (float32).

    gumbels: (Dp, L, B, H, S, f) float32. ``q`` may be the slice [query_start, +L) of
    ``total_queries`` queries (the causal boundary is that of the full call).
    """
    L, B, H, D = q.shape
    dp = len(summ)
    S = num_samples
    j = np.zeros((L, B, H, S), dtype=np.int64)
    lp = np.zeros((L, B, H, S), dtype=np.float32)
    boundary = _boundary(L, num_keys, query_start, total_queries)
    for d in range(dp):
        child = summ[d]                                   # level d+1: (f^(d+1), B, H, D)
        idx = j[..., None] * fanout + np.arange(fanout)   # (L,B,H,S,f)
        rows = child[idx, np.arange(B)[None, :, None, None, None],
                     np.arange(H)[None, None, :, None, None]]  # (L,B,H,S,f,D)
        z = np.einsum("lbhd,lbhsfd->lbhsf", q.astype(np.float32), rows).astype(np.float32)
        if causal:
            span = num_keys // fanout ** (d + 1)
            first_key = idx * span
            valid = first_key <= boundary[:, None, None, None, None]
        else:
            valid = np.ones_like(z, dtype=bool)
        lsm = _log_softmax_masked(z, valid)
        score = np.where(valid, lsm + gumbels[d], -np.inf)
        dirn = score.argmax(-1)
        lp = (lp + np.take_along_axis(lsm, dirn[..., None], -1)[..., 0]).astype(np.float32)
        j = j * fanout + dirn
    return j, lp


def leaf_block_attention(q, k, v, blk, leaf_block, softmax_scale, causal, query_start=0,
                         total_queries=None):
    """o_s = softmax(scale q . K_blk) V_blk per path: (L, B, H, S, D) float32, and P."""
    L, B, H, D = q.shape
    N = k.shape[0]
    S = blk.shape[-1]
    keys = blk[..., None] * leaf_block + np.arange(leaf_block)       # (L,B,H,S,Lb)
    bi = np.arange(B)[None, :, None, None, None]
    hi = np.arange(H)[None, None, :, None, None]
    kr = k[keys, bi, hi].astype(np.float32)                            # (L,B,H,S,Lb,D)
    vr = v[keys, bi, hi].astype(np.float32)
    a = np.float32(softmax_scale) * np.einsum("lbhd,lbhskd->lbhsk", q.astype(np.float32), kr)
    if causal:
        boundary = _boundary(L, N, query_start, total_queries)
        a = np.where(keys <= boundary[:, None, None, None, None], a, -np.inf)
    m = a.max(-1, keepdims=True)
    e = np.exp(a - m)
    p = (e / e.sum(-1, keepdims=True)).astype(np.float32)
    return np.einsum("lbhsk,lbhskd->lbhsd", p, vr).astype(np.float32), p


def forward(q, k, v, gumbels, num_samples, fanout, leaf_block, causal=False, softmax_scale=None,
            query_start=0, total_queries=None, summ=None):
    """dict(out (L,B,H,D), weights (L,B,H,S), block (L,B,H,S)); q/k/v (seq, B, H, D) float32.

    ``q`` / ``gumbels`` may cover the query slice [query_start, +L) of ``total_queries`` (large
    problems are checked a slice at a time); ``summ`` reuses precomputed ``summaries``.
    """
    D = q.shape[-1]
    scale = D ** -0.5 if softmax_scale is None else softmax_scale
    summ = summaries(k, fanout, leaf_block) if summ is None else summ
    blk, lp = sample_blocks(q, summ, gumbels, num_samples, fanout, leaf_block, k.shape[0], causal,
                            query_start, total_queries)
    o, _ = leaf_block_attention(q, k, v, blk, leaf_block, scale, causal, query_start, total_queries)
    m = lp.max(-1, keepdims=True)
    e = np.exp(lp - m)
    w = (e / e.sum(-1, keepdims=True)).astype(np.float32)
    out = np.einsum("lbhs,lbhsd->lbhd", w, o).astype(np.float32)
    return dict(out=out, weights=w, block=blk, log_prob=lp)


def forward_torch(q, k, v, block, fanout, leaf_block, causal=False, softmax_scale=None,
                  query_start=0, total_queries=None):
    """Differentiable torch (CPU, float64-capable) restatement given the sampled blocks, for
    gradients: returns out (L, B, H, D). The path of block b is its base-f digits. ``q`` may
    be the query slice [query_start, +L) of ``total_queries``."""
    import torch

    L, B, H, D = q.shape
    N = k.shape[0]
    scale = D ** -0.5 if softmax_scale is None else softmax_scale
    dp = depth_of(N, fanout, leaf_block)
    blk = torch.as_tensor(block, dtype=torch.long)
    S = blk.shape[-1]
    bi = torch.arange(B)[None, :, None, None, None]
    hi = torch.arange(H)[None, None, :, None, None]
    boundary = torch.as_tensor(_boundary(L, N, query_start, total_queries))
    lp = torch.zeros(L, B, H, S, dtype=q.dtype)
    for d in range(dp):
        n = fanout ** (d + 1)
        span = N // n
        summ = k.reshape(n, span, B, H, D).mean(dim=1) / 2
        parent = blk // fanout ** (dp - d)
        dirn = (blk // fanout ** (dp - d - 1)) % fanout
        idx = parent[..., None] * fanout + torch.arange(fanout)
        rows = summ[idx, bi, hi]
        z = torch.einsum("lbhd,lbhsfd->lbhsf", q, rows)
        if causal:
            valid = idx * span <= boundary[:, None, None, None, None]
            z = z.masked_fill(~valid, float("-inf"))
        lsm = torch.log_softmax(z, dim=-1)
        lp = lp + torch.gather(lsm, -1, dirn[..., None])[..., 0]
    keys = blk[..., None] * leaf_block + torch.arange(leaf_block)
    kr = k[keys, bi, hi]
    vr = v[keys, bi, hi]
    a = scale * torch.einsum("lbhd,lbhskd->lbhsk", q, kr)
    if causal:
        a = a.masked_fill(~(keys <= boundary[:, None, None, None, None]), float("-inf"))
    p = torch.softmax(a, dim=-1)
    o = torch.einsum("lbhsk,lbhskd->lbhsd", p, vr)
    w = torch.softmax(lp, dim=-1)
    return torch.einsum("lbhs,lbhsd->lbhd", w, o)
