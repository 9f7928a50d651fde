"""Float32 torch (CPU) restatement of the causal and exact tree-attention modes, for gradients.

TEST INFRASTRUCTURE ONLY (same rules as ``oracle/tree_oracle.py``): autograd through these
functions gives the reference gradients of the causal sampler with its boundary correction
and of the exact (deterministic) mode, which the CUDA backward is checked against. Gumbel
noise is injected, so the functions are deterministic given their inputs.

Pinned against the reference: ``tests/test_oracle_golden.py`` compares outputs and
autograd gradients with fixtures recorded from treeattn-torch itself.

Reference: packages/treeattn-torch/src/treeattn_torch/_tree_mha.py
(``_sample_paths_causal`` :125-268, ``_deterministic_attention`` :271-321,
``hierarchical_attention`` :324-413).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _log_n(num_leaves: int) -> int:
    return max(num_leaves.bit_length() - 1, 0)


def deterministic_attention(q, k, v, is_causal):
    """Exact attention over all leaves (_tree_mha.py:271-321); (L,B,H,D) tensors, float32."""
    L, B, H, D = q.shape
    N = v.shape[0]
    log_n = _log_n(N)
    lp = torch.zeros(L, B, H, 1, dtype=q.dtype)
    for d in range(log_n):
        kd = k[(1 << d) - 1:(1 << (d + 1)) - 1]                    # (2^d, B, H, D)
        s = torch.einsum("lbhd,nbhd->lbhn", q, kd)
        lp = torch.stack([lp + F.logsigmoid(s), lp + F.logsigmoid(-s)], dim=-1).reshape(L, B, H, -1)
    if is_causal:
        mask = torch.arange(N).view(1, N) > torch.arange(L).view(L, 1)
        lp = lp.masked_fill(mask[:, None, None, :], float("-inf"))
        w = torch.softmax(lp, dim=-1)
    else:
        w = torch.exp(lp)
    return torch.einsum("lbhn,nbhd->lbhd", w, v), w


def sample_paths_causal(q, k, gumbels, num_samples, causal_offset=0):
    """Causal sampler (_tree_mha.py:125-268), injected gumbels (L, log_n, B, H, S, 2)."""
    L, B, H, D = q.shape
    K = k.shape[0]
    log_n = _log_n(K + 1)
    S = num_samples
    kk = k.permute(1, 2, 0, 3)                                     # (B, H, K, D)
    leaves, lps = [], []
    for t in range(L):
        boundary = t + causal_offset
        nodes, node = [], 0
        for d in range(log_n):
            nodes.append(node)
            node = 2 * node + 1 + ((boundary >> (log_n - 1 - d)) & 1)
        sb = torch.einsum("bhd,pbhd->bhp", q[t], k[nodes])
        mass = [None] * (log_n + 1)
        mass[log_n] = torch.zeros(B, H, dtype=q.dtype)
        for d in range(log_n - 1, -1, -1):
            bdir = (boundary >> (log_n - 1 - d)) & 1
            lpl, lpr = F.logsigmoid(sb[..., d]), F.logsigmoid(-sb[..., d])
            if bdir == 0:
                on, off = lpl, lpr
                off_mass = torch.full_like(on, float("-inf"))
            else:
                on, off = lpr, lpl
                off_mass = torch.full_like(on, math.log(float(1 << (log_n - 1 - d))))
            mass[d] = torch.logsumexp(torch.stack([mass[d + 1] + on, off_mass + off]), dim=0)
        cur = torch.zeros(B, H, S, dtype=torch.long)
        acc = torch.zeros(B, H, S, dtype=q.dtype)
        for d in range(log_n):
            on_path = bool(torch.all(cur == nodes[d]))
            kd = torch.gather(kk, 2, cur.unsqueeze(-1).expand(B, H, S, D))
            s = (q[t].unsqueeze(2) * kd).sum(-1)
            lpl, lpr = F.logsigmoid(s), F.logsigmoid(-s)
            if on_path:
                bdir = (boundary >> (log_n - 1 - d)) & 1
                parent = mass[d].unsqueeze(-1)
                child = mass[d + 1].unsqueeze(-1)
                if bdir == 0:
                    ml, mr = child, torch.full_like(child, float("-inf"))
                else:
                    ml = torch.full_like(child, math.log(float(1 << (log_n - 1 - d))))
                    mr = child
                lpl = ml + lpl - parent
                lpr = mr + lpr - parent
            g = gumbels[t, d]
            direction = ((lpr + g[..., 1]) > (lpl + g[..., 0])).long()
            acc = acc + torch.where(direction == 1, lpr, lpl)
            cur = 2 * cur + 1 + direction
        leaves.append(cur - K)
        lps.append(acc)
    return torch.stack(leaves), torch.stack(lps)


def causal_attention(q, k, v, gumbels, num_samples):
    """hierarchical_attention(is_causal=True, mode='stochastic') (_tree_mha.py:379-412)."""
    L = q.shape[0]
    S = num_samples
    N = v.shape[0]
    hybrid = L > S
    if hybrid:
        out_det, _ = deterministic_attention(q[:S], k, v, True)
        leaf, lp = sample_paths_causal(q[S:], k, gumbels, S, causal_offset=S)
    else:
        leaf, lp = sample_paths_causal(q, k, gumbels, S)
    valid = (leaf >= 0) & (leaf < N)
    lp = lp.masked_fill(~valid, float("-inf"))
    w = torch.softmax(lp, dim=-1)
    B, H, D = v.shape[1:]
    vv = v.permute(1, 2, 0, 3)
    lq = leaf.shape[0]
    idx = leaf.clamp(0, N - 1)
    gathered = torch.gather(vv.unsqueeze(0).expand(lq, B, H, N, D), 3,
                            idx.unsqueeze(-1).expand(lq, B, H, S, D))
    out_sto = torch.einsum("lbhs,lbhsd->lbhd", w, gathered)
    out = torch.cat([out_det, out_sto]) if hybrid else out_sto
    return out, w, leaf
