"""Generalised tree attention: fanout f, leaf blocks of Lb keys (no reference counterpart).

The benchmark configurations name a fanout and a leaf block ("fanout 4, leaf block 128"); the
reference's tree is binary with one key per leaf. At fanout 2, leaf block 1 this mode is the
reference sampler on the tree-correct node layout (``node_layout="tree"``). Semantics, noise
and the deterministic backward are described in ``include/treeattn_b200.h``
(``ta_blocked_*``).

    out = blocked_tree_attention(q, k, v, causal=False, softmax_scale=None,
                                 num_samples=8, fanout=4, leaf_block=128)

q, k, v are bshd (B, S, H, D); out likewise. ``shard`` (``sharding.ShardSpec``) and
``query_rows`` = (row0, row_total) mark the call as one block of a larger problem: the noise
is keyed by global (batch, head, query), so a shard returns exactly its slice of the full call.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib as L
from . import ops


def depth(num_keys: int, fanout: int, leaf_block: int) -> int:
    rows = L.load().ta_blocked_summary_rows(num_keys, fanout, leaf_block)
    if rows < 0:
        raise ValueError(f"num_keys={num_keys} must be leaf_block ({leaf_block}) * fanout "
                         f"({fanout})^depth with power-of-two fanout in [2,16], leaf_block in [1,256]")
    d, n = 0, num_keys // leaf_block
    while n > 1:
        n //= fanout
        d += 1
    return d


def _config(fanout, leaf_block, causal, scale, Lq, B, H, shard, query_rows):
    b0, bt, h0, ht = 0, B, 0, H
    if shard is not None:
        b0, bt, h0, ht = shard.batch0, shard.batch_total, shard.head0, shard.head_total
    r0, rt = query_rows if query_rows is not None else (0, Lq)
    return L.Blocked(int(fanout), int(leaf_block), 1 if causal else 0, float(scale), r0, rt, b0, bt, h0, ht)


def reserve_stream(device: torch.device, num_samples: int, fanout: int, levels: int) -> L.Rng:
    """Reserve one call's noise from torch's CUDA generator: every (batch, head, query)
    subsequence uses offsets [offset, offset + levels * S * f)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    gen = torch.cuda.default_generators[idx]
    used = (levels * num_samples * fanout + 3) // 4 * 4
    offset = gen.get_offset()
    gen.set_offset(offset + max(used, 4))
    return L.Rng(gen.initial_seed(), offset, 0, 1)


def build(k_sbhd: torch.Tensor, cfg: L.Blocked, num_samples: int) -> torch.Tensor:
    """Node summaries [B*H][rows][D] float32 of (seq, B, H, D) keys."""
    N, B, H, D = k_sbhd.shape
    rows = L.load().ta_blocked_summary_rows(N, cfg.fanout, cfg.leaf_block)
    summ = torch.empty((B * H, max(rows, 1), D), device=k_sbhd.device, dtype=torch.float32)
    shape = L.Shape(B, 1, N, H, D, num_samples, ops.dtype_code(k_sbhd.dtype), ops.MAX_LOGIT)
    L.call("ta_blocked_build", ctypes.byref(shape), ctypes.byref(cfg), ops._ptr(k_sbhd),
           ops.layout(k_sbhd), ops._ptr(summ), ops._stream(k_sbhd.device))
    return summ


def gumbel_fill(shape: L.Shape, cfg: L.Blocked, rng: L.Rng, device) -> torch.Tensor:
    """The noise a forward with ``rng`` draws: (Dp, L, B, H, S, f) float32."""
    dp = depth(shape.num_leaves, cfg.fanout, cfg.leaf_block)
    out = torch.empty((dp, shape.num_queries, shape.batch, shape.num_heads, shape.num_samples,
                       cfg.fanout), device=device, dtype=torch.float32)
    L.call("ta_blocked_gumbel_fill", ctypes.byref(shape), ctypes.byref(cfg), ctypes.byref(rng),
           ops._ptr(out), ops._stream(torch.device(device)))
    return out


class BlockedTreeAttentionFunction(torch.autograd.Function):
    """Autograd op over bshd q, k, v."""

    @staticmethod
    def forward(ctx, q, k, v, num_samples, fanout, leaf_block, causal, scale, gumbels, shard,
                query_rows):
        B, Lq, H, D = q.shape
        N = k.shape[1]
        qv, kv, vv = (t.transpose(0, 1) for t in (q, k, v))
        cfg = _config(fanout, leaf_block, causal, scale, Lq, B, H, shard, query_rows)
        shape = L.Shape(B, Lq, N, H, D, num_samples, ops.dtype_code(q.dtype), ops.MAX_LOGIT)
        summ = build(kv, cfg, num_samples)
        out = torch.empty_like(q)
        blk = torch.empty((Lq, B, H, num_samples), device=q.device, dtype=torch.int32)
        w = torch.empty((Lq, B, H, num_samples), device=q.device, dtype=torch.float32)
        lib = L.load()
        path_out, ws = None, None
        if lib.ta_blocked_uses_tensor_cores(ctypes.byref(shape), ctypes.byref(cfg), 0):
            # w_s o_s rows [B*H][L*S][D] in the input dtype, then each pair's float32
            # log-sum-exp [B*H][L*S]
            path_out = torch.empty(B * H * Lq * num_samples * (D // 2 + 1), device=q.device,
                                   dtype=torch.float32)
            ws_bytes = lib.ta_blocked_forward_workspace_size(ctypes.byref(shape), ctypes.byref(cfg))
            ws = torch.empty(max(ws_bytes, 1), device=q.device, dtype=torch.uint8)
        rng_p, g_p = None, None
        if gumbels is not None:
            gumbels = gumbels.to(device=q.device, dtype=torch.float32).contiguous()
            g_p = ops._ptr(gumbels)
        else:
            rng_p = ctypes.byref(reserve_stream(q.device, num_samples, fanout,
                                                depth(N, fanout, leaf_block)))
        L.call("ta_blocked_forward", ctypes.byref(shape), ctypes.byref(cfg), ops._ptr(qv),
               ops.layout(qv), ops._ptr(kv), ops.layout(kv), ops._ptr(vv), ops.layout(vv),
               ops._ptr(summ), ops._ptr(out), ops.layout(out.transpose(0, 1)), rng_p, g_p,
               ops._ptr(blk), ops._ptr(w), ops._ptr(path_out), ops._ptr(ws),
               ws.numel() if ws is not None else 0, ops._stream(q.device))
        ctx.save_for_backward(q, k, v, summ, blk, w, path_out)
        ctx.cfg, ctx.shape = cfg, shape
        ctx.mark_non_differentiable(blk, w)
        return out, blk, w

    @staticmethod
    def backward(ctx, grad_out, _gb, _gw):
        q, k, v, summ, blk, w, path_out = ctx.saved_tensors
        cfg, shape = ctx.cfg, ctx.shape
        grad_out = grad_out if grad_out.stride(-1) == 1 else grad_out.contiguous()
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        lib = L.load()
        ws_bytes = lib.ta_blocked_backward_workspace_size(ctypes.byref(shape), ctypes.byref(cfg))
        if ws_bytes == 0:
            raise ValueError("invalid blocked backward shape")
        ws = torch.empty(ws_bytes, device=q.device, dtype=torch.uint8)
        t = lambda x: x.transpose(0, 1)  # noqa: E731
        L.call("ta_blocked_backward", ctypes.byref(shape), ctypes.byref(cfg), ops._ptr(t(q)),
               ops.layout(t(q)), ops._ptr(t(k)), ops.layout(t(k)), ops._ptr(t(v)), ops.layout(t(v)),
               ops._ptr(summ), ops._ptr(t(grad_out)), ops.layout(t(grad_out)), ops._ptr(blk),
               ops._ptr(w), ops._ptr(path_out), ops._ptr(t(dq)), ops.layout(t(dq)), ops._ptr(t(dk)),
               ops.layout(t(dk)),
               ops._ptr(t(dv)), ops.layout(t(dv)), ops._ptr(ws), ws_bytes, ops._stream(q.device))
        return dq, dk, dv, None, None, None, None, None, None, None, None


def blocked_tree_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                           softmax_scale: float | None = None, *, num_samples: int = 8,
                           fanout: int = 2, leaf_block: int = 64,
                           gumbels: torch.Tensor | None = None, shard=None,
                           query_rows: tuple[int, int] | None = None, return_paths: bool = False):
    """Generalised stochastic tree attention on bshd tensors (see the module docstring).

    ``return_paths`` also returns the sampled leaf blocks (L, B, H, S) int32 and the path
    weights (L, B, H, S) float32 (non-differentiable).
    """
    if q.dim() != 4 or k.dim() != 4 or k.shape != v.shape or q.shape[0] != k.shape[0] or \
            q.shape[2:] != k.shape[2:]:
        raise ValueError("q (B, L, H, D) and k, v (B, N, H, D) must agree in B, H, D")
    if q.dtype != k.dtype or k.dtype != v.dtype:
        raise ValueError("q, k and v must share a dtype")
    N = k.shape[1]
    depth(N, fanout, leaf_block)  # validates the geometry
    if causal and q.shape[1] > N:
        raise ValueError("causal blocked attention needs L <= N")
    scale = softmax_scale if softmax_scale is not None else q.shape[-1] ** -0.5
    q, k, v = (t if t.stride(-1) == 1 else t.contiguous() for t in (q, k, v))
    out, blk, w = BlockedTreeAttentionFunction.apply(q, k, v, int(num_samples), int(fanout),
                                                     int(leaf_block), bool(causal), float(scale),
                                                     gumbels, shard, query_rows)
    return (out, blk, w) if return_paths else out
