"""Autograd functions and the reference-facing entry points.

* ``hierarchical_attention`` -- same signature, argument meaning and errors as the
  reference op ``treeattn_cuda.hierarchical_attention``
  (packages/treeattn-cuda/src/treeattn_cuda/_autograd.py:863-915).
* ``tree_attention`` -- the attn-bench kernel contract ``fn(q, k, v, causal, softmax_scale)``
  on bshd tensors, including the Haar tree build (attn_bench/baselines/treeattn_cuda.py:24-59)
  fused into one autograd node.
"""

from __future__ import annotations

import os
from typing import Literal

import torch

from . import ops

Mode = Literal["deterministic", "stochastic"]
NUM_SAMPLES_ENV_VAR = "TREEATTN_NUM_SAMPLES"
_DEFAULT_BLOCK_SIZE = 256


_NOISE_STREAMS: dict = {}


def _noise_stream(device):
    """One side stream per device for the forward's noise draw."""
    key = torch.device(device).index
    st = _NOISE_STREAMS.get(key)
    if st is None:
        st = _NOISE_STREAMS[key] = torch.cuda.Stream(device)
    return st


class TreeAttentionFunction(torch.autograd.Function):
    """Stochastic non-causal tree attention on (seq, B, H, D) views.

    forward(q (L,B,H,D), k_int (N-1,B,H,D), v (N,B,H,D), num_samples, max_logit)
      -> (out (L,B,H,D), weights (L,B,H,S) float32, non-differentiable)
    Saves q, k_int, v and the sampled leaves / weights (8 bytes per path) for backward.
    """

    @staticmethod
    def forward(ctx, q, k_int, v, num_samples, max_logit):
        res = ops.forward(q, k_int, v, num_samples, max_logit=max_logit)
        ctx.save_for_backward(q, k_int, v, res.leaf, res.weights, res.branch_prob)
        ctx.num_samples = num_samples
        ctx.max_logit = max_logit
        ctx.mark_non_differentiable(res.weights)
        return res.out, res.weights

    @staticmethod
    def backward(ctx, grad_out, grad_weights):
        del grad_weights
        q, k_int, v, leaf, weights, bp = ctx.saved_tensors
        dq, dk, dv = ops.backward(q, k_int, v, grad_out, leaf, weights, bp, ctx.num_samples,
                                  max_logit=ctx.max_logit, dk_dtype=k_int.dtype)
        return dq, dk, dv, None, None


class TreeAttentionBshdFunction(torch.autograd.Function):
    """Tree build + stochastic tree attention on bshd tensors, one autograd node.

    The internal-node keys stay float32 in backward (dk_int is fed to the transposed tree
    build directly), so dK is rounded to the input dtype once.
    """

    @staticmethod
    def forward(ctx, q, k, v, num_samples, max_logit, gumbels=None, causal=False, shard=None,
                node_layout="reference"):
        qv, kv, vv = (t.transpose(0, 1) for t in (q, k, v))  # logical (S, B, H, D) views
        side = None
        if (q.is_cuda and not causal and gumbels is None and kv.shape[0] > 1
                and ops.is_power_of_two(kv.shape[0])):
            # the noise draw does not depend on the tree: it runs on a side stream beside the
            # tree build (the generator offsets are reserved on the host in the same order)
            # (the buffer is allocated on the current stream, which waits for the draw before
            # its first use, so the caching allocator reuses it step after step)
            Lq, B, H = qv.shape[:3]
            buf = torch.empty((ops.log_n_of(kv.shape[0]), Lq * B * H * num_samples * 2),
                              device=q.device, dtype=torch.float32)
            cur = torch.cuda.current_stream(q.device)
            side = _noise_stream(q.device)
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                gumbels = ops.draw_gumbels(Lq, B, H, kv.shape[0], num_samples, q.device,
                                           shard=shard, out=buf)
        k_int = ops.tree_build(kv, node_layout=node_layout)
        if side is not None:
            cur.wait_stream(side)
        ctx.node_layout = node_layout
        out = torch.empty_like(q)
        ctx.num_samples = num_samples
        ctx.max_logit = max_logit
        ctx.causal = causal
        if causal:
            st = _causal_fwd(qv, k_int, vv, num_samples, out.transpose(0, 1))
            ctx.save_for_backward(q, k_int, v, st.leaf, st.weights, st.branch_prob, st.corrected,
                                  st.masses)
            ctx.query_offset = st.query_offset
            return out
        res = ops.forward(qv, k_int, vv, num_samples, max_logit=max_logit, out=out.transpose(0, 1),
                          gumbels=gumbels, shard=shard)
        ctx.save_for_backward(q, k_int, v, res.leaf, res.weights, res.branch_prob)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        if ctx.causal:
            q, k_int, v, leaf, weights, bp, corrected, masses = ctx.saved_tensors
            st = ops.CausalState(leaf, weights, bp, corrected, masses, ctx.query_offset)
            B, S, H, D = q.shape
            dq = torch.empty_like(q)
            dk_int = torch.empty((B, H, S - 1, D), device=q.device, dtype=torch.float32).permute(2, 0, 1, 3)
            dv32 = torch.empty((S, B, H, D), device=q.device, dtype=torch.float32)
            grad_out = grad_out if grad_out.stride(-1) == 1 else grad_out.contiguous()
            _causal_bwd(q.transpose(0, 1), k_int, v.transpose(0, 1), grad_out.transpose(0, 1), st,
                        ctx.num_samples, dq.transpose(0, 1), dk_int, dv32)
            dk = torch.empty_like(q)
            ops.tree_build_backward(dk_int, dk.transpose(0, 1), ctx.node_layout)
            dv = dv32.transpose(0, 1).to(v.dtype).contiguous()
            return dq, dk, dv, None, None, None, None, None, None
        q, k_int, v, leaf, weights, bp = ctx.saved_tensors
        B, S, H, D = q.shape
        dq = torch.empty_like(q)
        dv = torch.empty_like(v)
        dk_int = torch.empty((B, H, S - 1, D), device=q.device, dtype=torch.float32).permute(2, 0, 1, 3)
        grad_out = grad_out if grad_out.stride(-1) == 1 else grad_out.contiguous()
        ops.backward(q.transpose(0, 1), k_int, v.transpose(0, 1), grad_out.transpose(0, 1), leaf,
                     weights, bp, ctx.num_samples, max_logit=ctx.max_logit, dq=dq.transpose(0, 1),
                     dk=dk_int, dv=dv.transpose(0, 1))
        dk = torch.empty_like(q)
        ops.tree_build_backward(dk_int, dk.transpose(0, 1), ctx.node_layout)
        return dq, dk, dv, None, None, None, None, None, None


def _causal_fwd(q, k_int, v, num_samples, out):
    """Causal stochastic forward on (seq,B,H,D) views (_tree_mha.py:379-412): the first S
    queries take exact causal attention when L > S, the rest the corrected sampler."""
    S = num_samples
    if q.shape[0] > S:
        ops.exact_forward(q[:S], k_int, v, True, 0, out=out[:S], want_weights=False)
        _, st = ops.causal_forward(q[S:], k_int, v, S, S, out=out[S:])
    else:
        _, st = ops.causal_forward(q, k_int, v, S, 0, out=out)
    return st


def _causal_bwd(q, k_int, v, grad_out, st, num_samples, dq, dk32, dv32):
    S = num_samples
    if q.shape[0] > S:
        ops.causal_backward(q[S:], k_int, v, grad_out[S:], st, S, dq=dq[S:], dk=dk32, dv=dv32)
        ops.exact_backward(q[:S], k_int, v, grad_out[:S], True, 0, dq=dq[:S], dk=dk32, dv=dv32,
                           accumulate=True)
    else:
        ops.causal_backward(q, k_int, v, grad_out, st, S, dq=dq, dk=dk32, dv=dv32)


class CausalTreeAttentionFunction(torch.autograd.Function):
    """Causal stochastic tree attention on (seq, B, H, D) views: exact causal prefix for the
    first S queries (when L > S) and the boundary-corrected sampler for the rest.
    Returns (out, weights of the sampled queries (L', B, H, S) float32)."""

    @staticmethod
    def forward(ctx, q, k_int, v, num_samples):
        out = torch.empty(q.shape, device=q.device, dtype=q.dtype)
        st = _causal_fwd(q, k_int, v, num_samples, out)
        ctx.save_for_backward(q, k_int, v, st.leaf, st.weights, st.branch_prob, st.corrected,
                              st.masses)
        ctx.query_offset = st.query_offset
        ctx.num_samples = num_samples
        ctx.mark_non_differentiable(st.weights)
        return out, st.weights

    @staticmethod
    def backward(ctx, grad_out, grad_weights):
        del grad_weights
        q, k_int, v, leaf, weights, bp, corrected, masses = ctx.saved_tensors
        st = ops.CausalState(leaf, weights, bp, corrected, masses, ctx.query_offset)
        dq = torch.empty(q.shape, device=q.device, dtype=q.dtype)
        dk = torch.empty(k_int.shape, device=q.device, dtype=torch.float32)
        dv = torch.empty(v.shape, device=q.device, dtype=torch.float32)
        _causal_bwd(q, k_int, v, grad_out, st, ctx.num_samples, dq, dk, dv)
        return dq, dk.to(k_int.dtype), dv.to(v.dtype), None


class ExactTreeAttentionFunction(torch.autograd.Function):
    """mode='deterministic': attention over all leaves (_tree_mha.py:271-321)."""

    @staticmethod
    def forward(ctx, q, k_int, v, causal):
        out, w = ops.exact_forward(q, k_int, v, causal, 0, want_weights=True)
        ctx.save_for_backward(q, k_int, v)
        ctx.causal = causal
        ctx.mark_non_differentiable(w)
        return out, w

    @staticmethod
    def backward(ctx, grad_out, grad_weights):
        del grad_weights
        q, k_int, v = ctx.saved_tensors
        dq = torch.empty(q.shape, device=q.device, dtype=q.dtype)
        dk = torch.empty(k_int.shape, device=q.device, dtype=torch.float32)
        dv = torch.empty(v.shape, device=q.device, dtype=torch.float32)
        ops.exact_backward(q, k_int, v, grad_out, ctx.causal, 0, dq=dq, dk=dk, dv=dv,
                           accumulate=False)
        return dq, dk.to(k_int.dtype), dv.to(v.dtype), None


def hierarchical_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    num_heads: int,
    is_causal: bool = False,
    mode: Mode = "stochastic",
    num_samples: int = 64,
    *,
    block_size: int = _DEFAULT_BLOCK_SIZE,
    max_logit: float = ops.MAX_LOGIT,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Hierarchical (tree) attention: query (L,B,E), key (N-1,B,E), value (N,B,E).

    Returns ``(output (L,B,E), weights float32)``: (L,B,H,S) for the non-causal sampler, the
    sampled queries' (L-S,B,H,S) in causal mode when L > S (as the reference), and (L,B,H,N)
    in mode='deterministic'. ``block_size`` is accepted for signature compatibility; the fused
    kernels have no host-side query blocking. Mirrors treeattn_cuda/_autograd.py:863-915
    (non-causal stochastic) and treeattn_torch/_tree_mha.py:324-413 (causal, deterministic).
    """
    del block_size
    if mode not in ("stochastic", "deterministic"):
        raise ValueError(f"unknown mode {mode!r}")
    if query.dim() != 3 or value.dim() != 3:
        raise ValueError("query and value must have shape (L, B, E) and (N, B, E)")
    if mode == "stochastic" and (num_samples is None or num_samples <= 0):
        raise ValueError(f"num_samples must be > 0, got {num_samples}")
    l_q, batch, embed = query.shape
    num_leaves = value.shape[0]
    if embed % num_heads != 0:
        raise ValueError(f"embed_dim={embed} is not divisible by num_heads={num_heads}")
    width = embed // num_heads
    if num_leaves > 1 and key.shape[0] != num_leaves - 1:
        raise ValueError(f"Key tensor length must be N-1 ({num_leaves - 1}), but got {key.shape[0]}.")

    q = query.reshape(l_q, batch, num_heads, width)
    v = value.reshape(num_leaves, batch, num_heads, width)
    if num_leaves == 0:
        out = torch.zeros_like(query)
        return out, torch.empty((l_q, batch, num_heads, 0), device=query.device, dtype=query.dtype)
    if num_leaves == 1:
        # a single leaf: every path ends there (_autograd.py:668-683)
        out = value.expand(l_q, -1, -1)
        return out.contiguous(), torch.ones((l_q, batch, num_heads, 1), device=query.device,
                                            dtype=query.dtype)
    if not ops.is_power_of_two(num_leaves):
        raise ValueError(f"treeattn_b200 requires a power-of-two number of leaves, got {num_leaves}")
    k = key.reshape(num_leaves - 1, batch, num_heads, width)
    if mode == "deterministic":
        out, weights = ExactTreeAttentionFunction.apply(q, k, v, bool(is_causal))
    elif is_causal:
        out, weights = CausalTreeAttentionFunction.apply(q, k, v, num_samples)
    else:
        out, weights = TreeAttentionFunction.apply(q, k, v, num_samples, max_logit)
    return out.reshape(l_q, batch, embed), weights


def resolve_num_samples() -> int | None:
    """``TREEATTN_NUM_SAMPLES`` (attn_bench/baselines/_treeattn_common.py:30-47)."""
    raw = os.environ.get(NUM_SAMPLES_ENV_VAR, "").strip()
    if not raw or raw == "0":
        return None
    try:
        n = int(raw)
    except ValueError as e:
        raise ValueError(f"{NUM_SAMPLES_ENV_VAR}={raw!r} is not an integer") from e
    if n < 0:
        raise ValueError(f"{NUM_SAMPLES_ENV_VAR}={n} must be >= 0")
    return n or None


def tree_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                   softmax_scale: float | None = None, *, num_samples: int | None = None,
                   max_logit: float = ops.MAX_LOGIT,
                   gumbels: torch.Tensor | None = None, shard=None,
                   node_layout: str = "reference", scale_logits: bool = False) -> torch.Tensor:
    """attn-bench kernel contract: bshd q/k/v (B,S,H,D) -> out (B,S,H,D).

    ``k`` are leaf keys; the internal-node keys are their sequence-axis Haar transform in
    the reference's layout. ``causal=True`` follows treeattn-torch's causal mode (exact causal
    prefix for the first ``num_samples`` queries, boundary-corrected sampling for the rest,
    attn_bench/baselines/treeattn_torch.py:48-90). ``softmax_scale`` is ignored, as in the reference adapters
    (baselines/treeattn_cuda.py:25). ``num_samples`` defaults to ``TREEATTN_NUM_SAMPLES``.
    ``gumbels`` (float32 (log2 S, S, B, H, num_samples, 2)) replaces the generator's noise,
    for replaying a recorded draw. ``shard`` (``sharding.ShardSpec``, non-causal only) marks
    q/k/v as this rank's (batch, head) block of a larger problem; the result is that block
    of the unsharded call's result.

    Two opt-in departures from the reference's semantics: ``node_layout="tree"`` builds the
    tree-correct node keys (every heap node summarises its own subtree, ``ops.tree_build``),
    and ``scale_logits=True`` multiplies every tree logit q . k by ``softmax_scale`` (default
    1/sqrt(head_dim)) by scaling q, which the reference adapters never do.
    """
    if shard is not None and causal:
        raise ValueError("causal mode couples all heads of a query and cannot be head/batch sharded")
    if num_samples is None:
        num_samples = resolve_num_samples()
    if num_samples is None:
        raise ValueError("num_samples is required (argument or TREEATTN_NUM_SAMPLES)")
    if q.dim() != 4 or q.shape != k.shape or q.shape != v.shape:
        raise ValueError("q, k, v must share one (B, S, H, D) shape")
    B, S, H, D = q.shape
    if not ops.is_power_of_two(S) or S < 2:
        raise ValueError(f"treeattn_b200 requires power-of-two seqlen, got {S}")
    if node_layout not in ops.LAYOUTS:
        raise ValueError(f"node_layout must be 'reference' or 'tree', got {node_layout!r}")
    if scale_logits:
        scale = softmax_scale if softmax_scale is not None else q.shape[-1] ** -0.5
        q = q * scale
    q, k, v = (t if t.stride(-1) == 1 else t.contiguous() for t in (q, k, v))
    return TreeAttentionBshdFunction.apply(q, k, v, num_samples, max_logit, gumbels, bool(causal),
                                           shard, node_layout)
