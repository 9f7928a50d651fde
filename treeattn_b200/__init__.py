"""treeattn_b200 -- B200-native (sm_100a) stochastic tree attention.

Public API (drop-in for the TreeAttention reference's hot path):

* ``hierarchical_attention(query, key, value, num_heads, is_causal=False,
  mode="stochastic", num_samples=64, *, block_size=256, max_logit=1e3)``
  -- the reference op's signature (treeattn_cuda/_autograd.py:863-915).
* ``tree_attention(q, k, v, causal=False, softmax_scale=None, *, num_samples=None)``
  -- the attn-bench kernel contract on bshd tensors (Haar tree build included).
* ``bench.adapter()`` -- an attn-bench ``KernelAdapter`` for ``treeattn_b200``.
* ``ops`` -- tensor-level wrappers of every C-ABI entry point.
* ``sharding`` -- head/batch sharding over one process per GPU (no collective).
"""

from . import ops, sharding
from .blocked import blocked_tree_attention
from .autograd import (
    CausalTreeAttentionFunction,
    ExactTreeAttentionFunction,
    TreeAttentionBshdFunction,
    TreeAttentionFunction,
    hierarchical_attention,
    resolve_num_samples,
    tree_attention,
)
from .ops import get_runtime_stats, reset_runtime_stats


def has_native_kernels() -> bool:
    """True when the in-tree CUDA library loads (there is no non-native path)."""
    try:
        from . import _lib

        _lib.load(build_if_missing=False)
        return True
    except OSError:
        return False


__all__ = [
    "hierarchical_attention",
    "tree_attention",
    "blocked_tree_attention",
    "TreeAttentionFunction",
    "CausalTreeAttentionFunction",
    "ExactTreeAttentionFunction",
    "TreeAttentionBshdFunction",
    "resolve_num_samples",
    "get_runtime_stats",
    "reset_runtime_stats",
    "has_native_kernels",
    "ops",
    "sharding",
]
