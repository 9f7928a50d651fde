"""attn-bench integration: ``treeattn_b200.bench:adapter`` is a loadable entrypoint.

``attn_bench.adapters.load_entrypoint("treeattn_b200.bench:adapter")`` returns a
``KernelAdapter`` wrapping ``tree_attention`` (attn_bench/adapters.py:32-93). When
attn-bench is not installed, a structurally identical dataclass is returned.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable

import torch

from .autograd import tree_attention

BASELINE_NAME = "treeattn_b200"


@dataclass(frozen=True)
class _KernelAdapter:
    name: str
    fn: Callable
    supports_backward: bool = True
    supports_causal: bool = True
    allowed_dtypes: frozenset = field(default_factory=lambda: frozenset({torch.float16, torch.bfloat16}))
    allowed_head_dims: frozenset = field(default_factory=lambda: frozenset({32, 64, 96, 128}))
    layout: str = "bshd"

    def is_compatible(self, dtype, head_dim, causal):
        if dtype not in self.allowed_dtypes:
            return False, f"dtype {dtype} not in allowed_dtypes"
        if head_dim not in self.allowed_head_dims:
            return False, f"head_dim {head_dim} not in allowed_head_dims"
        if causal and not self.supports_causal:
            return False, "kernel does not support causal=True"
        return True, ""


def _call(q, k, v, causal, softmax_scale):
    return tree_attention(q, k, v, causal, softmax_scale)


def adapter():
    try:
        from attn_bench.adapters import KernelAdapter
    except ImportError:
        KernelAdapter = _KernelAdapter
    return KernelAdapter(
        name=BASELINE_NAME,
        fn=_call,
        supports_backward=True,
        supports_causal=True,
        allowed_dtypes=frozenset({torch.float16, torch.bfloat16, torch.float32}),
        allowed_head_dims=frozenset({32, 64, 96, 128}),
        layout="bshd",
    )


# Tree-aware accounting. attn-bench's flops.py counts dense attention (4 b h s^2 d forward,
# attn_bench/flops.py:19-27), which overstates a sampled tree by orders of magnitude. Per
# (query, head), stochastic tree attention does num_samples root-to-leaf walks of log2(N)
# node dot products (2 d FLOPs each) plus a num_samples-row weighted value sum (2 d each).

def _log2(n: int) -> int:
    return max(int(n).bit_length() - 1, 0)


def fwd_flops(batch: int, seqlen: int, nheads: int, head_dim: int, causal: bool,
              num_samples: int = 8) -> float:
    """Forward FLOPs of stochastic tree attention (causal: the same walk, corrected)."""
    del causal
    per_query = num_samples * (_log2(seqlen) + 1) * 2.0 * head_dim
    return float(batch) * seqlen * nheads * per_query


def bwd_flops(batch: int, seqlen: int, nheads: int, head_dim: int, causal: bool,
              num_samples: int = 8) -> float:
    """Backward: per path and level dq and dK updates (2 x 2d) plus the node logit replay
    read from the forward's branch probabilities; per path g = dO . v and the dV update."""
    del causal
    per_query = num_samples * (_log2(seqlen) * 4.0 + 4.0) * head_dim
    return float(batch) * seqlen * nheads * per_query


def compulsory_bytes(batch: int, seqlen: int, nheads: int, head_dim: int, elem_bytes: int = 2,
                     backward: bool = True) -> float:
    """Unique HBM bytes: read q, k, v and write out (forward); read q, k, v, out, dO and write
    dq, dk, dv (backward). The roofline denominator for these gather-bound kernels."""
    unit = float(batch) * seqlen * nheads * head_dim * elem_bytes
    return unit * (4 + (8 if backward else 0))


def is_available() -> bool:
    from . import has_native_kernels

    return has_native_kernels()
