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


def is_available() -> bool:
    from . import has_native_kernels

    return has_native_kernels()
