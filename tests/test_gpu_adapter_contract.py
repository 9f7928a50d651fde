"""The attn-bench kernel contract for ``treeattn_b200.bench:adapter``.

The reference harness requires of every adapter ``fn(q, k, v, causal, softmax_scale)``
(README.md "Kernel contract"; attn_bench/adapters.py:139-154):

* no in-place modification of q, k, v: the harness compares ``data_ptr`` before and after the
  call (``check_no_inplace``); here the storage pointer, the autograd version counter and the
  values are all checked, through forward and backward;
* no host synchronisation in the hot path: forward + backward run under
  ``torch.cuda.set_sync_debug_mode("error")``, which raises on any synchronising CUDA call torch
  makes (device-to-host copies, ``.item()``, stream or device synchronisation); the library's
  own sources contain no synchronising call on these paths either
  (``tests/test_capi_host.py::test_library_sources_have_no_blocking_calls``);
* bshd in, bshd out, same dtype, autograd-capable.
"""

import pytest
import torch

from treeattn_b200.bench import adapter

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _snapshot(ts):
    return [(t.data_ptr(), t._version, t.detach().clone()) for t in ts]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("B,S,H,D", [(2, 1024, 4, 64), (1, 2048, 2, 128)])
def test_adapter_no_inplace_no_sync(dtype, causal, B, S, H, D, monkeypatch):
    monkeypatch.setenv("TREEATTN_NUM_SAMPLES", "8")
    ad = adapter()
    ok, why = ad.is_compatible(dtype, D, causal)
    assert ok, why
    g = torch.Generator(device=DEV).manual_seed(S + D)
    q, k, v, go = (torch.randn(B, S, H, D, device=DEV, generator=g).to(dtype) for _ in range(4))
    q, k, v = (t.requires_grad_(True) for t in (q, k, v))
    before = _snapshot((q, k, v))
    torch.manual_seed(0)
    # warm the allocator and the library (first calls load the module and size workspaces)
    ad.fn(q, k, v, causal, None).backward(go)
    q.grad = k.grad = v.grad = None
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        out = ad.fn(q, k, v, causal, None)
        out.backward(go)
    finally:
        torch.cuda.set_sync_debug_mode("default")
    torch.cuda.synchronize()
    assert out.shape == q.shape and out.dtype == dtype
    assert all(t.grad is not None and t.grad.shape == t.shape for t in (q, k, v))
    for t, (ptr, ver, val) in zip((q, k, v), before):
        assert t.data_ptr() == ptr, "input storage replaced"
        assert t._version == ver, "input modified in place (version counter moved)"
        assert torch.equal(t.detach(), val), "input values changed"
    assert torch.isfinite(out.float()).all()


def test_blocked_mode_no_sync():
    """The generalised (fanout, leaf block) mode's autograd op under the same sync check."""
    from treeattn_b200 import blocked as TB

    g = torch.Generator(device=DEV).manual_seed(1)
    q, k, v, go = (torch.randn(2, 2048, 2, 128, device=DEV, generator=g).to(torch.bfloat16) for _ in range(4))
    q, k, v = (t.requires_grad_(True) for t in (q, k, v))
    TB.blocked_tree_attention(q, k, v, True, None, num_samples=8, fanout=4, leaf_block=128).backward(go)
    torch.cuda.synchronize()
    before = _snapshot((q, k, v))
    torch.cuda.set_sync_debug_mode("error")
    try:
        out = TB.blocked_tree_attention(q, k, v, True, None, num_samples=8, fanout=4, leaf_block=128)
        out.backward(go)
    finally:
        torch.cuda.set_sync_debug_mode("default")
    torch.cuda.synchronize()
    for t, (ptr, ver, val) in zip((q, k, v), before):
        assert t.data_ptr() == ptr and t._version == ver and torch.equal(t.detach(), val)
