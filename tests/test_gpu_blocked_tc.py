"""The tcgen05 (TMEM) leaf-block forward and backward against the mma.sync ones on the same
sampled paths, and their bounded-wait status word."""

import pytest
import torch

from tests.tolerance import assert_within
from treeattn_b200 import _lib as L
from treeattn_b200 import blocked as TB

pytestmark = pytest.mark.gpu


def _run(q, k, v, causal, S, f, Lb, tc):
    lib = L.load()
    old = lib.ta_blocked_set_tcgen05(1 if tc else 0)
    try:
        torch.manual_seed(42)
        return TB.blocked_tree_attention(q, k, v, causal, None, num_samples=S, fanout=f,
                                         leaf_block=Lb, return_paths=True)
    finally:
        lib.ta_blocked_set_tcgen05(old)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,N,H,D,S,f,Lb,causal", [
    (1, 256, 1, 128, 4, 2, 64, False),
    (2, 1024, 2, 64, 8, 4, 16, True),
    (1, 2048, 2, 128, 8, 2, 128, True),
    (2, 512, 3, 64, 8, 2, 32, False),
])
def test_tcgen05_forward_matches_mma_sync(dtype, B, N, H, D, S, f, Lb, causal):
    g = torch.Generator(device="cuda").manual_seed(N + D)
    q, k, v = (torch.randn(B, N, H, D, device="cuda", generator=g).to(dtype) for _ in range(3))
    out_tc, blk_tc, w_tc = _run(q, k, v, causal, S, f, Lb, True)
    out_ms, blk_ms, w_ms = _run(q, k, v, causal, S, f, Lb, False)
    torch.cuda.synchronize()
    assert torch.equal(blk_tc, blk_ms) and torch.equal(w_tc, w_ms)  # same walk
    tol = 2e-2 if dtype == torch.bfloat16 else 5e-3
    assert (out_tc.float() - out_ms.float()).abs().max().item() < tol


def test_expired_wait_is_reported_by_the_next_call():
    """A 1 ns bound makes the tcgen05 forward's first mbarrier wait expire (the MMA cannot
    finish that fast). The CTA records it in the host-visible status word, drains its MMA under
    the normal bound and frees its TMEM; the next blocked call raises instead of running, and
    once reported the status is clear again. Nothing waits on a flag that is never set."""
    lib = L.load()
    g = torch.Generator(device="cuda").manual_seed(3)
    q, k, v = (torch.randn(1, 1024, 2, 128, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3))
    lib.ta_blocked_status(1)
    old_tc = lib.ta_blocked_set_tcgen05(1)
    old = lib.ta_blocked_set_tc_wait_ns(1)
    try:
        TB.blocked_tree_attention(q, k, v, False, None, num_samples=8, fanout=2, leaf_block=64)
        torch.cuda.synchronize()
    finally:
        lib.ta_blocked_set_tc_wait_ns(old)
    try:
        assert lib.ta_blocked_status(0) == 1
        with pytest.raises(L.TreeAttnError, match="expired"):
            TB.blocked_tree_attention(q, k, v, False, None, num_samples=8, fanout=2, leaf_block=64)
        assert lib.ta_blocked_status(0) == 0
        out = TB.blocked_tree_attention(q, k, v, False, None, num_samples=8, fanout=2, leaf_block=64)
        torch.cuda.synchronize()
        assert torch.isfinite(out).all() and lib.ta_blocked_status(0) == 0
    finally:
        lib.ta_blocked_set_tcgen05(old_tc)


def _fwd_bwd(q, k, v, go, causal, S, f, Lb, tc_bwd):
    lib = L.load()
    old = lib.ta_blocked_set_tcgen05_backward(1 if tc_bwd else 0)
    try:
        qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
        torch.manual_seed(7)
        out, blk, _ = TB.blocked_tree_attention(qq, kk, vv, causal, None, num_samples=S, fanout=f,
                                                leaf_block=Lb, return_paths=True)
        out.backward(go)
        torch.cuda.synchronize()
        return blk, qq.grad, kk.grad, vv.grad
    finally:
        lib.ta_blocked_set_tcgen05_backward(old)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,N,H,D,S,f,Lb,causal", [
    (1, 2048, 2, 64, 8, 4, 128, True),     # keys as the dV / dK MMA rows (config-3 shape)
    (2, 2048, 1, 64, 8, 2, 128, False),
    (1, 1024, 2, 128, 8, 2, 64, False),    # head_dim as the rows (config-2 shape)
    (1, 512, 3, 128, 4, 2, 64, True),      # partial tiles, blocks no pair reaches
])
def test_tcgen05_backward_matches_mma_sync(dtype, B, N, H, D, S, f, Lb, causal):
    """The tcgen05 leaf-block backward (TMEM accumulators, P from the forward's log-sum-exp)
    against the mma.sync one on the same sampled paths, at the north-star bar."""
    g = torch.Generator(device="cuda").manual_seed(N + 3 * D)
    sd = 0.5 if dtype == torch.float16 else 1.0
    q, k, v, go = (torch.randn(B, N, H, D, device="cuda", generator=g).mul(sd).to(dtype)
                   for _ in range(4))
    blk_t, *g_tc = _fwd_bwd(q, k, v, go, causal, S, f, Lb, True)
    blk_m, *g_ms = _fwd_bwd(q, k, v, go, causal, S, f, Lb, False)
    assert torch.equal(blk_t, blk_m)
    name = "bf16" if dtype == torch.bfloat16 else "f16"
    for n_, a, b in zip(("dq", "dk", "dv"), g_tc, g_ms):
        assert torch.isfinite(a).all(), n_
        assert_within(a.float().cpu().numpy(), b.float().cpu().numpy(), name, n_)


def test_tcgen05_backward_expired_wait_is_reported():
    """A 1 ns bound around the backward alone: the tcgen05 backward's first wait expires, the
    CTA drains its MMAs and frees its TMEM, and the next blocked call raises."""
    lib = L.load()
    g = torch.Generator(device="cuda").manual_seed(5)
    q, k, v, go = (torch.randn(1, 2048, 2, 64, device="cuda", generator=g).to(torch.bfloat16)
                   for _ in range(4))
    lib.ta_blocked_status(1)
    old_b = lib.ta_blocked_set_tcgen05_backward(1)
    try:
        qq = q.clone().requires_grad_(True)
        out = TB.blocked_tree_attention(qq, k, v, True, None, num_samples=8, fanout=4, leaf_block=128)
        torch.cuda.synchronize()
        old = lib.ta_blocked_set_tc_wait_ns(1)
        try:
            out.backward(go)
            torch.cuda.synchronize()
        finally:
            lib.ta_blocked_set_tc_wait_ns(old)
        assert lib.ta_blocked_status(0) == 1
        with pytest.raises(L.TreeAttnError, match="expired"):
            TB.blocked_tree_attention(q, k, v, True, None, num_samples=8, fanout=4, leaf_block=128)
        assert lib.ta_blocked_status(0) == 0
    finally:
        lib.ta_blocked_set_tcgen05_backward(old_b)
