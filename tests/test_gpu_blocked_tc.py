"""The tcgen05 (TMEM) leaf-block forward against the mma.sync one on the same sampled paths,
and its bounded-wait status word."""

import pytest
import torch

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
