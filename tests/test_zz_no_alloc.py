"""ta_tree_build_noalloc: the tree build with fixed device scratch instead of a workspace.

Named to be collected last, so it also runs after every other test has used the library.
The GPU tests call the C ABI directly and compare with ta_tree_build (caller workspace) on
two calls in a row; the build is bit-exact, so the tolerance is zero.
"""

import pytest
import torch

from treeattn_b200 import _lib as L
from treeattn_b200 import ops

SCRATCH_BYTES = 8 << 20  # TA_NOALLOC_SCRATCH_BYTES


def _noalloc(k: torch.Tensor) -> torch.Tensor:
    S, B, H, D = k.shape
    out = torch.empty((B, H, S - 1, D), device=k.device, dtype=k.dtype).permute(2, 0, 1, 3)
    L.call("ta_tree_build_noalloc", ops.dtype_code(k.dtype), B, S, H, D, ops._ptr(k),
           ops.layout(k), ops._ptr(out), ops.layout(out), ops._stream(k.device))
    return out


def test_rejects_shape_beyond_scratch():
    lib = L.load()
    B, S, H, D = 1, 1 << 20, 16, 128
    assert lib.ta_tree_build_workspace_size(B, S, H, D, L.TA_BF16) > SCRATCH_BYTES
    lay = L.Layout(B * H * D, H * D, D)
    rc = lib.ta_tree_build_noalloc(L.TA_BF16, B, S, H, D, None, lay, None, lay, None)
    assert rc == L.TA_ERR_WORKSPACE
    assert b"ta_tree_build_noalloc" in lib.ta_last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,B,S,H,D", [
    (torch.bfloat16, 1, 16384, 16, 128),   # 4.2 MB of scratch: three passes
    (torch.float32, 2, 4096, 4, 64),
    (torch.float16, 1, 32, 2, 64),         # one pass, no scratch used
])
def test_matches_workspace_build_twice(dtype, B, S, H, D):
    lib = L.load()
    assert lib.ta_tree_build_workspace_size(B, S, H, D, ops.dtype_code(dtype)) <= SCRATCH_BYTES
    gen = torch.Generator(device="cuda").manual_seed(1234 + S)
    for call in range(2):  # fresh inputs each call: stale scratch must not leak through
        k = torch.randn(S, B, H, D, device="cuda", generator=gen).to(dtype)
        want = ops.tree_build(k)
        got = _noalloc(k)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16 if dtype != torch.float32 else torch.int32),
                           want.view(torch.int16 if dtype != torch.float32 else torch.int32)), \
            f"call {call} differs"


@pytest.mark.gpu
def test_bshd_view_input():
    B, S, H, D = 2, 2048, 8, 128
    x = torch.randn(B, S, H, D, device="cuda", dtype=torch.bfloat16)
    k = x.transpose(0, 1)  # (S, B, H, D) view of bshd memory
    torch.testing.assert_close(_noalloc(k), ops.tree_build(k), rtol=0, atol=0)
    torch.testing.assert_close(_noalloc(k), ops.tree_build(k), rtol=0, atol=0)
