"""CPU-side checks: the C-ABI library loads and exports every declared symbol; host logic."""

import ctypes
import os
import re

import pytest
import torch

import treeattn_b200 as ta
from treeattn_b200 import _lib, ops
from tests.conftest import ROOT


def _declared_symbols():
    syms = set()
    for name in os.listdir(os.path.join(ROOT, "include")):
        if name.endswith(".h"):
            text = open(os.path.join(ROOT, "include", name)).read()
            syms |= set(re.findall(r"^\S[^;(]*?\b(ta_\w+)\s*\(", text, flags=re.M))
    return syms


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared_symbols()
    assert {"ta_forward", "ta_backward", "ta_tree_build", "ta_tree_build_backward",
            "ta_sample_paths"} <= declared
    for s in declared:
        assert hasattr(lib, s), s
        assert s in _lib.SIGNATURES, f"{s} missing from the ctypes signature table"
    assert lib.ta_abi_version() == 1


def test_philox_plan_matches_torch_policy():
    # torch calc_execution_policy: block 256, grid <= SMs * (maxThreads/256), 4 per trip
    for numel, sms, mt in [(16, 148, 2048), (4194304, 148, 2048), (303104, 148, 2048),
                           (303105, 148, 2048), (10**8, 132, 2048), (1, 108, 2048)]:
        grid = min(sms * (mt // 256), (numel + 255) // 256)
        step = ((numel - 1) // (256 * grid * 4) + 1) * 4
        assert ops.philox_plan(numel, sms, mt) == (step, 256 * grid)


def test_invalid_arguments_report_errors_without_a_gpu():
    lib = _lib.load()
    shape = _lib.Shape(1, 8, 7, 1, 16, 4, _lib.TA_F32, 1e3)  # N=7: not a power of two
    lay = _lib.Layout(16, 16, 16)
    rc = lib.ta_forward(ctypes.byref(shape), None, lay, None, lay, None, lay, None, lay, None,
                        None, None, None, None, None, None)
    assert rc == _lib.TA_ERR_UNSUPPORTED
    assert b"power of two" in lib.ta_last_error()
    shape.num_leaves = 8
    rc = lib.ta_forward(ctypes.byref(shape), None, lay, None, lay, None, lay, None, lay, None,
                        None, None, None, None, None, None)
    assert rc == _lib.TA_ERR_INVALID and b"q is NULL" in lib.ta_last_error()
    shape.head_dim = 6  # 24 bytes: not a 16-byte multiple
    assert lib.ta_backward_workspace_size(ctypes.byref(shape)) == 0
    with pytest.raises(ValueError):
        _lib.call("ta_philox_plan", 0, 148, 2048, ctypes.byref(ctypes.c_uint64()),
                  ctypes.byref(ctypes.c_int64()))
    assert lib.ta_tree_build(_lib.TA_BF16, 1, 6, 1, 8, None, lay, None, lay, None, 0, None) \
        == _lib.TA_ERR_INVALID


def test_workspace_sizes():
    lib = _lib.load()
    shape = _lib.Shape(1, 16384, 16384, 16, 128, 8, _lib.TA_BF16, 1e3)
    ws = lib.ta_backward_workspace_size(ctypes.byref(shape))
    P = 16384 * 8 * 16
    assert ws >= P * 4 * 4 + P * 4  # records (2 buffers x key/val) + per-path dlp
    assert lib.ta_tree_build_workspace_size(1, 16384, 16, 128, _lib.TA_BF16) > 0
    assert lib.ta_tree_build_workspace_size(1, 32, 16, 128, _lib.TA_BF16) == 0


def test_ops_refuse_cpu_tensors():
    q = torch.randn(8, 1, 2, 16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.forward(q, q[:7], q, 4)
    with pytest.raises(ValueError, match="CUDA"):
        ops.tree_build(q)


def test_hierarchical_attention_argument_errors():
    q = torch.randn(8, 1, 32)
    with pytest.raises(ValueError, match="N-1"):
        ta.hierarchical_attention(q, torch.randn(6, 1, 32), q, num_heads=2, num_samples=4)
    with pytest.raises(ValueError, match="divisible"):
        ta.hierarchical_attention(q, torch.randn(7, 1, 32), q, num_heads=3, num_samples=4)
    with pytest.raises(ValueError, match="num_samples"):
        ta.hierarchical_attention(q, torch.randn(7, 1, 32), q, num_heads=2, num_samples=0)
    with pytest.raises(ValueError, match="shape"):
        ta.hierarchical_attention(q[0], torch.randn(7, 32), q, num_heads=2)
    with pytest.raises(ValueError, match="mode"):
        ta.hierarchical_attention(q, torch.randn(7, 1, 32), q, num_heads=2, mode="other")
    # degenerate trees are handled without kernels, as in the reference (_autograd.py:660-683)
    v1 = torch.randn(1, 1, 32)
    out, w = ta.hierarchical_attention(q, torch.empty(0, 1, 32), v1, num_heads=2, num_samples=4)
    assert torch.equal(out, v1.expand(8, 1, 32)) and w.shape == (8, 1, 2, 1)
    out, w = ta.hierarchical_attention(q, torch.empty(0, 1, 32), torch.empty(0, 1, 32), num_heads=2)
    assert torch.equal(out, torch.zeros_like(q)) and w.shape == (8, 1, 2, 0)


def test_num_samples_env(monkeypatch):
    monkeypatch.setenv("TREEATTN_NUM_SAMPLES", "8")
    assert ta.resolve_num_samples() == 8
    monkeypatch.setenv("TREEATTN_NUM_SAMPLES", "0")
    assert ta.resolve_num_samples() is None
    monkeypatch.setenv("TREEATTN_NUM_SAMPLES", "x")
    with pytest.raises(ValueError):
        ta.resolve_num_samples()
    monkeypatch.delenv("TREEATTN_NUM_SAMPLES")
    q = torch.randn(1, 8, 2, 16)
    with pytest.raises(ValueError, match="num_samples"):
        ta.tree_attention(q, q, q)
    with pytest.raises(ValueError, match="power-of-two"):
        ta.tree_attention(q[:, :6], q[:, :6], q[:, :6], num_samples=4)


def test_bench_adapter_metadata():
    from treeattn_b200.bench import adapter

    a = adapter()
    assert a.name == "treeattn_b200" and a.layout == "bshd" and a.supports_backward
    assert a.is_compatible(torch.bfloat16, 128, False)[0]
    assert a.is_compatible(torch.bfloat16, 128, True)[0]


def test_tree_aware_accounting():
    from treeattn_b200 import bench as tb
    from_dense = 4.0 * 1 * 16 * 16384 * 16384 * 128
    f = tb.fwd_flops(1, 16384, 16, 128, False, 8)
    assert f == 16384 * 16 * 8 * 15 * 2 * 128
    assert f < from_dense / 100
    assert tb.bwd_flops(1, 16384, 16, 128, False, 8) > f
    assert tb.compulsory_bytes(1, 16384, 16, 128) == 12 * 16384 * 16 * 128 * 2


def test_library_sources_have_no_blocking_calls():
    """The attn-bench contract forbids host synchronisation in the hot path: no kernel-path
    source calls a synchronising CUDA API. Allowed: the profiler's collection call
    (ta_profile_collect, off the hot path) and the one-time pinned allocation of the tcgen05
    status word. (cudaStreamWaitEvent, which orders two streams on the device without blocking
    the host, is allowed: the backward forks its path sort onto a side stream.)"""
    csrc = os.path.join(ROOT, "treeattn_b200", "csrc")
    banned = re.compile(r"\b(cudaDeviceSynchronize|cudaStreamSynchronize|cudaMemcpy|cudaMemcpy2D|"
                        r"cudaMemset|cudaMalloc|cudaFree|cudaEventSynchronize)\s*\(")
    allowed = {("ta_capi.cu", "cudaEventSynchronize")}
    found = []
    for name in sorted(os.listdir(csrc)):
        text = open(os.path.join(csrc, name)).read()
        text = re.sub(r"//[^\n]*", "", text)
        for m in banned.finditer(text):
            if (name, m.group(1)) not in allowed:
                found.append((name, m.group(1)))
    assert not found, found


def test_blocked_status_word_readable_without_a_gpu():
    lib = _lib.load()
    assert lib.ta_blocked_status(0) == 0
    old = lib.ta_blocked_set_tc_wait_ns(5)
    assert lib.ta_blocked_set_tc_wait_ns(old) == 5
