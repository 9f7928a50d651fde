"""Generate the golden fixtures in this directory by running the REFERENCE implementation.

Run in a container that has the TreeAttention reference checked out (read-only is fine):

    python tests/golden/make_golden.py /path/to/TreeAttention

It imports the reference's own packages (treeattn-torch, treeattn-cuda's autograd op and
attn-bench's Haar tree build) on CPU, drives them with seeded inputs, and records:

* ``attn_*.npz``  -- hierarchical_attention(stochastic, non-causal) fp32 at the five shapes of
  the reference's end-to-end parity test (test_harness_smoke.py:894-917; the largest shape is
  halved in sequence length to keep fixtures small): inputs, the Gumbel noise the reference
  drew (captured from ``Tensor.exponential_`` after its in-place ``log_().neg_()``), outputs,
  weights, sampled leaves / log-probs / packed bits, and autograd gradients from both
  treeattn-torch and treeattn-cuda's custom autograd path (CPU fallback).
* ``haar_*.npz``  -- haar_internal_node_keys forward + autograd backward in f32/f16/bf16.
* ``adapter_*.npz`` -- the attn-bench treeattn_cuda adapter fn(q,k,v) end to end in bshd
  (Haar build + attention + backward), fp32 and bf16.
* ``causal_*.npz`` -- treeattn-torch hierarchical_attention(is_causal=True, stochastic): the
  exact causal prefix for the first S queries and the boundary-corrected sampler for the
  rest, with its recorded noise (one (B,H,S,2) draw per query and level) and gradients.
* ``exact_*.npz`` -- mode="deterministic" (all leaves), causal and not, with gradients.

``python tests/golden/make_golden.py REF [attention|haar|adapter|causal ...]`` regenerates a subset.

The fixtures are small; the tests never need the reference at run time.
"""

from __future__ import annotations

import os
import sys

import numpy as np


def _setup(ref_root: str):
    pk = os.path.join(ref_root, "packages")
    for sub in ("treeattn-torch/src", "treeattn-cuda/src", "attn-bench/src"):
        sys.path.insert(0, os.path.join(pk, sub))


class GumbelRecorder:
    """Wrap torch.Tensor.exponential_ and keep every tensor it filled."""

    def __init__(self, torch):
        self.torch = torch
        self.tensors = []
        self._orig = torch.Tensor.exponential_

    def __enter__(self):
        orig = self._orig
        rec = self.tensors

        def patched(t, *a, **kw):
            out = orig(t, *a, **kw)
            rec.append(t)
            return out

        self.torch.Tensor.exponential_ = patched
        return self

    def __exit__(self, *exc):
        self.torch.Tensor.exponential_ = self._orig


def _np(t):
    return t.detach().float().cpu().numpy()


def make_attention(torch, out_dir):
    import treeattn_torch
    from treeattn_torch import _tree_mha
    import treeattn_cuda

    shapes = [(8, 1, 2, 16, 4), (32, 2, 2, 16, 4), (64, 1, 8, 16, 4), (128, 1, 2, 64, 8),
              (256, 1, 4, 32, 8)]
    for (L, B, H, D, S) in shapes:
        E = H * D
        torch.manual_seed(1234)
        q = torch.randn(L, B, E)
        k = torch.randn(L - 1, B, E)
        v = torch.randn(L, B, E)
        g = torch.randn(L, B, E)
        res = {"q": _np(q), "k": _np(k), "v": _np(v), "grad_out": _np(g),
               "shape": np.array([L, B, H, D, S])}
        # treeattn-torch (the reference op), seed 0 before the call as in the reference test
        qt, kt, vt = (x.clone().requires_grad_(True) for x in (q, k, v))
        torch.manual_seed(0)
        with GumbelRecorder(torch) as rec:
            out, w = treeattn_torch.hierarchical_attention(
                qt, kt, vt, num_heads=H, is_causal=False, mode="stochastic", num_samples=S)
        out.backward(g)
        res["gumbels"] = np.stack([_np(t) for t in rec.tensors])  # (log_n, L, B, H, S, 2)
        res.update(out=_np(out), weights=_np(w), dq=_np(qt.grad), dk=_np(kt.grad),
                   dv=_np(vt.grad))
        # sampled leaves / log-probs with the same noise
        torch.manual_seed(0)
        idx, lp = _tree_mha._sample_paths_non_causal(
            q.reshape(L, B, H, D), k.reshape(L - 1, B, H, D), S, L)
        res.update(leaf=idx.numpy().astype(np.int64), log_prob=_np(lp))
        # treeattn-cuda's custom autograd op (CPU fallback path) on the same seed
        qc, kc, vc = (x.clone().requires_grad_(True) for x in (q, k, v))
        torch.manual_seed(0)
        with GumbelRecorder(torch) as rec2:
            out_c, w_c = treeattn_cuda.hierarchical_attention(
                qc, kc, vc, num_heads=H, is_causal=False, mode="stochastic", num_samples=S,
                block_size=min(256, L))
        out_c.backward(g)
        np.testing.assert_array_equal(np.stack([_np(t) for t in rec2.tensors]), res["gumbels"])
        from treeattn_cuda import _autograd as ag
        torch.manual_seed(0)
        idx_c, lp_c, packed_c = ag._sample_paths_non_causal_streaming_python(
            q.reshape(L, B, H, D), k.reshape(L - 1, B, H, D), S, block_size=min(256, L),
            max_logit=1e3)
        res.update(cuda_out=_np(out_c), cuda_weights=_np(w_c), cuda_dq=_np(qc.grad),
                   cuda_dk=_np(kc.grad), cuda_dv=_np(vc.grad),
                   cuda_leaf=idx_c.numpy().astype(np.int64), cuda_log_prob=_np(lp_c),
                   cuda_packed=packed_c.numpy())
        name = os.path.join(out_dir, f"attn_L{L}_B{B}_H{H}_D{D}_S{S}.npz")
        np.savez_compressed(name, **res)
        print("wrote", name)


def make_causal(torch, out_dir):
    """Causal stochastic mode (hybrid exact prefix + corrected sampler) and exact mode."""
    import treeattn_torch

    for (L, B, H, D, S) in [(4, 1, 2, 16, 4), (16, 1, 2, 16, 4), (32, 2, 2, 16, 8),
                            (64, 1, 2, 32, 4)]:
        E = H * D
        torch.manual_seed(4321)
        q = torch.randn(L, B, E)
        k = torch.randn(L - 1, B, E)
        v = torch.randn(L, B, E)
        g = torch.randn(L, B, E)
        qt, kt, vt = (x.clone().requires_grad_(True) for x in (q, k, v))
        torch.manual_seed(0)
        with GumbelRecorder(torch) as rec:
            out, w = treeattn_torch.hierarchical_attention(
                qt, kt, vt, num_heads=H, is_causal=True, mode="stochastic", num_samples=S)
        out.backward(g)
        log_n = (L - 1).bit_length()
        lsto = L - S if L > S else L
        gum = np.stack([_np(t) for t in rec.tensors]).reshape(lsto, log_n, B, H, S, 2)
        fn = os.path.join(out_dir, f"causal_L{L}_B{B}_H{H}_D{D}_S{S}.npz")
        np.savez_compressed(fn, q=_np(q), k=_np(k), v=_np(v), grad_out=_np(g), gumbels=gum,
                            out=_np(out), weights=_np(w), dq=_np(qt.grad), dk=_np(kt.grad),
                            dv=_np(vt.grad), shape=np.array([L, B, H, D, S]))
        print("wrote", fn)
    for causal in (False, True):
        for (L, B, H, D) in [(16, 1, 2, 16), (32, 2, 2, 16)]:
            E = H * D
            torch.manual_seed(99)
            q = torch.randn(L, B, E)
            k = torch.randn(L - 1, B, E)
            v = torch.randn(L, B, E)
            g = torch.randn(L, B, E)
            qt, kt, vt = (x.clone().requires_grad_(True) for x in (q, k, v))
            out, w = treeattn_torch.hierarchical_attention(
                qt, kt, vt, num_heads=H, is_causal=causal, mode="deterministic")
            out.backward(g)
            fn = os.path.join(out_dir, f"exact_{'causal' if causal else 'full'}_L{L}_B{B}_H{H}_D{D}.npz")
            np.savez_compressed(fn, q=_np(q), k=_np(k), v=_np(v), grad_out=_np(g), out=_np(out),
                                weights=_np(w), dq=_np(qt.grad), dk=_np(kt.grad), dv=_np(vt.grad),
                                shape=np.array([L, B, H, D]))
            print("wrote", fn)


def make_haar(torch, out_dir):
    from attn_bench.baselines._treeattn_common import haar_internal_node_keys

    dts = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
    for S, B, H, D in [(8, 1, 1, 4), (64, 2, 2, 16), (256, 1, 3, 32)]:
        for name, dt in dts.items():
            torch.manual_seed(7)
            k = torch.randn(S, B, H, D).to(dt)
            gk = torch.randn(S - 1, B, H, D).to(dt)
            kk = k.clone().requires_grad_(True)
            out = haar_internal_node_keys(kk)
            out.backward(gk)
            fn = os.path.join(out_dir, f"haar_{name}_S{S}_B{B}_H{H}_D{D}.npz")
            np.savez_compressed(fn, k=_np(k), out=_np(out), grad_in=_np(gk), grad_k=_np(kk.grad))
            print("wrote", fn)


def make_adapter(torch, out_dir):
    from attn_bench.baselines import treeattn_cuda as ad_cuda

    os.environ["TREEATTN_NUM_SAMPLES"] = "4"
    dts = {"f32": torch.float32, "bf16": torch.bfloat16}
    for (B, S, H, D) in [(1, 64, 2, 32), (2, 128, 2, 16)]:
        for name, dt in dts.items():
            torch.manual_seed(5)
            q = torch.randn(B, S, H, D).to(dt)
            k = torch.randn(B, S, H, D).to(dt)
            v = torch.randn(B, S, H, D).to(dt)
            g = torch.randn(B, S, H, D).to(dt)
            qq, kk, vv = (x.clone().requires_grad_(True) for x in (q, k, v))
            torch.manual_seed(11)
            with GumbelRecorder(torch) as rec:
                out = ad_cuda._call(qq, kk, vv, False, None)
            out.backward(g)
            fn = os.path.join(out_dir, f"adapter_{name}_B{B}_S{S}_H{H}_D{D}.npz")
            np.savez_compressed(
                fn, q=_np(q), k=_np(k), v=_np(v), grad_out=_np(g), num_samples=np.array(4),
                gumbels=np.stack([_np(t) for t in rec.tensors]), out=_np(out),
                dq=_np(qq.grad), dk=_np(kk.grad), dv=_np(vv.grad))
            print("wrote", fn)


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("TREEATTN_REFERENCE_ROOT")
    if not ref_root:
        raise SystemExit("usage: make_golden.py /path/to/TreeAttention")
    _setup(ref_root)
    import torch

    torch.set_num_threads(min(8, os.cpu_count() or 1))
    out_dir = os.path.dirname(os.path.abspath(__file__))
    which = sys.argv[2:] or ["attention", "haar", "adapter", "causal"]
    if "attention" in which:
        make_attention(torch, out_dir)
    if "haar" in which:
        make_haar(torch, out_dir)
    if "adapter" in which:
        make_adapter(torch, out_dir)
    if "causal" in which:
        make_causal(torch, out_dir)


if __name__ == "__main__":
    main()
