"""Time the reference's own CPU path beside the oracle port on the same host (calibration).

The reference is Python and does not travel to the GPU box, so the timed CPU baseline there is
the numpy port (``oracle/tree_oracle.py``). This script, run where the TreeAttention reference
is checked out, times both on the same workload and host so the port's speed can be related
to the reference's:

    python oracle/calibrate_port.py /path/to/TreeAttention [S H D P]

Default workload: BASELINE config 1 in the reference's semantics (B=1, S=1024, H=4, d=64, bf16
inputs, 4 paths, non-causal, attn-bench adapter: Haar build + hierarchical_attention + backward).
Rows: the reference's attn-bench ``treeattn_torch`` adapter path, treeattn-cuda's autograd op on
CPU (its Python fallback), and the port. Prints one JSON line. Test infrastructure only.
"""

from __future__ import annotations

import json
import os
import statistics
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))


def _median_s(fn, warm=1, iters=5):
    for _ in range(warm):
        fn()
    ts = []
    for _ in range(iters):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts)


def main():
    ref = sys.argv[1]
    S, H, D, P = (int(x) for x in sys.argv[2:6]) if len(sys.argv) >= 6 else (1024, 4, 64, 4)
    for sub in ("treeattn-torch/src", "treeattn-cuda/src", "attn-bench/src"):
        sys.path.insert(0, os.path.join(ref, "packages", sub))
    import torch

    from attn_bench.baselines._treeattn_common import haar_internal_node_keys
    from oracle import tree_oracle as O
    import treeattn_cuda
    import treeattn_torch

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    B = 1
    q, k, v, go = (torch.randn(B, S, H, D, generator=g).to(torch.bfloat16) for _ in range(4))
    rows = {}

    def ref_step(mod):
        qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
        to = lambda t: t.transpose(0, 1).reshape(S, B, H * D)  # noqa: E731 (seq, B, E)
        k_int = haar_internal_node_keys(kk.transpose(0, 1)).reshape(S - 1, B, H * D)
        out, _ = mod.hierarchical_attention(to(qq), k_int, to(vv), num_heads=H, num_samples=P)
        out.backward(to(go))

    torch.manual_seed(0)
    rows["treeattn_torch"] = _median_s(lambda: ref_step(treeattn_torch), 1, 3)
    torch.manual_seed(0)
    rows["treeattn_cuda_cpu_fallback"] = _median_s(lambda: ref_step(treeattn_cuda), 1, 5)

    f = lambda t: t.float().transpose(0, 1).numpy()  # noqa: E731 (seq, B, H, D) float32
    qn, kn, vn, gon = f(q), f(k), f(v), f(go)
    gum = -np.log(np.random.default_rng(0).exponential(size=(O.log_n_of(S), S, B, H, P, 2))).astype(np.float32)

    def port_step():
        k_int = O.haar_internal_node_keys(kn, "bf16")
        fw = O.forward(qn, k_int, vn, gum, P)
        _, dk_int, _ = O.backward(qn, k_int, vn, gon, fw["leaf"], fw["weights"])
        O.haar_internal_node_keys_backward(dk_int)

    rows["port_single_process"] = _median_s(port_step, 1, 5)
    print(json.dumps({"workload": dict(B=B, S=S, H=H, D=D, num_samples=P, dtype="bf16"),
                      "threads": torch.get_num_threads(), "cores": os.cpu_count(),
                      "fwd_bwd_seconds": rows,
                      "tokens_per_s": {k_: B * S / t for k_, t in rows.items()}}))


if __name__ == "__main__":
    main()
