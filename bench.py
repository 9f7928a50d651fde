#!/usr/bin/env python
"""Benchmark: fwd+bwd tokens/s of stochastic tree attention on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one forward + backward pass of the attn-bench kernel contract
``tree_attention(q, k, v)`` on bshd bf16 tensors: Haar tree build from k, fused Gumbel-max
path sampling + softmax + value gather, deterministic backward (dq, dk, dv) and the
transposed tree build. Workload (the headline metric "S=16k, d=128 bf16"): B=1 per GPU,
S=16384, H=16, d=128, 8 sampled paths per query, reference tree semantics (binary tree, one
token per leaf). Inputs q, k, v, grad_out ~ N(0, 1) from a seeded CUDA generator.

N > 1 (torchrun, one process per GPU, NCCL): the (batch, head) trees are independent, so
every rank runs its own batch element with no data-path collective (weak scaling); the
timed region is bracketed by barriers and the max over ranks is reported.

``--impl reference`` times the CPU oracle (numpy restatement of the reference, forked over
all host cores by head) on a bounded sample of the same workload and extrapolates to a full
step. Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "fwd+bwd tokens/s/GPU at S=16k,d=128 bf16; % of HBM/tensor roofline; vs FA2"
WORKLOAD = dict(workload="stochastic tree attention fwd+bwd (attn-bench bshd contract), "
                         "reference semantics: binary tree, 1 token per leaf",
                batch_per_gpu=1, seq_len=16384, heads=16, head_dim=128, num_samples=8,
                dtype="bf16")


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--seq-len", type=int, default=WORKLOAD["seq_len"])
    p.add_argument("--heads", type=int, default=WORKLOAD["heads"])
    p.add_argument("--head-dim", type=int, default=WORKLOAD["head_dim"])
    p.add_argument("--num-samples", type=int, default=WORKLOAD["num_samples"])
    p.add_argument("--batch", type=int, default=WORKLOAD["batch_per_gpu"])
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-fa2", action="store_true")
    p.add_argument("--fanout", type=int, default=2)
    p.add_argument("--leaf-block", type=int, default=64)
    p.add_argument("--causal", action="store_true")
    p.add_argument("--dtype", choices=["bf16", "f16"], default="bf16")
    p.add_argument("--mode", choices=["shard", "sp", "blocked"], default="shard",
                   help="shard: (batch, head)-sharded headline workload; sp: sequence-parallel "
                        "causal long context (B=1, S=65536, H=32, d=128, 16 paths unless overridden); "
                        "blocked: generalised fanout / leaf-block tree (B=4, S=4096, H=16, d=128, "
                        "fanout 2, leaf block 64, 8 paths: the single-B200 benchmark config)")
    return p.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        rows = [r.split(",") for r in self.file.read().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        load = [x for x in sm if mx and x > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------------------
# algorithmic bytes per launch (compulsory unique traffic of each kernel)
# ---------------------------------------------------------------------------------------
def algorithmic_bytes(kernel: str, B, S, H, D, P, elt, launches_per_step):
    rows = B * S * H * D * elt          # one (B, S, H, D) tensor
    paths = B * S * H * P
    table = {
        # read q, k_int, v; write out; write leaf + weight per path
        "fwd_fused": 4 * rows + 8 * paths,
        # the walk alone: read q, k_int; write leaf + weight per path
        "fwd_walk": 2 * rows + 8 * paths,
        # read v, leaf + weight per path; write out
        "value_sum": 2 * rows + 8 * paths,
        # read q, dO, k_int, v, leaf + weight; write dq
        "bwd_query": 5 * rows + 8 * paths,
        # read q, dO per path-sorted chunk; write dk (float32) and dv
        "bwd_node": 2 * rows + B * S * H * D * 4 + rows,
        # read k, write k_int (all passes of one step, split evenly over its launches)
        "tree_build": 2 * rows / max(1, launches_per_step),
        # read dk_int (float32), write dk
        "tree_build_bwd": (B * S * H * D * 4 + rows) / max(1, launches_per_step),
    }
    return table.get(kernel)


# ---------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)

    import treeattn_b200 as ta
    from treeattn_b200 import ops

    B, S, H, D, P = args.batch, args.seq_len, args.heads, args.head_dim, args.num_samples
    dtype = torch.bfloat16
    gen = torch.Generator(device=dev).manual_seed(1000 * rank)
    q, k, v, go = (torch.randn(B, S, H, D, device=dev, generator=gen).to(dtype) for _ in range(4))
    for t in (q, k, v):
        t.requires_grad_(True)
    # every rank draws its slice of ONE global problem's noise (same seed everywhere), so
    # the N-rank run computes exactly what one GPU would on the global batch
    from treeattn_b200.sharding import shard_for_rank
    shard = shard_for_rank(world * B, H, rank, world, "batch") if world > 1 else None
    torch.manual_seed(0)

    def step():
        for t in (q, k, v):
            t.grad = None
        out = ta.tree_attention(q, k, v, False, None, num_samples=P, shard=shard)
        out.backward(go)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    barrier()
    stream = torch.cuda.current_stream(dev)
    clocks = ClockSampler(dev.index)
    ops.profile_enable(True)
    clocks.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    barrier()
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    barrier()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1)
    prof = ops.profile_collect()
    ops.profile_enable(False)
    if world > 1:
        tm = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        ms = float(tm.item())
    ms_step = ms / args.steps
    tokens_step = world * B * S
    value = tokens_step / (ms_step / 1e3)

    # end to end through the public API with host buffers: every step uploads its inputs from
    # pinned host memory and downloads its output and gradients. Uploads run on a copy-in
    # stream into two alternating device buffers, downloads on a copy-out stream, so step i+1's
    # upload and step i-1's download overlap step i's kernels; the events bracket all of it.
    e2e = None
    if not args.no_e2e:
        hq, hk, hv, hgo = (t.detach().cpu().pin_memory() for t in (q, k, v, go))
        hout, hdq, hdk, hdv = (torch.empty_like(hq).pin_memory() for _ in range(4))
        bufs = [[torch.empty_like(t) for t in (q, k, v, go)] for _ in range(2)]
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        free = [None, None]  # event: compute done with buffer i

        def step_e2e(i):
            buf = bufs[i % 2]
            with torch.cuda.stream(s_in):
                if free[i % 2] is not None:
                    s_in.wait_event(free[i % 2])
                for dst, src in zip(buf, (hq, hk, hv, hgo)):
                    dst.copy_(src, non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(s_in)
            stream.wait_event(ready)
            dq_, dk_, dv_ = (t.detach().requires_grad_(True) for t in buf[:3])
            out = ta.tree_attention(dq_, dk_, dv_, False, None, num_samples=P, shard=shard)
            out.backward(buf[3])
            done = torch.cuda.Event()
            done.record(stream)
            free[i % 2] = done
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                for dst, src in ((hout, out), (hdq, dq_.grad), (hdk, dk_.grad), (hdv, dv_.grad)):
                    src.record_stream(s_out)
                    dst.copy_(src.detach(), non_blocking=True)

        def drain():
            fin = torch.cuda.Event()
            fin.record(s_out)
            stream.wait_event(fin)

        for i in range(max(1, args.warmup)):
            step_e2e(i)
        drain()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        s_in.wait_event(e0)
        for i in range(args.steps):
            step_e2e(i)
        drain()
        e1.record(stream)
        barrier()
        ems = e0.elapsed_time(e1)
        if world > 1:
            tm = torch.tensor([ems], device=dev, dtype=torch.float64)
            dist.all_reduce(tm, op=dist.ReduceOp.MAX)
            ems = float(tm.item())
        nbytes = hq.numel() * hq.element_size()
        e2e = {"value": tokens_step / (ems / args.steps / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": 4 * nbytes, "d2h_bytes_per_step": 4 * nbytes,
               "ms_per_step": ems / args.steps}

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    # kernel shares and the dominant kernel's roofline
    total = sum(v[1] for v in prof.values()) or 1.0
    kernels = {n: {"launches_per_step": c / args.steps, "ms_per_step": t / args.steps,
                   "share": t / total} for n, (c, t) in sorted(prof.items(), key=lambda x: -x[1][1])}
    top = max(prof.items(), key=lambda x: x[1][1])[0] if prof else None
    hbm, peak_kind = peaks()
    roof = None
    if top is not None:
        cnt, tms = prof[top]
        per_launch_s = tms / cnt / 1e3
        lps = cnt / args.steps
        alg = algorithmic_bytes(top, B, S, H, D, P, 2, lps)
        achieved = alg / per_launch_s / 1e9 if alg else None
        traffic = None
        tpath = os.path.join(ROOT, "profiles", "traffic_per_launch.json")
        if os.path.exists(tpath):
            with open(tpath) as f:
                traffic = json.load(f).get(top)
        roof = {"kernel": top, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm if achieved else None, "traffic": traffic,
                "peak_source": f"{peak_kind} MEASURED_PEAKS.json hbm_gbs" if peak_kind == "measured"
                else "fallback 6.65 TB/s",
                "algorithmic_bytes_per_launch": alg, "launch_ms": tms / cnt}
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic N(0,1) q/k/v/grad_out from a seeded CUDA generator",
        "config": {**WORKLOAD, "batch_per_gpu": B, "seq_len": S, "heads": H, "head_dim": D,
                   "num_samples": P, "global_batch": world * B,
                   "parallelism": f"batch-sharded x{world} (independent (batch, head) trees, no collective; "
                                  "each rank draws its slice of the global problem's noise)",
                   "l2": "inputs larger than L2 (q, k, v, grad_out: 4 x %d MiB)" % (B * S * H * D * 2 >> 20)},
        "value_per_gpu": value / world,
        "gpu_launches": int(sum(c for c, _ in prof.values())),
        "kernels": kernels,
        "roofline": roof,
        "clocks": clk,
        "e2e": e2e,
    }
    if world == 1 and not args.no_fa2:
        line["fa2"] = fa2_reference(q.detach(), k.detach(), v.detach(), go, args)
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_reference(args, budget_s=20.0)
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def fa2_reference(q, k, v, go, args):
    """Dense FlashAttention-2 (flash_attn library, the metric's comparator) fwd+bwd on the
    same bshd tensors and GPU: tokens/s, CUDA events, same warm-up / step counts."""
    import torch
    try:
        from flash_attn import flash_attn_func
    except Exception as exc:  # noqa: BLE001 - a comparator only
        return {"unavailable": f"flash_attn not importable: {exc}"}
    qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))

    def step():
        for t in (qq, kk, vv):
            t.grad = None
        flash_attn_func(qq, kk, vv, causal=False).backward(go)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    B, S = q.shape[0], q.shape[1]
    return {"value": B * S / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
            "what": "flash_attn_func dense attention fwd+bwd, same bshd bf16 q/k/v/grad_out, "
                    "non-causal (library comparator, not this package's path)"}


# ---------------------------------------------------------------------------------------
# CPU arm: the numpy oracle (a port of the reference; the reference itself is Python and
# does not travel), forked over heads on every host core
# ---------------------------------------------------------------------------------------
_SHARED = {}


def _cpu_heads(hs):
    """Oracle work for heads [hs[0], hs[1]): (tree-build seconds, query seconds)."""
    from oracle import tree_oracle as O

    d = _SHARED
    sl = slice(hs[0], hs[1])
    t0 = time.perf_counter()
    k_int = O.haar_internal_node_keys(d["k"][:, :, sl], "bf16")
    O.haar_internal_node_keys_backward(np.zeros_like(k_int))
    t1 = time.perf_counter()
    q, v, go, g = d["q"][:, :, sl], d["v"][:, :, sl], d["go"][:, :, sl], d["g"][:, :, :, sl]
    fw = O.forward(q, k_int, v, g, d["P"])
    O.backward(q, k_int, v, go, fw["leaf"], fw["weights"])
    t2 = time.perf_counter()
    return t1 - t0, t2 - t1


def cpu_reference(args, budget_s=20.0):
    """Time the oracle on all S tree nodes but only Ls queries; extrapolate to a full step.

    Each worker process owns a slice of the heads and times the tree build (all S keys) and
    the fwd+bwd of the Ls sampled queries separately; a full step is
    max(build) + max(query) * S / Ls.
    """
    import multiprocessing as mp

    sys.path.insert(0, ROOT)
    from oracle import tree_oracle as O

    B, S, H, D, P = 1, args.seq_len, args.heads, args.head_dim, args.num_samples
    rng = np.random.default_rng(0)
    Ls = 64
    rb = lambda *s: O.round_to_bf16(rng.standard_normal(s, dtype=np.float32))  # noqa: E731
    _SHARED.update(q=rb(Ls, B, H, D), k=rb(S, B, H, D), v=rb(S, B, H, D), go=rb(Ls, B, H, D),
                   g=-np.log(rng.exponential(size=(O.log_n_of(S), Ls, B, H, P, 2)).astype(np.float32)),
                   P=P)
    cores = min(os.cpu_count() or 1, H)
    chunks = [(i * H // cores, (i + 1) * H // cores) for i in range(cores)]
    ctx = mp.get_context("fork")
    samples = []
    with ctx.Pool(cores) as pool:
        deadline = time.perf_counter() + budget_s
        while True:
            res = pool.map(_cpu_heads, chunks)
            samples.append((max(r[0] for r in res), max(r[1] for r in res)))
            if time.perf_counter() > deadline or len(samples) >= 3:
                break
    t_build = min(s[0] for s in samples)
    t_query = min(s[1] for s in samples)
    t_step = t_build + t_query * (S / Ls)
    return {"value": B * S / t_step, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"numpy oracle (oracle/tree_oracle.py), Haar build + transpose of all {S} keys "
                      f"and fwd+bwd of {Ls} of {S} queries x {H} heads, {cores} processes over heads; "
                      f"step = build + query part x {S // Ls}",
            "build_s": t_build, "query_sample_s": t_query, "extrapolated_step_s": t_step}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    r = cpu_reference(args, budget_s=30.0)
    vals = [r["value"]]
    value = r["value"]
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": args.seq_len / value * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic N(0,1), bf16-rounded", "config": {**WORKLOAD, "batch_per_gpu": 1},
            "cpu_baseline": {**r, "value": value},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_sp(args):
    """Sequence-parallel causal long context: the global problem is fixed and split over the
    ranks by sequence position (strong scaling). N=1 runs the plain causal op."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    import treeattn_b200 as ta
    from treeattn_b200 import ops
    from treeattn_b200.sequence_parallel import sp_tree_attention

    d = dict(seq_len=65536, heads=32, num_samples=16)
    S = args.seq_len if args.seq_len != WORKLOAD["seq_len"] else d["seq_len"]
    H = args.heads if args.heads != WORKLOAD["heads"] else d["heads"]
    P = args.num_samples if args.num_samples != WORKLOAD["num_samples"] else d["num_samples"]
    B, D, n = 1, args.head_dim, S // world
    gen = torch.Generator(device=dev).manual_seed(0)
    full = [torch.randn(B, S, H, D, device=dev, generator=gen).to(torch.bfloat16) for _ in range(4)]
    sl = slice(rank * n, (rank + 1) * n)
    q, k, v, go = (t[:, sl].contiguous() for t in full)
    del full
    for t in (q, k, v):
        t.requires_grad_(True)

    def step():
        for t in (q, k, v):
            t.grad = None
        torch.manual_seed(0)
        if world > 1:
            out = sp_tree_attention(q, k, v, True, num_samples=P)
        else:
            out = ta.tree_attention(q, k, v, True, None, num_samples=P)
        out.backward(go)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    barrier()
    clocks = ClockSampler(dev.index)
    ops.profile_enable(True)
    clocks.start()
    stream = torch.cuda.current_stream(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    barrier()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1)
    prof = ops.profile_collect()
    ops.profile_enable(False)
    if world > 1:
        tm = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        ms = float(tm.item())
    ms_step = ms / args.steps
    if rank == 0:
        total = sum(t for _, t in prof.values()) or 1.0
        line = {"metric": "causal long-context fwd+bwd tokens/s (sequence parallel)",
                "value": B * S / (ms_step / 1e3), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic N(0,1) q/k/v/grad_out from a seeded CUDA generator",
                "config": {"workload": "stochastic tree attention, causal (exact prefix + corrected "
                                       "sampler), sequence split over ranks", "batch": B, "seq_len": S,
                           "heads": H, "head_dim": D, "num_samples": P,
                           "parallelism": f"sequence-parallel x{world}: NCCL all-gather of K/V, "
                                          "reduce-scatter of dK/dV"},
                "gpu_launches": int(sum(c for c, _ in prof.values())),
                "kernels": {k_: {"launches_per_step": c / args.steps, "ms_per_step": t / args.steps,
                                 "share": t / total} for k_, (c, t) in
                            sorted(prof.items(), key=lambda x: -x[1][1])},
                "clocks": clk}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_blocked(args):
    """Generalised tree (fanout, leaf block), one GPU or (batch, head)-sharded ranks."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    from treeattn_b200 import ops
    from treeattn_b200.blocked import blocked_tree_attention
    from treeattn_b200.sharding import shard_for_rank

    S = args.seq_len if args.seq_len != WORKLOAD["seq_len"] else 4096
    B = args.batch if args.batch != WORKLOAD["batch_per_gpu"] else 4
    H, D, P = args.heads, args.head_dim, args.num_samples
    f, Lb = args.fanout, args.leaf_block
    dt = torch.bfloat16 if args.dtype == "bf16" else torch.float16
    sd = 1.0 if dt == torch.bfloat16 else 0.5
    gen = torch.Generator(device=dev).manual_seed(1000 * rank)
    q, k, v, go = (torch.randn(B, S, H, D, device=dev, generator=gen).mul(sd).to(dt) for _ in range(4))
    for t in (q, k, v):
        t.requires_grad_(True)
    shard = shard_for_rank(world * B, H, rank, world, "batch") if world > 1 else None

    def step():
        for t in (q, k, v):
            t.grad = None
        torch.manual_seed(0)
        out = blocked_tree_attention(q, k, v, args.causal, None, num_samples=P, fanout=f,
                                     leaf_block=Lb, shard=shard)
        out.backward(go)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    barrier()
    clocks = ClockSampler(dev.index)
    ops.profile_enable(True)
    clocks.start()
    stream = torch.cuda.current_stream(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    barrier()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1)
    prof = ops.profile_collect()
    ops.profile_enable(False)
    if world > 1:
        tm = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        ms = float(tm.item())
    ms_step = ms / args.steps
    if rank == 0:
        # leaf-block attention FLOPs (QK^T and PV per sampled path; backward 2.5x)
        leaf_flops = B * S * H * P * Lb * D * 4.0 * 3.5
        total = sum(t for _, t in prof.values()) or 1.0
        line = {"metric": "generalised tree attention fwd+bwd tokens/s (fanout, leaf block)",
                "value": world * B * S / (ms_step / 1e3), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": args.dtype,
                "data": "synthetic N(0,1) (fp16: N(0,0.5)) q/k/v/grad_out, seeded CUDA generator",
                "config": {"workload": "stochastic tree attention, generalised tree", "batch_per_gpu": B,
                           "seq_len": S, "heads": H, "head_dim": D, "num_samples": P, "fanout": f,
                           "leaf_block": Lb, "causal": args.causal},
                "leaf_block_tflops": leaf_flops / (ms_step / 1e3) / 1e12,
                "gpu_launches": int(sum(c for c, _ in prof.values())),
                "kernels": {k_: {"launches_per_step": c / args.steps, "ms_per_step": t / args.steps,
                                 "share": t / total} for k_, (c, t) in
                            sorted(prof.items(), key=lambda x: -x[1][1])},
                "clocks": clk}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse_args()
    sys.path.insert(0, ROOT)
    if args.impl == "reference":
        run_reference(args)
    elif args.mode == "sp":
        run_sp(args)
    elif args.mode == "blocked":
        run_blocked(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
