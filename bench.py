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
all host cores by head) over whole steps of a subset of the heads (every query, the full
tree), sized so that the run takes a few minutes; throughput is quoted for the full config.
Rank 0 prints one JSON line.
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
    p.add_argument("--no-extra", action="store_true",
                   help="skip the config-3 (head-sharded generalised tree) and config-4 "
                        "(sequence-parallel causal) records of the default line")
    p.add_argument("--fanout", type=int, default=2)
    p.add_argument("--leaf-block", type=int, default=64)
    p.add_argument("--causal", action="store_true")
    p.add_argument("--dtype", choices=["bf16", "f16"], default="bf16")
    p.add_argument("--mode", choices=["shard", "sp", "blocked", "sweep"], default="shard",
                   help="shard: (batch, head)-sharded headline workload; sp: sequence-parallel "
                        "causal long context (B=1, S=65536, H=32, d=128, 16 paths unless overridden); "
                        "blocked: generalised fanout / leaf-block tree (B=4, S=4096, H=16, d=128, "
                        "fanout 2, leaf block 64, 8 paths: the single-B200 benchmark config); "
                        "sweep: the attn-bench-style sweep of config 5 against FA2")
    return p.parse_args()


def tensor_peak():
    """Dense 16-bit tensor peak in TFLOP/s: the measured burst cuBLAS figure (a kernel timed
    inside a step of a few ms), else the fallback."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        if "bf16_tflops" in d:
            return float(d["bf16_tflops"]), "measured MEASURED_PEAKS.json bf16_tflops (burst)"
    return 1590.0, "fallback 1.59 PFLOP/s"


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


def bind_local_cpus(dev) -> dict:
    """Pin this process to the host cores of its GPU's NUMA node (sysfs ``local_cpulist`` of
    the GPU's PCI function), so pinned host buffers allocated afterwards are first-touched on
    the GPU's own socket. Returns what was found, for the bench line."""
    import torch

    pr = torch.cuda.get_device_properties(dev)
    bdf = "%04x:%02x:%02x.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
    base = os.path.join("/sys/bus/pci/devices", bdf)
    info = {"pci": bdf}
    try:
        with open(os.path.join(base, "numa_node")) as f:
            info["numa_node"] = int(f.read().strip())
        with open(os.path.join(base, "local_cpulist")) as f:
            spec = f.read().strip()
        cpus = set()
        for part in spec.split(","):
            a, _, b = part.partition("-")
            cpus.update(range(int(a), int(b or a) + 1))
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
            info["cpus"] = len(cpus)
    except (OSError, ValueError) as e:
        info["error"] = str(e)[:80]
    return info


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
# shared timing helpers
# ---------------------------------------------------------------------------------------
def _barrier(world, dev):
    import torch
    import torch.distributed as dist

    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)


def _timed(step, steps, warmup, world, dev, profile=False):
    """`warmup` untimed steps, then `steps` steps bracketed by barrier + synchronize and timed
    with CUDA events on the current stream; the max over ranks, in ms per step. With
    ``profile`` the library's per-launch events cover the timed steps only: returns
    (ms, {kernel: (launches, ms)})."""
    import torch
    import torch.distributed as dist
    from treeattn_b200 import ops

    for _ in range(warmup):
        step()
    _barrier(world, dev)
    if profile:
        ops.profile_collect()  # drop anything recorded before
        ops.profile_enable(True)
    stream = torch.cuda.current_stream(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        step()
    t1.record(stream)
    _barrier(world, dev)
    ms = t0.elapsed_time(t1)
    prof = None
    if profile:
        prof = ops.profile_collect()
        ops.profile_enable(False)
    global _LAST_RANK_MS
    _LAST_RANK_MS = [ms / steps]
    if world > 1:
        allm = torch.zeros(world, device=dev, dtype=torch.float64)
        allm[dist.get_rank()] = ms
        dist.all_reduce(allm)  # every rank's time (the others contribute zeros)
        _LAST_RANK_MS = [float(x) / steps for x in allm.tolist()]
        ms = float(allm.max().item())
    return (ms / steps, prof) if profile else ms / steps


_LAST_RANK_MS = None  # per-rank ms per step of the last _timed call


def _fa2_ms(shape, dtype, causal, steps, warmup, world, dev, sd=1.0):
    """Dense FlashAttention-2 fwd+bwd (flash_attn library, a comparator) on this rank's bshd
    shape; max over ranks in ms per step, or None when flash_attn is not importable."""
    import torch
    try:
        from flash_attn import flash_attn_func
    except Exception:  # noqa: BLE001 - a comparator only
        return None
    g = torch.Generator(device=dev).manual_seed(7)
    q, k, v, go = (torch.randn(*shape, device=dev, generator=g).mul(sd).to(dtype) for _ in range(4))
    for t in (q, k, v):
        t.requires_grad_(True)

    def step():
        for t in (q, k, v):
            t.grad = None
        flash_attn_func(q, k, v, causal=causal).backward(go)

    return _timed(step, steps, warmup, world, dev)


def _kernels(prof, steps):
    total = sum(t for _, t in prof.values()) or 1.0
    return {k_: {"launches_per_step": c / steps, "ms_per_step": t / steps, "share": t / total}
            for k_, (c, t) in sorted(prof.items(), key=lambda x: -x[1][1])}


def record_c3(args, world, rank, dev):
    """B=8, S=8192, H=32, d=64, fp16 N(0, 0.5), fanout 4, leaf block 128,
    8 paths, causal; the fixed global problem is head-sharded over the ranks (strong scaling,
    no collective: rank r runs heads [r H/N, (r+1) H/N) with that slice of the global noise)."""
    import torch
    from treeattn_b200 import ops
    from treeattn_b200.blocked import blocked_tree_attention
    from treeattn_b200.sharding import shard_for_rank

    B, S, H, D, P, f, Lb = 8, 8192, 32, 64, 8, 4, 128
    if H % world:
        return {"skipped": f"H={H} not divisible by {world} ranks"}
    shard = shard_for_rank(B, H, rank, world, "head") if world > 1 else None
    hl = H // world
    gen = torch.Generator(device=dev).manual_seed(3000 + rank)
    q, k, v, go = (torch.randn(B, S, hl, D, device=dev, generator=gen).mul(0.5).to(torch.float16)
                   for _ in range(4))
    for t in (q, k, v):
        t.requires_grad_(True)

    def step():
        for t in (q, k, v):
            t.grad = None
        torch.manual_seed(0)
        blocked_tree_attention(q, k, v, True, None, num_samples=P, fanout=f, leaf_block=Lb,
                               shard=shard).backward(go)

    ms, prof = _timed(step, args.steps, args.warmup, world, dev, profile=True)
    rank_ms = _LAST_RANK_MS
    fa2 = None if args.no_fa2 else _fa2_ms((B, S, hl, D), torch.float16, True, args.steps,
                                            args.warmup, world, dev, 0.5)
    # tensor roofline of the dominant kernel: the five leaf-block products of the backward
    # (S, dP, dq, dV, dK), 2 * Lb * D flops each per (query, path) pair, as issued (masked keys
    # included), over its average launch time, against the measured dense 16-bit peak
    roof = None
    bk = "blocked_attn_bwd_tc" if "blocked_attn_bwd_tc" in prof else "blocked_attn_bwd_mma"
    if bk in prof:
        cnt, tms = prof[bk]
        flops = 5 * 2 * Lb * D * B * S * hl * P
        peak, kind = tensor_peak()
        ach = flops / (tms / cnt / 1e3) / 1e12
        roof = {"kernel": bk, "bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s",
                "frac": ach / peak, "peak_source": kind, "algorithmic_flops_per_launch": flops,
                "launch_ms": tms / cnt, "traffic": None}
    rec = {"config": {"workload": "generalised tree (fanout 4, leaf block 128), causal", "batch": B,
                      "seq_len": S, "heads": H, "head_dim": D, "num_samples": P, "fanout": f,
                      "leaf_block": Lb, "dtype": "f16", "data": "N(0, 0.5)",
                      "parallelism": f"head-sharded x{world} ({hl} heads per GPU), no collective"},
           "scaling": "strong", "value": B * S / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
           "gpu_launches": int(sum(c for c, _ in prof.values())), "kernels": _kernels(prof, args.steps),
           "roofline": roof, "ms_per_step_by_rank": rank_ms}
    if fa2 is not None:
        rec["fa2"] = {"value": B * S / (fa2 / 1e3), "unit": "tokens/s", "ms_per_step": fa2,
                      "what": "flash_attn_func dense causal fwd+bwd on each rank's head slice"}
    return rec


def record_c4(args, world, rank, dev):
    """B=1, S=65536, H=32, d=128, bf16, 16 paths, causal; the sequence is
    split evenly over the ranks (sequence parallel, strong scaling); one rank runs the plain
    causal op."""
    import torch
    from treeattn_b200 import ops
    import treeattn_b200 as ta
    from treeattn_b200.sequence_parallel import sp_tree_attention

    B, S, H, D, P = 1, 65536, 32, 128, 16
    n = S // world
    gen = torch.Generator(device=dev).manual_seed(4000)
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

    ms, prof = _timed(step, args.steps, args.warmup, world, dev, profile=True)
    rank_ms = _LAST_RANK_MS
    rec = {"config": {"workload": "stochastic tree attention, causal (exact prefix + corrected "
                                  "sampler)", "batch": B, "seq_len": S, "heads": H, "head_dim": D,
                      "num_samples": P, "dtype": "bf16",
                      "parallelism": f"sequence-parallel x{world}: NCCL all-gather of K/V, "
                                     "reduce-scatter of dK/dV" if world > 1 else "one GPU"},
           "scaling": "strong", "value": B * S / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
           "ms_per_step_by_rank": rank_ms,
           "gpu_launches": int(sum(c for c, _ in prof.values())), "kernels": _kernels(prof, args.steps)}
    if world == 1 and not args.no_fa2:
        fa2 = _fa2_ms((B, S, H, D), torch.bfloat16, True, 2, 1, world, dev)
        if fa2 is not None:
            rec["fa2"] = {"value": B * S / (fa2 / 1e3), "unit": "tokens/s", "ms_per_step": fa2,
                          "what": "flash_attn_func dense causal fwd+bwd, whole sequence on one GPU "
                                  "(1 warm-up, 2 timed steps)"}
    del q, k, v, go
    torch.cuda.empty_cache()
    return rec


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
        numa = bind_local_cpus(dev) if world > 1 else None
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
        # the host link alone: every rank uploads its four inputs at once, then downloads
        # them (pinned memory, one stream); the slowest rank's rate, GB/s per rank
        link = {}
        for name, pairs in (("h2d", [(b, h) for b, h in zip(bufs[0], (hq, hk, hv, hgo))]),
                            ("d2h", [(h, b) for b, h in zip(bufs[0], (hout, hdq, hdk, hdv))])):
            barrier()
            c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            c0.record(stream)
            for dst, src in pairs:
                dst.copy_(src, non_blocking=True)
            c1.record(stream)
            barrier()
            cms = c0.elapsed_time(c1)
            if world > 1:
                tm = torch.tensor([cms], device=dev, dtype=torch.float64)
                dist.all_reduce(tm, op=dist.ReduceOp.MAX)
                cms = float(tm.item())
            link[name + "_gbs_per_rank"] = 4 * nbytes / (cms / 1e3) / 1e9
        e2e["host_link"] = {**link, "ranks_at_once": world,
                            **({"numa": numa} if numa else {})}

    # FA2 beside every N (each rank its own batch element), then the configs 3 and 4 records
    fa2_ms = None if args.no_fa2 else _fa2_ms((B, S, H, D), dtype, False, args.steps, args.warmup,
                                              world, dev)
    extra = {}
    if not args.no_extra:
        extra["c3_head_sharded"] = record_c3(args, world, rank, dev)
        extra["c4_sequence_parallel"] = record_c4(args, world, rank, dev)

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
        "value_is": "whole-job tokens/s over all GPUs (value_per_gpu: per GPU)",
        "gpu_launches": int(sum(c for c, _ in prof.values())),
        "kernels": kernels,
        "roofline": roof,
        "clocks": clk,
        "e2e": e2e,
    }
    if fa2_ms is not None:
        line["fa2"] = {"value": world * B * S / (fa2_ms / 1e3), "unit": "tokens/s",
                       "ms_per_step": fa2_ms,
                       "what": "flash_attn_func dense attention fwd+bwd, same bshd bf16 shape per "
                               "GPU, non-causal (library comparator, not this package's path)"}
    line.update(extra)
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args)
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------------------
# CPU arm: the numpy oracle (a port of the reference; the reference itself is Python and
# does not travel), forked over heads on every host core. A step is the whole fwd+bwd of a
# subset of the heads (every query, the full tree): heads are independent trees, so the
# subset is an exact fraction of the workload, and throughput is quoted for the full config.
# ---------------------------------------------------------------------------------------
_SHARED = {}


def _cpu_heads(heads):
    """Full fwd+bwd of the oracle for the given heads: Haar build, sampler, softmax, value
    sum, analytic backward, transposed Haar build. Returns seconds."""
    from oracle import tree_oracle as O

    d = _SHARED
    t0 = time.perf_counter()
    for h in heads:
        sl = slice(h, h + 1)
        q, k, v, go = (d[n][:, :, sl] for n in ("q", "k", "v", "go"))
        g = d["g"][:, :, :, sl]
        k_int = O.haar_internal_node_keys(k, "bf16")
        fw = O.forward(q, k_int, v, g, d["P"])
        _, dk_int, _ = O.backward(q, k_int, v, go, fw["leaf"], fw["weights"])
        O.haar_internal_node_keys_backward(dk_int)
    return time.perf_counter() - t0


class CpuReference:
    """The oracle port on the host cores, one process per core, heads split over them."""

    def __init__(self, S, H, D, P):
        import multiprocessing as mp

        sys.path.insert(0, ROOT)
        from oracle import tree_oracle as O

        rng = np.random.default_rng(0)
        rb = lambda *s: O.round_to_bf16(rng.standard_normal(s, dtype=np.float32))  # noqa: E731
        _SHARED.update(q=rb(S, 1, H, D), k=rb(S, 1, H, D), v=rb(S, 1, H, D), go=rb(S, 1, H, D),
                       g=-np.log(rng.exponential(size=(O.log_n_of(S), S, 1, H, P, 2)).astype(np.float32)),
                       P=P)
        self.S, self.H = S, H
        self.cores = min(os.cpu_count() or 1, H)
        self.pool = mp.get_context("fork").Pool(self.cores)

    def step(self, n_heads):
        """One step over the first n_heads heads; returns wall seconds."""
        parts = [list(range(i, n_heads, self.cores)) for i in range(self.cores)]
        t0 = time.perf_counter()
        self.pool.map(_cpu_heads, [p for p in parts if p])
        return time.perf_counter() - t0

    def close(self):
        self.pool.close()
        self.pool.join()


def cpu_baseline(args):
    """One bounded step (one head per host core) for our arm's line."""
    S, H, D, P = args.seq_len, args.heads, args.head_dim, args.num_samples
    ref = CpuReference(S, H, D, P)
    try:
        n = ref.cores
        t = ref.step(n)
    finally:
        ref.close()
    return {"value": S * (n / H) / t, "unit": "tokens/s", "cores": ref.cores, "kind": "port",
            "sample": f"numpy oracle (oracle/tree_oracle.py): full fwd+bwd (Haar build, sampler, "
                      f"value sum, backward, Haar transpose) of {n} of {H} heads, all {S} queries, "
                      f"one process per core; value = tokens/s of the full {H}-head config",
            "step_s": t, "heads_per_step": n}


def run_reference(args):
    """The reference arm: the oracle port timed over whole steps on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    S, H, D, P = args.seq_len, args.heads, args.head_dim, args.num_samples
    ref = CpuReference(S, H, D, P)
    try:
        # calibration step (counts as the first warm-up): one head per core
        n = ref.cores
        t1 = ref.step(n)
        # size a step so that warm-up + timed steps take about 150 s in all
        per_step = 150.0 / max(1, args.steps + args.warmup)
        n = min(H, n * max(1, int(per_step // max(t1, 1e-3))))
        for _ in range(max(0, args.warmup - 1)):
            ref.step(n)
        times = [ref.step(n) for _ in range(args.steps)]
    finally:
        ref.close()
    t = statistics.mean(times)
    value = S * (n / H) / t
    sample = (f"numpy oracle (oracle/tree_oracle.py): full fwd+bwd (Haar build, sampler, value sum, "
              f"backward, Haar transpose) of {n} of {H} heads per step, all {S} queries, one process "
              f"per host core; value = tokens/s of the full {H}-head config")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic N(0,1), bf16-rounded", "config": {**WORKLOAD, "batch_per_gpu": 1},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": ref.cores, "kind": "port",
                             "sample": sample, "heads_per_step": n, "step_s": times},
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


def run_sweep(args):
    """BASELINE config 5, attn-bench style: S in {1k..16k} with B*S = 16384 tokens, H=16,
    d in {32, 64, 96, 128}, bf16 / fp16, causal off / on, 8 paths; this package's op and dense
    FA2 on the same inputs. Per configuration 10 warm-up and 50 timed iterations of the forward
    alone and of forward + backward, each iteration timed with CUDA events; bwd = median(step) -
    median(fwd) (attn_bench/harness.py). One JSON line with every row."""
    import torch
    import treeattn_b200 as ta

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    try:
        from flash_attn import flash_attn_func
    except Exception:  # noqa: BLE001 - a comparator only
        flash_attn_func = None
    warm, iters = 10, 50

    def med_ms(fn):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
        for a, b in ev:
            a.record()
            fn()
            b.record()
        torch.cuda.synchronize()
        return statistics.median(a.elapsed_time(b) for a, b in ev)

    rows = []
    for dname, dt in (("bf16", torch.bfloat16), ("fp16", torch.float16)):
        for causal in (False, True):
            for D in (32, 64, 96, 128):
                for S in (1024, 2048, 4096, 8192, 16384):
                    B, H, P = 16384 // S, 16, 8
                    g = torch.Generator(device=dev).manual_seed(S + D)
                    q, k, v, go = (torch.randn(B, S, H, D, device=dev, generator=g).to(dt) for _ in range(4))
                    for t in (q, k, v):
                        t.requires_grad_(True)

                    def fwd_ours():
                        with torch.no_grad():
                            ta.tree_attention(q, k, v, causal, None, num_samples=P)

                    def step_ours():
                        for t in (q, k, v):
                            t.grad = None
                        ta.tree_attention(q, k, v, causal, None, num_samples=P).backward(go)

                    torch.manual_seed(0)
                    f_ms, s_ms = med_ms(fwd_ours), med_ms(step_ours)
                    row = {"dtype": dname, "causal": causal, "seq_len": S, "batch": B, "heads": H,
                           "head_dim": D, "ours_fwd_ms": f_ms, "ours_bwd_ms": s_ms - f_ms,
                           "ours_step_ms": s_ms, "ours_tokens_per_s": B * S / (s_ms / 1e3)}
                    if flash_attn_func is not None:
                        def fwd_fa():
                            with torch.no_grad():
                                flash_attn_func(q, k, v, causal=causal)

                        def step_fa():
                            for t in (q, k, v):
                                t.grad = None
                            flash_attn_func(q, k, v, causal=causal).backward(go)

                        ff, fs = med_ms(fwd_fa), med_ms(step_fa)
                        row.update(fa2_fwd_ms=ff, fa2_bwd_ms=fs - ff, fa2_step_ms=fs,
                                   fa2_tokens_per_s=B * S / (fs / 1e3), speedup=fs / s_ms)
                    rows.append(row)
                    print(json.dumps(row), file=sys.stderr, flush=True)
                    del q, k, v, go
    print(json.dumps({"metric": "attn-bench sweep (BASELINE config 5): fwd / bwd ms, ours vs FA2",
                      "warmup": warm, "iters": iters, "num_samples": 8, "rows": rows}), flush=True)


def main():
    args = parse_args()
    sys.path.insert(0, ROOT)
    if args.impl == "reference":
        run_reference(args)
    elif args.mode == "sp":
        run_sp(args)
    elif args.mode == "blocked":
        run_blocked(args)
    elif args.mode == "sweep":
        run_sweep(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
