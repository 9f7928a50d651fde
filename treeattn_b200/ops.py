"""Torch-tensor wrappers over the C ABI (device memory, streams, RNG reservation).

Every function here launches the in-tree CUDA library on the current CUDA stream of the
tensors' device. There is no CPU or eager fallback: CPU tensors and a missing library raise.

Tensors are described to the C ABI as strided (seq, batch, head, dim) views; ``lbhd`` below
means a 4-D tensor whose logical axes are in that order (it may be a permuted view, e.g. of
a bshd tensor) with a contiguous ``dim`` axis.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib as L

_DTYPES = {torch.float32: L.TA_F32, torch.float16: L.TA_F16, torch.bfloat16: L.TA_BF16}
MAX_LOGIT = 1e3

_STATS_TEMPLATE = {
    "tree_build_calls": 0,
    "tree_build_backward_calls": 0,
    "forward_calls": 0,
    "backward_calls": 0,
    "sample_calls": 0,
    "replay_calls": 0,
    "value_sum_calls": 0,
    "causal_forward_calls": 0,
    "causal_backward_calls": 0,
    "exact_forward_calls": 0,
    "exact_backward_calls": 0,
}
_STATS = dict(_STATS_TEMPLATE)


def reset_runtime_stats() -> None:
    """Zero the per-op native call counters (mirrors treeattn_cuda._autograd:38-49)."""
    _STATS.clear()
    _STATS.update(_STATS_TEMPLATE)


def get_runtime_stats() -> dict[str, int]:
    return dict(_STATS)


def _note(op: str) -> None:
    _STATS[op + "_calls"] += 1


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}; expected float32, float16 or bfloat16")


def layout(t: torch.Tensor) -> L.Layout:
    """Strides of a logical (seq, batch, head, dim) 4-D view."""
    if t.dim() != 4:
        raise ValueError(f"expected a 4-D (seq, batch, head, dim) view, got {tuple(t.shape)}")
    if t.stride(3) != 1 and t.shape[3] > 1:
        raise ValueError("the head_dim axis must be contiguous")
    s = t.stride()
    return L.Layout(s[0], s[1], s[2])


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise ValueError("treeattn_b200 ops run on CUDA tensors only (no CPU path)")


def is_power_of_two(n: int) -> bool:
    return n > 0 and (n & (n - 1)) == 0


def log_n_of(num_leaves: int) -> int:
    return max(num_leaves.bit_length() - 1, 0)


# ---------------------------------------------------------------------------------------
# Gumbel stream reservation (torch's default CUDA generator)
# ---------------------------------------------------------------------------------------

def philox_plan(numel: int, sm_count: int, max_threads_per_sm: int) -> tuple[int, int]:
    """(offset increment, grid stride) of one torch exponential_() draw of ``numel``."""
    step = ctypes.c_uint64()
    stride = ctypes.c_int64()
    L.call("ta_philox_plan", numel, sm_count, max_threads_per_sm, ctypes.byref(step),
           ctypes.byref(stride))
    return step.value, stride.value


_GEOM: dict[int, tuple[int, int]] = {}


def device_rng_geometry(device: torch.device) -> tuple[int, int]:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _GEOM:
        a, b = ctypes.c_int32(), ctypes.c_int32()
        L.call("ta_device_rng_geometry", idx, ctypes.byref(a), ctypes.byref(b))
        _GEOM[idx] = (a.value, b.value)
    return _GEOM[idx]


def reserve_gumbel_stream(device: torch.device, numel: int, depths: int) -> L.Rng:
    """Reserve ``depths`` exponential_() draws of ``numel`` from torch's CUDA generator.

    Consumes exactly the generator offsets the reference's per-depth
    ``torch.empty(...).exponential_()`` calls would (_autograd.py:188-195), so a call made
    after ``torch.manual_seed(s)`` sees the same noise as the reference after the same seed.
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    gen = torch.cuda.default_generators[idx]
    sms, mtps = device_rng_geometry(device)
    step, stride = philox_plan(numel, sms, mtps)
    seed = gen.initial_seed()
    offset = gen.get_offset()
    gen.set_offset(offset + depths * step)
    return L.Rng(seed, offset, step, stride)


def gumbel_fill(out: torch.Tensor, rng: L.Rng, depth0: int = 0) -> torch.Tensor:
    """Fill float32 ``out`` (depths, numel) -- or (numel,) for one depth -- with the Gumbel
    noise of depths depth0.. of the stream ``rng`` (bit-identical to torch's draws)."""
    _require_cuda(out)
    if out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError("out must be a contiguous float32 tensor")
    depths = out.shape[0] if out.dim() > 1 else 1
    numel = out.numel() // depths
    L.call("ta_gumbel_fill", _ptr(out), numel, ctypes.byref(rng), depth0, depths,
           _stream(out.device))
    return out


def gumbel_fill_shard(out: torch.Tensor, rng: L.Rng, rows: int, shard, row_elems: int,
                      depth0: int = 0, *, row_total: int | None = None, row0: int = 0) -> torch.Tensor:
    """Fill float32 ``out`` (depths, rows * batch_count * head_count * row_elems) with this
    shard's slice of the full (row_total, batch_total, head_total, row_elems) draw of ``rng``
    (``rng`` is the plan of the FULL numel); the shard's rows are row0 .. row0 + rows - 1
    (all rows by default)."""
    _require_cuda(out)
    if out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError("out must be a contiguous float32 tensor")
    depths = out.shape[0] if out.dim() > 1 else 1
    if out.numel() != depths * rows * shard.batch_count * shard.head_count * row_elems:
        raise ValueError("out does not hold this shard's draw")
    row_total = rows if row_total is None else row_total
    sh = L.Shard(row_total, row0, rows, shard.batch_total, shard.batch0, shard.batch_count,
                 shard.head_total, shard.head0, shard.head_count)
    L.call("ta_gumbel_fill_shard", _ptr(out), ctypes.byref(rng), ctypes.byref(sh), row_elems,
           depth0, depths, _stream(out.device))
    return out


def branch_prob_stride(num_leaves: int) -> int:
    return (log_n_of(num_leaves) + 3) & ~3


# ---------------------------------------------------------------------------------------
# tree build
# ---------------------------------------------------------------------------------------

LAYOUTS = {"reference": L.TA_LAYOUT_REFERENCE, "tree": L.TA_LAYOUT_TREE}


def _layout_code(node_layout: str) -> int:
    try:
        return LAYOUTS[node_layout]
    except KeyError:
        raise ValueError(f"node layout must be 'reference' or 'tree', got {node_layout!r}") from None


def tree_build(k_lbhd: torch.Tensor, out: torch.Tensor | None = None,
               node_layout: str = "reference") -> torch.Tensor:
    """Internal-node keys (S-1, B, H, D) from leaf keys (S, B, H, D) (Haar, input dtype).

    The result is allocated head-major, memory (B, H, S-1, D), and returned as a logical
    (S-1, B, H, D) view: each head's tree is one contiguous block. ``node_layout`` "reference"
    reproduces attn-bench's array (position order, read as a heap by the samplers); "tree"
    puts every coefficient on the heap node of the subtree it summarises.
    """
    _require_cuda(k_lbhd)
    S, B, H, D = k_lbhd.shape
    if not is_power_of_two(S) or S < 2:
        raise ValueError(f"treeattn requires power-of-two seqlen >= 2, got {S}")
    if out is None:
        out = torch.empty((B, H, S - 1, D), device=k_lbhd.device, dtype=k_lbhd.dtype).permute(2, 0, 1, 3)
    dt = dtype_code(k_lbhd.dtype)
    lib = L.load()
    ws_bytes = lib.ta_tree_build_workspace_size(B, S, H, D, dt)
    ws = torch.empty(max(ws_bytes, 1), device=k_lbhd.device, dtype=torch.uint8)
    L.call("ta_tree_build_ex", dt, B, S, H, D, _ptr(k_lbhd), layout(k_lbhd), _ptr(out), layout(out),
           _layout_code(node_layout), _ptr(ws), ws_bytes, _stream(k_lbhd.device))
    _note("tree_build")
    return out


def tree_build_backward(dk_int: torch.Tensor, dk_leaf: torch.Tensor,
                        node_layout: str = "reference") -> torch.Tensor:
    """dk_leaf (S, B, H, D view, any float dtype) <- transpose of the Haar build of float32 dk_int."""
    _require_cuda(dk_int, dk_leaf)
    if dk_int.dtype != torch.float32:
        raise ValueError("dk_int must be float32")
    S, B, H, D = dk_leaf.shape
    lib = L.load()
    ws_bytes = lib.ta_tree_build_backward_workspace_size(B, S, H, D)
    ws = torch.empty(max(ws_bytes, 1), device=dk_int.device, dtype=torch.uint8)
    L.call("ta_tree_build_backward_ex", dtype_code(dk_leaf.dtype), B, S, H, D, _ptr(dk_int),
           layout(dk_int), _ptr(dk_leaf), layout(dk_leaf), _layout_code(node_layout), _ptr(ws),
           ws_bytes, _stream(dk_int.device))
    _note("tree_build_backward")
    return dk_leaf


# ---------------------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------------------

def _shape(q: torch.Tensor, num_leaves: int, num_samples: int, max_logit: float) -> L.Shape:
    Lq, B, H, D = q.shape
    return L.Shape(B, Lq, num_leaves, H, D, num_samples, dtype_code(q.dtype), float(max_logit))


@dataclass
class ForwardResult:
    out: torch.Tensor       # (L, B, H, D) view, input dtype
    leaf: torch.Tensor      # (L, B, H, S) int32
    weights: torch.Tensor   # (L, B, H, S) float32
    packed: torch.Tensor | None
    branch_prob: torch.Tensor | None  # (B*H, L*S, stride) float32, for the backward


def draw_gumbels(Lq: int, B: int, H: int, N: int, num_samples: int, device, *, shard=None,
                 query_rows: tuple[int, int] | None = None, rng: L.Rng | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """The Gumbel noise ``forward`` would draw for q of shape (Lq, B, H, D) over N keys, as a
    float32 (log2 N, Lq * B * H * num_samples * 2) tensor on the current stream: reserved from
    torch's CUDA generator exactly as the reference's per-depth draws are (the matching slice of
    the full problem's draw for a ``shard`` or ``query_rows`` block). Passing it to ``forward``
    as ``gumbels`` gives the same result as letting ``forward`` draw it. ``out`` is an optional
    float32 (log2 N, numel) buffer to fill."""
    numel = Lq * B * H * num_samples * 2
    ln = log_n_of(N)
    if out is None:
        out = torch.empty((ln, numel), device=device, dtype=torch.float32)
    sharded = (shard is not None and not shard.is_full) or query_rows is not None
    if not sharded:
        if rng is None:
            rng = reserve_gumbel_stream(device, numel, ln)
        return gumbel_fill(out, rng)
    from .sharding import ShardSpec
    spec = shard if shard is not None else ShardSpec(B, 0, B, H, 0, H)
    if (spec.batch_count, spec.head_count) != (B, H):
        raise ValueError(f"shard {spec} does not match q's (batch, heads) = ({B}, {H})")
    row0, row_total = query_rows if query_rows is not None else (0, Lq)
    if row0 < 0 or row0 + Lq > row_total:
        raise ValueError(f"query rows {row0}..{row0 + Lq} outside {row_total}")
    if rng is None:
        rng = reserve_gumbel_stream(
            device, row_total * spec.batch_total * spec.head_total * num_samples * 2, ln)
    return gumbel_fill_shard(out, rng, Lq, spec, num_samples * 2, row_total=row_total, row0=row0)


def forward(q: torch.Tensor, k_int: torch.Tensor, v: torch.Tensor, num_samples: int, *,
            max_logit: float = MAX_LOGIT, out: torch.Tensor | None = None,
            gumbels: torch.Tensor | None = None, want_packed: bool = False,
            rng: L.Rng | None = None, for_backward: bool = True,
            fused_rng: bool = False, shard=None,
            query_rows: tuple[int, int] | None = None) -> ForwardResult:
    """Fused sampler + softmax + value gather. q (L,B,H,D), k_int (N-1,B,H,D), v (N,B,H,D).

    The Gumbel noise comes from torch's default CUDA generator (reserved here, exactly as
    the reference's per-depth draws consume it) unless ``gumbels`` (float32
    (log2 N, L, B, H, S, 2)) or an explicit ``rng`` is given. By default all depths' noise is
    drawn first by ``ta_gumbel_fill`` (each philox 4-vector used four times);
    ``fused_rng=True`` draws it inside the sampler instead. ``for_backward`` also returns the
    per-path branch probabilities ``ta_backward`` needs. ``shard`` (a
    ``sharding.ShardSpec``) marks q/k/v as one (batch, head) block of a larger problem: the
    noise is then the matching slice of the full problem's draw (see ``gumbel_fill_shard``).
    ``query_rows`` = (row0, row_total) does the same along the query axis: q holds queries
    row0 .. row0 + L - 1 of a row_total-query problem (sequence parallelism).
    """
    _require_cuda(q, k_int, v)
    Lq, B, H, D = q.shape
    N = v.shape[0]
    if not (q.dtype == k_int.dtype == v.dtype):
        raise ValueError("q, k and v must share a dtype")
    shape = _shape(q, N, num_samples, max_logit)
    dev = q.device
    if out is None:
        out = torch.empty((Lq, B, H, D), device=dev, dtype=q.dtype)
    leaf = torch.empty((Lq, B, H, num_samples), device=dev, dtype=torch.int32)
    weights = torch.empty((Lq, B, H, num_samples), device=dev, dtype=torch.float32)
    packed = None
    if want_packed:
        packed = torch.empty((Lq, B, H, num_samples, (log_n_of(N) + 7) // 8), device=dev,
                             dtype=torch.uint8)
    numel = Lq * B * H * num_samples * 2
    rng_p = None
    sharded = (shard is not None and not shard.is_full) or query_rows is not None
    if sharded and gumbels is None:
        if fused_rng:
            raise ValueError("fused_rng does not support shards")
        gumbels = draw_gumbels(Lq, B, H, N, num_samples, dev, shard=shard, query_rows=query_rows,
                               rng=rng)
    if gumbels is not None:
        gumbels = gumbels.to(device=dev, dtype=torch.float32).contiguous()
    else:
        if rng is None:
            rng = reserve_gumbel_stream(dev, numel, log_n_of(N))
        if fused_rng:
            rng_p = ctypes.byref(rng)
        else:
            gumbels = gumbel_fill(torch.empty((log_n_of(N), numel), device=dev, dtype=torch.float32), rng)
    bp = None
    if for_backward:
        bp = torch.empty((B * H, Lq * num_samples, branch_prob_stride(N)), device=dev,
                         dtype=torch.float32)
    L.call("ta_forward", ctypes.byref(shape), _ptr(q), layout(q), _ptr(k_int), layout(k_int),
           _ptr(v), layout(v), _ptr(out), layout(out), rng_p, _ptr(gumbels), _ptr(leaf),
           _ptr(weights), _ptr(packed), _ptr(bp), _stream(dev))
    _note("forward")
    return ForwardResult(out, leaf, weights, packed, bp)


def backward(q, k_int, v, grad_out, leaf, weights, branch_prob, num_samples, *,
             max_logit=MAX_LOGIT, dq=None, dk=None, dv=None, dk_dtype: torch.dtype | None = None):
    """Deterministic gradients (dq, dk, dv) of ``forward``. All (seq, B, H, D) views; dk and
    dv may be float32 buffers whatever the input dtype."""
    _require_cuda(q, k_int, v, grad_out, leaf, weights, branch_prob)
    Lq, B, H, D = q.shape
    N = v.shape[0]
    dev = q.device
    shape = _shape(q, N, num_samples, max_logit)
    dk_dtype = dk_dtype or q.dtype
    if dq is None:
        dq = torch.empty((Lq, B, H, D), device=dev, dtype=q.dtype)
    if dk is None:
        dk = torch.empty((N - 1, B, H, D), device=dev, dtype=dk_dtype)
    if dv is None:
        dv = torch.empty((N, B, H, D), device=dev, dtype=v.dtype)
    lib = L.load()
    ws_bytes = lib.ta_backward_workspace_size(ctypes.byref(shape))
    if ws_bytes == 0:
        raise ValueError("invalid backward shape")
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    grad_out = grad_out if grad_out.stride(-1) == 1 else grad_out.contiguous()
    L.call("ta_backward", ctypes.byref(shape), _ptr(q), layout(q), _ptr(k_int), layout(k_int),
           _ptr(v), layout(v), _ptr(grad_out), layout(grad_out), _ptr(leaf.contiguous()),
           _ptr(weights.contiguous()), _ptr(branch_prob), _ptr(dq), layout(dq), _ptr(dk), layout(dk),
           dtype_code(dk.dtype), _ptr(dv), layout(dv), dtype_code(dv.dtype), _ptr(ws), ws_bytes,
           _stream(dev))
    _note("backward")
    return dq, dk, dv


def sample_paths(q, k_int, num_samples, *, max_logit=MAX_LOGIT, gumbels=None, rng=None):
    """Sampler only: (leaf int32, log_prob float32, packed uint8), all (L,B,H,S[,P])."""
    _require_cuda(q, k_int)
    Lq, B, H, D = q.shape
    N = k_int.shape[0] + 1
    dev = q.device
    shape = _shape(q, N, num_samples, max_logit)
    leaf = torch.empty((Lq, B, H, num_samples), device=dev, dtype=torch.int32)
    lp = torch.empty((Lq, B, H, num_samples), device=dev, dtype=torch.float32)
    packed = torch.empty((Lq, B, H, num_samples, (log_n_of(N) + 7) // 8), device=dev,
                         dtype=torch.uint8)
    if gumbels is not None:
        gumbels = gumbels.to(device=dev, dtype=torch.float32).contiguous()
        rng_p = None
    else:
        if rng is None:
            rng = reserve_gumbel_stream(dev, Lq * B * H * num_samples * 2, log_n_of(N))
        rng_p = ctypes.byref(rng)
    L.call("ta_sample_paths", ctypes.byref(shape), _ptr(q), layout(q), _ptr(k_int), layout(k_int),
           rng_p, _ptr(gumbels), _ptr(leaf), _ptr(lp), _ptr(packed), _stream(dev))
    _note("sample")
    return leaf, lp, packed


def replay_paths(q, k_int, packed, *, softmax=False, max_logit=MAX_LOGIT):
    """Replay packed bits: (leaf int32, log_prob or softmax weights float32)."""
    _require_cuda(q, k_int, packed)
    Lq, B, H, D = q.shape
    S = packed.shape[3]
    N = k_int.shape[0] + 1
    dev = q.device
    shape = _shape(q, N, S, max_logit)
    leaf = torch.empty((Lq, B, H, S), device=dev, dtype=torch.int32)
    val = torch.empty((Lq, B, H, S), device=dev, dtype=torch.float32)
    L.call("ta_replay_paths", ctypes.byref(shape), _ptr(q), layout(q), _ptr(k_int), layout(k_int),
           _ptr(packed.contiguous()), 1 if softmax else 0, _ptr(leaf), _ptr(val), _stream(dev))
    _note("replay")
    return leaf, val


def weighted_value_sum(v, leaf, weights, *, out=None):
    """out[l,b,h] = sum_s w v[clamp(leaf)]; v (N,B,H,D), leaf/weights (L,B,H,S)."""
    _require_cuda(v, leaf, weights)
    Lq, B, H, S = leaf.shape
    N, _, _, D = v.shape
    dev = v.device
    shape = L.Shape(B, Lq, N, H, D, S, dtype_code(v.dtype), MAX_LOGIT)
    if out is None:
        out = torch.empty((Lq, B, H, D), device=dev, dtype=v.dtype)
    L.call("ta_weighted_value_sum", ctypes.byref(shape), _ptr(v), layout(v),
           _ptr(leaf.to(torch.int32).contiguous()), _ptr(weights.float().contiguous()), _ptr(out),
           layout(out), _stream(dev))
    _note("value_sum")
    return out


# ---------------------------------------------------------------------------------------
# per-launch profiling (CUDA events recorded by the library on each launch's stream)
# ---------------------------------------------------------------------------------------

def profile_enable(on: bool = True) -> None:
    L.call("ta_profile_enable", 1 if on else 0)


def profile_collect() -> dict[str, tuple[int, float]]:
    """{kernel: (launches, total_ms)} of every launch since the last collect (synchronises)."""
    lib = L.load()
    buf = ctypes.create_string_buffer(1 << 16)
    n = lib.ta_profile_collect(buf, len(buf))
    if n >= len(buf):
        raise RuntimeError("profile text truncated")
    out = {}
    for line in buf.value.decode().splitlines():
        name, cnt, ms = line.split()
        out[name] = (int(cnt), float(ms))
    return out


# ---------------------------------------------------------------------------------------
# causal sampler (A9) and exact mode (A10)
# ---------------------------------------------------------------------------------------

def reserve_causal_stream(device: torch.device, numel_per_draw: int, draws: int) -> L.Rng:
    """Reserve ``draws`` exponential_() calls of ``numel_per_draw`` (one per query and level)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    gen = torch.cuda.default_generators[idx]
    sms, mtps = device_rng_geometry(device)
    step, stride = philox_plan(numel_per_draw, sms, mtps)
    seed = gen.initial_seed()
    offset = gen.get_offset()
    gen.set_offset(offset + draws * step)
    return L.Rng(seed, offset, step, stride)


@dataclass
class CausalState:
    leaf: torch.Tensor
    weights: torch.Tensor
    branch_prob: torch.Tensor
    corrected: torch.Tensor
    masses: torch.Tensor
    query_offset: int


def causal_forward(q, k_int, v, num_samples, query_offset=0, *, out=None, gumbels=None,
                   rng: L.Rng | None = None):
    """Causal sampler with the boundary correction for queries q (L,B,H,D) whose causal
    boundaries are t + query_offset. Returns (out, CausalState). The noise of query t, level d
    is the draw at ``rng.offset + (t * log2 N + d) * rng.offset_step`` (reserved from the
    generator when ``rng`` is None)."""
    _require_cuda(q, k_int, v)
    Lq, B, H, D = q.shape
    N = v.shape[0]
    dev = q.device
    S = num_samples
    ln = log_n_of(N)
    shape = L.Shape(B, Lq, N, H, D, S, dtype_code(q.dtype), MAX_LOGIT)
    if out is None:
        out = torch.empty((Lq, B, H, D), device=dev, dtype=q.dtype)
    leaf = torch.empty((Lq, B, H, S), device=dev, dtype=torch.int32)
    weights = torch.empty((Lq, B, H, S), device=dev, dtype=torch.float32)
    bp = torch.empty((B * H, Lq * S, branch_prob_stride(N)), device=dev, dtype=torch.float32)
    corrected = torch.empty((max(Lq, 1),), device=dev, dtype=torch.int32)
    masses = torch.empty((max(Lq, 1), B, H, 2 * ln + 1), device=dev, dtype=torch.float32)
    rng_p = None
    if gumbels is not None:
        gumbels = gumbels.to(device=dev, dtype=torch.float32).contiguous()
    else:
        if rng is None:
            rng = reserve_causal_stream(dev, B * H * S * 2, Lq * ln)
        rng_p = ctypes.byref(rng)
    L.call("ta_causal_forward", ctypes.byref(shape), int(query_offset), _ptr(q), layout(q),
           _ptr(k_int), layout(k_int), _ptr(v), layout(v), _ptr(out), layout(out), rng_p,
           _ptr(gumbels), _ptr(leaf), _ptr(weights), _ptr(bp), _ptr(corrected), _ptr(masses),
           _stream(dev))
    _note("causal_forward")
    return out, CausalState(leaf, weights, bp, corrected, masses, int(query_offset))


def causal_backward(q, k_int, v, grad_out, state: CausalState, num_samples, *, dq, dk, dv):
    """Gradients of causal_forward: writes dq (input dtype) and float32 dk / dv (all rows)."""
    Lq, B, H, D = q.shape
    N = v.shape[0]
    dev = q.device
    S = num_samples
    SP = S + 1
    stride = branch_prob_stride(N)
    shape = L.Shape(B, Lq, N, H, D, S, dtype_code(q.dtype), MAX_LOGIT)
    coef = torch.empty((B * H, Lq * SP, stride), device=dev, dtype=torch.float32)
    vw = torch.empty((B * H, Lq * SP), device=dev, dtype=torch.float32)
    keys = torch.empty((B * H, Lq * SP), device=dev, dtype=torch.int32)
    vals = torch.empty((B * H, Lq * SP), device=dev, dtype=torch.int32)
    grad_out = grad_out if grad_out.stride(-1) == 1 else grad_out.contiguous()
    L.call("ta_causal_coefficients", ctypes.byref(shape), state.query_offset, _ptr(q), layout(q),
           _ptr(k_int), layout(k_int), _ptr(v), layout(v), _ptr(grad_out), layout(grad_out),
           _ptr(state.leaf), _ptr(state.weights), _ptr(state.branch_prob), _ptr(state.corrected),
           _ptr(state.masses), _ptr(coef), _ptr(vw), _ptr(keys), _ptr(vals), _stream(dev))
    shape2 = L.Shape(B, Lq, N, H, D, SP, dtype_code(q.dtype), MAX_LOGIT)
    lib = L.load()
    ws_bytes = lib.ta_backward_workspace_size(ctypes.byref(shape2))
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    L.call("ta_backward_coef", ctypes.byref(shape2), _ptr(q), layout(q), _ptr(k_int), layout(k_int),
           _ptr(grad_out), layout(grad_out), _ptr(coef), _ptr(vw), _ptr(keys), _ptr(vals),
           _ptr(dq), layout(dq), _ptr(dk), layout(dk), L.TA_F32, _ptr(dv), layout(dv), L.TA_F32,
           _ptr(ws), ws_bytes, _stream(dev))
    _note("causal_backward")


def exact_forward(q, k_int, v, causal, query_offset=0, *, out=None, want_weights=True):
    """Exact attention over all leaves (mode='deterministic'). Returns (out, weights|None)."""
    _require_cuda(q, k_int, v)
    Lq, B, H, D = q.shape
    N = v.shape[0]
    dev = q.device
    shape = L.Shape(B, Lq, N, H, D, 1, dtype_code(q.dtype), MAX_LOGIT)
    if out is None:
        out = torch.empty((Lq, B, H, D), device=dev, dtype=q.dtype)
    w = torch.empty((Lq, B, H, N), device=dev, dtype=torch.float32) if want_weights else None
    lib = L.load()
    ws_bytes = lib.ta_exact_workspace_size(ctypes.byref(shape))
    if ws_bytes == 0:
        raise ValueError("invalid shape for exact attention")
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    L.call("ta_exact_forward", ctypes.byref(shape), 1 if causal else 0, int(query_offset), _ptr(q),
           layout(q), _ptr(k_int), layout(k_int), _ptr(v), layout(v), _ptr(out), layout(out),
           _ptr(w), _ptr(ws), ws_bytes, _stream(dev))
    _note("exact_forward")
    return out, w


def exact_backward(q, k_int, v, grad_out, causal, query_offset=0, *, dq, dk, dv, accumulate):
    """Gradients of exact_forward: dq written (input dtype); float32 dk / dv written or added."""
    Lq, B, H, D = q.shape
    N = v.shape[0]
    dev = q.device
    shape = L.Shape(B, Lq, N, H, D, 1, dtype_code(q.dtype), MAX_LOGIT)
    lib = L.load()
    ws_bytes = lib.ta_exact_workspace_size(ctypes.byref(shape))
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    grad_out = grad_out if grad_out.stride(-1) == 1 else grad_out.contiguous()
    L.call("ta_exact_backward", ctypes.byref(shape), 1 if causal else 0, int(query_offset), _ptr(q),
           layout(q), _ptr(k_int), layout(k_int), _ptr(v), layout(v), _ptr(grad_out), layout(grad_out),
           _ptr(dq), layout(dq), _ptr(dk), layout(dk), _ptr(dv), layout(dv), 1 if accumulate else 0,
           _ptr(ws), ws_bytes, _stream(dev))
    _note("exact_backward")
