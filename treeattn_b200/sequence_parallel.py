"""Sequence parallelism for long context: the sequence split evenly over R ranks.

Rank r holds the bshd chunk of positions [r*n, (r+1)*n), n = N/R, of q, k, v (keys,
values and the queries at those positions) and returns the same chunk of the output and of
dq, dk, dv. The result equals one unsharded ``tree_attention`` call made after the same
``torch.manual_seed`` (the output bit for bit; dk/dv up to the order of the cross-rank sums).

Exchange, for the reference's tree layout. attn-bench's Haar build writes its coefficients
in position order and the kernels read that array as a heap (_treeattn_common.py:54-86,
_tree_mha.py:119): heap depth d is the positions
[2^d, 2^(d+1)), so the deepest level alone is the upper half of the sequence and every
sampled path reads rows of every rank. So the forward all-gathers the leaf keys and values
(NCCL over NVLink into local HBM, no peer reads inside kernels), builds the whole tree
locally (bit-identical on every rank: same inputs, same kernel) and samples only its own
queries, with causal boundaries and noise offsets at their global positions. The backward
produces full-size float32 partial dK (through the Haar transpose) and dV from the rank's
own queries and reduce-scatters them back to the owning ranks.

Noise: non-causal, each rank fills its query rows of the global per-depth draws
(ta_gumbel_fill_shard); causal, query t's draws sit at a fixed offset of the generator
(t * log2 N + d steps), so a rank starts at its first sampled query's offset. Every rank
advances its generator by the full problem's draw, like the unsharded call.

Causal hybrid: the first S = num_samples queries take the exact path, which reads the whole
tree of every head (O(N·D) per query and head). They all sit on rank 0, so when H divides by
R every rank runs the exact prefix for its own H/R heads instead: rank 0's prefix rows of q
(and, in the backward, of grad_out) are all-gathered (S·B·H·D elements), each rank adds its
heads' exact dK/dV into the full-size partials that are reduce-scattered anyway, and the
prefix rows of out and dq come back to rank 0 through one more all-gather. The exact GEMMs'
split-K slicing depends on the number of heads, so those S rows of out equal the unsharded
call's up to float32 summation order; every sampled row stays bit-identical.

``comm`` is any object with ``rank``, ``world``, ``all_gather_seq(out, chunk)`` and
``reduce_scatter_seq(out_chunk, full)`` along dim 0; ``TorchDistComm`` is the NCCL one.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops


class TorchDistComm:
    """Collectives over the default torch.distributed group (NCCL on GPUs; gloo works
    for CPU tensors through all_gather / all_reduce)."""

    def __init__(self, group=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.nccl = dist.get_backend(group) == "nccl"

    def all_gather_seq(self, out: torch.Tensor, chunk: torch.Tensor) -> None:
        if self.nccl:
            self.dist.all_gather_into_tensor(out, chunk.contiguous(), group=self.group)
        else:
            self.dist.all_gather(list(out.chunk(self.world, dim=0)), chunk.contiguous(),
                                 group=self.group)

    def reduce_scatter_seq(self, out_chunk: torch.Tensor, full: torch.Tensor) -> None:
        if self.nccl:
            self.dist.reduce_scatter_tensor(out_chunk, full.contiguous(), group=self.group)
        else:
            t = full.contiguous().clone()
            self.dist.all_reduce(t, group=self.group)
            out_chunk.copy_(t.chunk(self.world, dim=0)[self.rank])


@dataclass(frozen=True)
class SpPlan:
    """Which of a rank's queries take which path (positions are global)."""

    seq_len: int          # N
    chunk: int            # n = N / R
    q0: int               # first query position of this rank
    exact: int            # local queries [0, exact) take the exact causal path
    sampled_t0: int       # index of the first sampled query in the global sampled order
    causal: bool
    prefix: int = 0       # global exact queries [0, prefix) (causal hybrid)

    def balanced(self, world: int, heads: int) -> bool:
        """True when the exact prefix is split over the ranks by heads: it lies inside rank
        0's chunk and the heads divide evenly (``BALANCE_PREFIX`` switches it off)."""
        return (BALANCE_PREFIX and world > 1 and 0 < self.prefix <= self.chunk
                and heads % world == 0)

    @property
    def sampled_offset(self) -> int:
        """Causal boundary of the first sampled local query."""
        return self.q0 + self.exact


def plan(seq_len: int, world: int, rank: int, num_samples: int, causal: bool) -> SpPlan:
    """Split of a rank's queries between the exact causal prefix and the sampler.

    treeattn-torch's causal mode (_tree_mha.py:379-412) gives the first S = num_samples
    queries exact causal attention when L > S and samples the rest with causal offset S.
    """
    if world <= 0 or not 0 <= rank < world or seq_len % world:
        raise ValueError(f"cannot split {seq_len} positions evenly over {world} ranks")
    n = seq_len // world
    if not ops.is_power_of_two(n):
        raise ValueError(f"the per-rank chunk {n} must be a power of two")
    q0 = rank * n
    if not causal:
        return SpPlan(seq_len, n, q0, 0, q0, False)
    hybrid = seq_len > num_samples
    exact = min(max(num_samples - q0, 0), n) if hybrid else 0
    t0 = q0 + exact - (num_samples if hybrid else 0)
    return SpPlan(seq_len, n, q0, exact, t0, True, num_samples if hybrid else 0)


BALANCE_PREFIX = True


def _prefix_heads(comm, heads: int) -> slice:
    hr = heads // comm.world
    return slice(comm.rank * hr, (comm.rank + 1) * hr)


def _from_rank0(comm, rows: torch.Tensor) -> torch.Tensor:
    """Rank 0's (E, B, H, D) rows on every rank (all-gather; the other ranks' slots unused)."""
    E = rows.shape[0]
    buf = torch.empty((comm.world * E,) + tuple(rows.shape[1:]), device=rows.device,
                      dtype=rows.dtype)
    comm.all_gather_seq(buf, rows)
    return buf[:E]


def _heads_to_rank0(comm, dst, part: torch.Tensor) -> None:
    """Every rank's (E, B, H/R, D) head slice into rank 0's (E, B, H, D) ``dst``."""
    E, B, hr, D = part.shape
    R = comm.world
    buf = torch.empty((R * E, B, hr, D), device=part.device, dtype=part.dtype)
    comm.all_gather_seq(buf, part)
    if comm.rank == 0:
        dst.copy_(buf.view(R, E, B, hr, D).permute(1, 2, 0, 3, 4).reshape(E, B, R * hr, D))


def _offset_rng(base, draws: int):
    from . import _lib as L

    return L.Rng(base.seed, base.offset + draws * base.offset_step, base.offset_step,
                 base.draw_stride)


def reserve_stream(device, batch: int, seq_len: int, heads: int, num_samples: int, causal: bool):
    """Reserve the FULL problem's noise from the CUDA generator (every rank does the same)."""
    ln = ops.log_n_of(seq_len)
    if causal:
        sampled = seq_len - num_samples if seq_len > num_samples else seq_len
        return ops.reserve_causal_stream(device, batch * heads * num_samples * 2, sampled * ln)
    return ops.reserve_gumbel_stream(device, seq_len * batch * heads * num_samples * 2, ln)


@dataclass
class SpSaved:
    """What the backward needs from the forward."""

    plan: SpPlan
    num_samples: int
    tensors: tuple
    prefix_q: torch.Tensor | None = None   # rank 0's prefix query rows (balanced prefix)


def sp_forward(q, k, v, num_samples: int, causal: bool, comm, rng):
    """Forward on this rank's bshd chunks (B, n, H, D): returns (out chunk, SpSaved)."""
    B, n, H, D = q.shape
    R = comm.world
    N = n * R
    S = num_samples
    p = plan(N, R, comm.rank, S, causal)
    dev = q.device
    kf = torch.empty((N, B, H, D), device=dev, dtype=k.dtype)
    vf = torch.empty((N, B, H, D), device=dev, dtype=v.dtype)
    comm.all_gather_seq(kf, k.transpose(0, 1))
    comm.all_gather_seq(vf, v.transpose(0, 1))
    k_int = ops.tree_build(kf)
    out = torch.empty_like(q)
    qv, ov = q.transpose(0, 1), out.transpose(0, 1)
    if not causal:
        res = ops.forward(qv, k_int, vf, S, out=ov, rng=rng, query_rows=(p.q0, N))
        return out, SpSaved(p, S, (q, k_int, vf, res.leaf, res.weights, res.branch_prob))
    e = p.exact
    qpre = None
    if p.balanced(R, H):
        E, hs = p.prefix, _prefix_heads(comm, H)
        qpre = _from_rank0(comm, qv[:E])
        opart = torch.empty((E, B, hs.stop - hs.start, D), device=dev, dtype=q.dtype)
        ops.exact_forward(qpre[:, :, hs], k_int[:, :, hs], vf[:, :, hs], True, 0, out=opart,
                          want_weights=False)
        _heads_to_rank0(comm, ov[:E], opart)
    elif e:
        ops.exact_forward(qv[:e], k_int, vf, True, p.q0, out=ov[:e], want_weights=False)
    saved = (q, k_int, vf)
    if e < n:
        rng_l = _offset_rng(rng, p.sampled_t0 * ops.log_n_of(N))
        _, st = ops.causal_forward(qv[e:], k_int, vf, S, p.sampled_offset, out=ov[e:], rng=rng_l)
        saved += (st.leaf, st.weights, st.branch_prob, st.corrected, st.masses)
    return out, SpSaved(p, S, saved, qpre)


def sp_backward(saved: SpSaved, grad_out, comm):
    """Backward of ``sp_forward``: (dq, dk, dv) chunks (B, n, H, D) in the input dtype."""
    p, S = saved.plan, saved.num_samples
    q, k_int, vf = saved.tensors[:3]
    B, n, H, D = q.shape
    N = p.seq_len
    dev = q.device
    grad_out = grad_out if grad_out.stride(-1) == 1 else grad_out.contiguous()
    qv, gv = q.transpose(0, 1), grad_out.transpose(0, 1)
    dq = torch.empty_like(q)
    dqv = dq.transpose(0, 1)
    dk_int = torch.empty((B, H, N - 1, D), device=dev, dtype=torch.float32).permute(2, 0, 1, 3)
    dv32 = torch.empty((N, B, H, D), device=dev, dtype=torch.float32)
    if not p.causal:
        leaf, weights, bp = saved.tensors[3:]
        ops.backward(qv, k_int, vf, gv, leaf, weights, bp, S, dq=dqv, dk=dk_int, dv=dv32)
    else:
        e = p.exact
        if e < n:
            st = ops.CausalState(*saved.tensors[3:], p.sampled_offset)
            ops.causal_backward(qv[e:], k_int, vf, gv[e:], st, S, dq=dqv[e:], dk=dk_int, dv=dv32)
        else:
            dk_int.zero_()
            dv32.zero_()
        if saved.prefix_q is not None:
            E, hs, qpre = p.prefix, _prefix_heads(comm, H), saved.prefix_q
            gpre = _from_rank0(comm, gv[:E])
            dqpart = torch.empty((E, B, hs.stop - hs.start, D), device=dev, dtype=q.dtype)
            ops.exact_backward(qpre[:, :, hs], k_int[:, :, hs], vf[:, :, hs], gpre[:, :, hs], True,
                               0, dq=dqpart, dk=dk_int[:, :, hs], dv=dv32[:, :, hs],
                               accumulate=True)
            _heads_to_rank0(comm, dqv[:E], dqpart)
        elif e:
            ops.exact_backward(qv[:e], k_int, vf, gv[:e], True, p.q0, dq=dqv[:e], dk=dk_int,
                               dv=dv32, accumulate=True)
    dk32 = torch.empty((N, B, H, D), device=dev, dtype=torch.float32)
    ops.tree_build_backward(dk_int, dk32)
    dk_loc = torch.empty((n, B, H, D), device=dev, dtype=torch.float32)
    dv_loc = torch.empty((n, B, H, D), device=dev, dtype=torch.float32)
    comm.reduce_scatter_seq(dk_loc, dk32)
    comm.reduce_scatter_seq(dv_loc, dv32)
    dk = dk_loc.transpose(0, 1).to(q.dtype).contiguous()
    dv = dv_loc.transpose(0, 1).to(q.dtype).contiguous()
    return dq, dk, dv


class SequenceParallelTreeAttention(torch.autograd.Function):
    """Autograd op over this rank's bshd chunks (B, n, H, D) of q, k, v."""

    @staticmethod
    def forward(ctx, q, k, v, num_samples, causal, comm, rng):
        out, ctx.sp_saved = sp_forward(q, k, v, num_samples, causal, comm, rng)
        ctx.comm = comm
        return out

    @staticmethod
    def backward(ctx, grad_out):
        dq, dk, dv = sp_backward(ctx.sp_saved, grad_out, ctx.comm)
        ctx.sp_saved = None
        return dq, dk, dv, None, None, None, None


def sp_tree_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False, *,
                      num_samples: int, comm=None, rng=None) -> torch.Tensor:
    """Sequence-parallel ``tree_attention`` on this rank's bshd chunks (B, N/R, H, D).

    ``comm`` defaults to ``TorchDistComm()`` (the default process group). ``rng`` is the full
    problem's noise plan (``reserve_stream``); by default it is reserved from this rank's
    CUDA generator, so ranks seeded alike draw alike.
    """
    if q.dim() != 4 or q.shape != k.shape or q.shape != v.shape:
        raise ValueError("q, k, v must share one (B, n, H, D) shape")
    comm = comm if comm is not None else TorchDistComm()
    B, n, H, D = q.shape
    N = n * comm.world
    if not ops.is_power_of_two(N) or N < 2:
        raise ValueError(f"treeattn_b200 requires power-of-two seqlen, got {N}")
    plan(N, comm.world, comm.rank, num_samples, causal)  # validates the split
    if rng is None:
        rng = reserve_stream(q.device, B, N, H, num_samples, causal)
    q, k, v = (t if t.stride(-1) == 1 else t.contiguous() for t in (q, k, v))
    return SequenceParallelTreeAttention.apply(q, k, v, num_samples, bool(causal), comm, rng)
