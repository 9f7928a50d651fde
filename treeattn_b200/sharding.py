"""Head/batch sharding across GPUs: one process per GPU, independent (batch, head) trees.

Every (batch, head) tree of stochastic tree attention is independent (the reference's
sampler, _autograd.py:141-220, never mixes heads), so a multi-GPU run splits the (batch,
head) units across ranks and needs no collective on the data path. The one coupling is the
random stream: the reference draws each depth's Gumbel noise as ONE torch exponential_()
call over the full (L, B, H, S, 2) tensor (_autograd.py:188-195), whose element -> philox
mapping depends on the full size. A shard therefore reserves the generator offsets of the
full draw and fills only its own slice at the full draw's global element indices
(ta_gumbel_fill_shard), so the union of the shards' results equals one unsharded call made
after the same ``torch.manual_seed`` -- sampled leaves bit for bit.

Causal mode is not shardable this way: its correction predicate (every (b, h, s) sample of
a query on the boundary node, _tree_mha.py:204-207) couples all heads of a query.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class ShardSpec:
    """This rank's contiguous block of batches and heads of the full problem."""

    batch_total: int
    batch0: int
    batch_count: int
    head_total: int
    head0: int
    head_count: int

    def __post_init__(self):
        if self.batch_total <= 0 or self.head_total <= 0:
            raise ValueError("batch_total and head_total must be > 0")
        if self.batch_count <= 0 or self.head_count <= 0:
            raise ValueError("a shard must own at least one batch and one head")
        if self.batch0 < 0 or self.batch0 + self.batch_count > self.batch_total:
            raise ValueError("batch range outside the full batch")
        if self.head0 < 0 or self.head0 + self.head_count > self.head_total:
            raise ValueError("head range outside the full head count")

    @property
    def is_full(self) -> bool:
        return self.batch_count == self.batch_total and self.head_count == self.head_total

    def units(self) -> list[tuple[int, int]]:
        """The (batch, head) pairs this shard owns."""
        return [(b, h) for b in range(self.batch0, self.batch0 + self.batch_count)
                for h in range(self.head0, self.head0 + self.head_count)]

    def slices(self) -> tuple[slice, slice]:
        """(batch, head) index slices of this shard in the full tensors."""
        return (slice(self.batch0, self.batch0 + self.batch_count),
                slice(self.head0, self.head0 + self.head_count))


def partition(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous split of ``total`` units over ``world`` ranks: (start, count) of ``rank``.
    The first ``total % world`` ranks take one extra unit."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if total < world:
        raise ValueError(f"cannot split {total} units over {world} ranks")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def shard_for_rank(batch: int, heads: int, rank: int, world: int, axis: str = "auto") -> ShardSpec:
    """This rank's shard of a (batch, heads) problem.

    ``axis`` "batch" splits whole batches, "head" splits heads (every rank keeps every batch),
    "auto" splits batches when there are at least as many as ranks, else heads.
    """
    if axis == "auto":
        axis = "batch" if batch >= world else "head"
    if axis == "batch":
        b0, bc = partition(batch, rank, world)
        return ShardSpec(batch, b0, bc, heads, 0, heads)
    if axis == "head":
        h0, hc = partition(heads, rank, world)
        return ShardSpec(batch, 0, batch, heads, h0, hc)
    raise ValueError(f"unknown shard axis {axis!r}")


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank scalar over the default process group (the timing rule for
    multi-GPU numbers); the value itself when torch.distributed is not initialised."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_heads(local, spec: ShardSpec, head_dim_axis: int = 2):
    """All-gather every rank's shard of a (B, S, H, D)-like tensor into the full tensor.

    For parity checks and result collection only -- the op itself needs no collective.
    Every rank must hold a shard of the same shape (an even split).
    """
    import torch
    import torch.distributed as dist

    world = dist.get_world_size()
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local.contiguous())
    axis = 0 if spec.batch_count != spec.batch_total else head_dim_axis
    return torch.cat(parts, dim=axis)
