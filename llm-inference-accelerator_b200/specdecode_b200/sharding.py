"""Placement of the paged verify path over the GPUs of one node.

Two partitions, one process per GPU:

* Requests, data-parallel (verify batches, append/rollback): sequences are
  independent, so every rank owns whole sequences, its own page pool and
  block tables, and nothing crosses NVLink on the data path.  ``lpt_partition``
  balances ranks by total context length (longest processing time first: the
  attention cost of a sequence is proportional to its cached tokens).
* KV heads, tensor-parallel (long contexts, where one batch per GPU would be
  too few sequences to fill the node): rank g owns KV heads
  ``[g·Hkv/G, (g+1)·Hkv/G)`` and the matching query heads (query head h reads
  KV head ``h // (Hq/Hkv)``, so a contiguous block of KV heads pairs with a
  contiguous block of query heads), runs attention over the full context for
  its heads, and one all-gather of the outputs rebuilds ``[B, Hq, k, D]``.

The collective is ``all_gather_into_tensor`` (NCCL over NVLink on GPUs; the
list form on gloo, which the CPU tests use).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence


def lpt_partition(lengths: Sequence[int], world: int) -> list[list[int]]:
    """Sequence indices per rank, longest first onto the least-loaded rank.

    Ties go to the lower index / lower rank, so the result is deterministic;
    each rank's list is returned in ascending order.
    """
    if world < 1:
        raise ValueError("world size must be at least 1")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    loads = [0] * world
    parts: list[list[int]] = [[] for _ in range(world)]
    for index in order:
        rank = min(range(world), key=lambda r: (loads[r], r))
        parts[rank].append(index)
        loads[rank] += int(lengths[index])
    return [sorted(p) for p in parts]


@dataclass(frozen=True)
class HeadShard:
    """The KV heads and query heads one rank owns."""

    rank: int
    world: int
    kv_heads: int
    query_heads: int

    @property
    def kv_per_rank(self) -> int:
        return self.kv_heads // self.world

    @property
    def q_per_rank(self) -> int:
        return self.query_heads // self.world

    @property
    def kv_range(self) -> range:
        return range(self.rank * self.kv_per_rank, (self.rank + 1) * self.kv_per_rank)

    @property
    def q_range(self) -> range:
        return range(self.rank * self.q_per_rank, (self.rank + 1) * self.q_per_rank)


def head_shard(rank: int, world: int, kv_heads: int, query_heads: int) -> HeadShard:
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world size {world}")
    if kv_heads % world:
        raise ValueError(f"{kv_heads} KV heads do not split over {world} ranks")
    if query_heads % kv_heads:
        raise ValueError("query heads must be a multiple of KV heads")
    return HeadShard(rank, world, kv_heads, query_heads)


def shard_query(query, shard: HeadShard):
    """This rank's query heads of a ``[B, Hq, k, D]`` query (a view)."""
    if query.shape[1] != shard.query_heads:
        raise ValueError("query head count does not match the shard")
    return query[:, shard.q_range.start:shard.q_range.stop]


def gather_heads(local, shard: HeadShard, group=None):
    """All-gather ``[B, Hq/G, k, D]`` head shards into ``[B, Hq, k, D]``."""
    import torch
    import torch.distributed as dist

    local = local.contiguous()
    if shard.world == 1:
        return local
    B, hq_local, k, D = local.shape
    if dist.get_backend(group) == "nccl":
        buffer = torch.empty((shard.world,) + tuple(local.shape), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(buffer, local, group=group)
    else:
        parts = [torch.empty_like(local) for _ in range(shard.world)]
        dist.all_gather(parts, local, group=group)
        buffer = torch.stack(parts)
    return buffer.permute(1, 0, 2, 3, 4).reshape(B, shard.world * hq_local, k, D)


class TensorParallelVerifyAttention:
    """Verify attention with KV heads split over the ranks of ``group``.

    ``attention(query_shard, block_tables, context_lens, max_context_len,
    layer)`` is this rank's attention over its own head-shard pool (for
    example a ``PagedVerifyAttention`` over a cache built with
    ``shard.kv_per_rank`` heads); calling the object runs it on this rank's
    query heads and all-gathers the outputs.  Every rank must call it in the
    same order with the same batch (the all-gather is a collective).
    """

    def __init__(self, attention: Callable, shard: HeadShard, group=None) -> None:
        self.attention = attention
        self.shard = shard
        self.group = group

    def local(self, query, block_tables, context_lens, max_context_len: int, layer: int):
        return self.attention(shard_query(query, self.shard), block_tables, context_lens, max_context_len, layer)

    def __call__(self, query, block_tables, context_lens, max_context_len: int, layer: int):
        out = self.local(query, block_tables, context_lens, max_context_len, layer)
        return gather_heads(out, self.shard, self.group)
