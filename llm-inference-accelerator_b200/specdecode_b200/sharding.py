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


class _DeviceWords:
    """A device allocation seen as a 1-D tensor of 16-bit words (``torch.as_tensor``
    reads ``__cuda_array_interface__``; the caller views it as bf16 / fp16)."""

    def __init__(self, pointer: int, words: int) -> None:
        self.__cuda_array_interface__ = {"shape": (words,), "typestr": "<i2", "data": (pointer, False),
                                         "version": 3, "strides": None}


class PeerHeadGather:
    """KV-head tensor-parallel verify attention whose all-gather is fused into
    the attention launch (``sdc_paged_verify_attention_gather``).

    Every rank owns one device buffer holding its gathered output ``[batch,
    query_heads, window, head_dim]`` and one flag word per rank.  The buffers
    are mapped into every rank's process once (inter-process handles
    exchanged over ``group``, the only use of torch.distributed here).  On a
    call, the kernel that writes this rank's output rows stores each row into
    every rank's buffer over NVLink; one more launch then raises this rank's
    flag in every buffer and waits (bounded) until every rank's flag in its
    own buffer carries the call's epoch.  When ``__call__`` returns, the
    returned tensor -- a view of this rank's buffer, valid until ``close`` --
    holds every rank's heads once the stream reaches that point.  No
    collective runs on the data path and no library kernel touches another
    GPU's memory.

    ``cache`` is this rank's head-shard pool (``shard.kv_per_rank`` KV
    heads); every rank must call with the same batch shape, in the same
    order.
    """

    def __init__(self, cache, shard: HeadShard, batch: int, window: int, *, dtype=None, group=None) -> None:
        import ctypes

        import torch
        import torch.distributed as dist

        from specdecode_b200 import _lib

        if shard.world > 8:
            raise ValueError("the fused head gather serves at most 8 ranks")
        if cache.config.num_heads != shard.kv_per_rank:
            raise ValueError("the cache must hold this rank's KV heads only")
        self.cache = cache
        self.shard = shard
        self.batch = int(batch)
        self.window = int(window)
        self.dtype = torch.bfloat16 if dtype is None else dtype
        if self.dtype not in (torch.bfloat16, torch.float16):
            raise ValueError("the gathered output is bf16 or fp16")
        self.group = group
        self.library = cache.library
        lib = self.library.handle
        D = cache.config.head_dim
        self.shape = (self.batch, shard.query_heads, self.window, D)
        elements = self.batch * shard.query_heads * self.window * D
        self._out_bytes = -(-elements * 2 // 256) * 256
        total = self._out_bytes + 256
        own = ctypes.c_void_p()
        self.library.check(lib.sdc_peer_buffer_alloc(total, ctypes.byref(own)), "peer buffer allocation")
        self._own = int(own.value)
        self._opened: list[int] = []
        try:
            handle = (ctypes.c_char * _lib.PEER_HANDLE_BYTES)()
            self.library.check(lib.sdc_peer_buffer_export(self._own, handle, len(handle)), "peer buffer export")
            handles: list = [None] * shard.world
            if shard.world > 1:
                dist.all_gather_object(handles, bytes(handle), group=group)
            else:
                handles = [bytes(handle)]
            bases = []
            for r, h in enumerate(handles):
                if r == shard.rank:
                    bases.append(self._own)
                    continue
                ptr = ctypes.c_void_p()
                raw = (ctypes.c_char * len(h)).from_buffer_copy(h)
                self.library.check(lib.sdc_peer_buffer_open(raw, len(h), ctypes.byref(ptr)), "peer buffer open")
                self._opened.append(int(ptr.value))
                bases.append(int(ptr.value))
        except BaseException:
            self._release_maps()
            raise
        self._outs = (ctypes.c_void_p * shard.world)(*bases)
        self._flags = (ctypes.c_void_p * shard.world)(*[b + self._out_bytes for b in bases])
        words = torch.as_tensor(_DeviceWords(self._own, elements), device=cache.device)
        self.output = words.view(self.dtype).view(self.shape)
        self._attention_sizes: dict[int, int] = {}
        self._workspace = None
        self.epoch = 0

    def _release_maps(self) -> None:
        lib = self.library.handle
        for ptr in self._opened:
            lib.sdc_peer_buffer_close(ptr)
        self._opened = []
        if self._own:
            lib.sdc_peer_buffer_free(self._own)
            self._own = 0

    def __call__(self, query, block_tables, context_lens, max_context_len: int, layer: int):
        import ctypes

        import torch

        from specdecode_b200.kv_cache import _dtype_code

        if self._own == 0:
            raise RuntimeError("the head gather is closed")
        if tuple(query.shape) != self.shape or query.dtype != self.dtype:
            raise ValueError(f"query must be {self.shape} in {self.dtype}")
        q = shard_query(query, self.shard).contiguous()
        B, hq, kw, _ = (int(d) for d in q.shape)
        if block_tables.dtype != torch.int32 or context_lens.dtype != torch.int32:
            raise ValueError("block tables and context lengths must be int32")
        device = torch.device(self.cache.device)
        if query.device != device or block_tables.device != device or context_lens.device != device:
            raise ValueError("query, block tables and context lengths must be on the pool's device")
        block_tables = block_tables.contiguous()
        lib = self.library.handle
        need = self._attention_sizes.get(int(max_context_len))
        if need is None:
            size = ctypes.c_size_t()
            self.library.check(lib.sdc_paged_attention_workspace_size(
                B, hq, self.cache.config.num_heads, self.cache.config.head_dim, kw, int(max_context_len),
                ctypes.byref(size)), "attention workspace sizing")
            need = self._attention_sizes[int(max_context_len)] = int(size.value)
        if self._workspace is None or self._workspace.numel() < need:
            self._workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=self.cache.device)
        self.epoch = self.epoch % 0xFFFFFFFF + 1
        stream = torch.cuda.current_stream(self.cache.device)
        self.library.check(lib.sdc_paged_verify_attention_gather(
            self.cache.pool_desc, int(layer), q.data_ptr(), _dtype_code(q.dtype), B, hq, kw,
            block_tables.data_ptr(), block_tables.stride(0), context_lens.data_ptr(), int(max_context_len),
            self._outs, self._flags, self.shard.world, self.shard.rank, self.epoch, self._workspace.data_ptr(),
            self._workspace.numel(), self.cache._status.data_ptr(), stream.cuda_stream), "fused head gather")
        return self.output

    def close(self) -> None:
        """Unmaps the other ranks' buffers and frees this rank's, after every
        rank has finished its calls (a barrier over ``group``)."""
        import torch
        import torch.distributed as dist

        if self._own == 0:
            return
        torch.cuda.synchronize(self.cache.device)
        if self.shard.world > 1:
            dist.barrier(group=self.group)
        self.output = None
        self._release_maps()
