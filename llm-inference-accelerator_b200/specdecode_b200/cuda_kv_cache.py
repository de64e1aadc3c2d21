"""Kernel-facing views of the device pool and the fused paged attention.

Keeps the reference's device-side surface (src/specdecode/cuda_kv_cache.py):

* ``CudaPagedKVCacheView`` — ``keys``/``values`` int8
  ``[block, offset, layer, head, dim]``, ``key_scales``/``value_scales`` f32
  ``[block, offset, layer, head]``, ``block_table``, ``token_count``,
  ``block_size`` (:21-37).  Here the tensors are permuted views of the pool's
  physical ``[block, layer, head, offset, dim]`` storage, and the block table
  is the sequence's int32 device row.
* ``CudaPagedKVCacheStorage`` — binds one sequence of a device
  ``PagedKVCache`` and returns its view from ``synchronize`` (:52-367).  The
  pool is already on the device, so synchronisation moves no data; the stats
  keep the reference's meaning (tokens written / slots cleared since the last
  synchronisation).
* ``submit_paged_attention`` — same signature and errors (:370-503); the
  gather/dequantize/GQA/mask/SDPA sequence is one fused kernel launch.

``PagedVerifyAttention`` is the batched form: many sequences, one launch.

The ``runtime`` these functions take is the caller's own execution runtime,
used as the reference's code uses its ``CudaExecutionRuntime``
(src/specdecode/cuda.py): an object with a ``device`` attribute and
``submit_target(fn, *, wait_for=(), label=...)`` /
``submit_transfer(fn, *, wait_for=(), label=...)`` methods that run ``fn``
on the runtime's target / transfer stream and return a task.  The
reference's runtime works unchanged; this module defines none of its own.
"""

from __future__ import annotations

import math
from collections.abc import Hashable, Sequence
from dataclasses import dataclass
from typing import Any

from . import _lib
from .kv_cache import KVCacheConfig, PagedKVCache, _dtype_code


class CudaPagedKVCacheError(RuntimeError):
    """Raised when a cache cannot be bound to CUDA storage."""


class CudaPagedAttentionError(RuntimeError):
    """Raised when cache tensors cannot serve an attention call."""


@dataclass(frozen=True, slots=True)
class CudaPagedKVCacheView:
    keys: Any
    values: Any
    key_scales: Any
    value_scales: Any
    block_table: Any
    token_count: int
    block_size: int
    context_lens: Any = None  # optional int32 [1] device length for the kernel


@dataclass(frozen=True, slots=True)
class CudaPagedKVCacheStats:
    synchronizations: int
    uploaded_tokens: int
    cleared_tokens: int
    active_tokens: int
    active_blocks: int
    device_storage_bytes: int


def pool_from_view(view: CudaPagedKVCacheView) -> _lib.PagePool:
    """Pool descriptor for the kernels from a view's tensors and strides."""
    keys, values, ks, vs = view.keys, view.values, view.key_scales, view.value_scales
    if keys.dim() != 5 or tuple(values.shape) != tuple(keys.shape):
        raise CudaPagedAttentionError("packed K/V tensors have invalid geometry")
    if ks.dim() != 4 or tuple(vs.shape) != tuple(ks.shape):
        raise CudaPagedAttentionError("packed scale tensors have invalid geometry")
    if tuple(ks.shape) != tuple(keys.shape[:-1]) or keys.shape[1] != view.block_size:
        raise CudaPagedAttentionError("packed scales do not match K/V geometry")
    nb, bs, L, H, D = (int(d) for d in keys.shape)
    if values.stride() != keys.stride() or vs.stride() != ks.stride():
        raise CudaPagedAttentionError("keys and values must share one layout")
    sb, so, sl, sh, sd = keys.stride()
    tb, to, tl, th = ks.stride()
    if sd != 1 or so != D or to != 1:
        raise CudaPagedAttentionError(
            "pool layout not supported: a page's token rows must be contiguous "
            "(dim stride 1, offset stride head_dim, scale offset stride 1)")
    return _lib.PagePool(keys.data_ptr(), values.data_ptr(), ks.data_ptr(), vs.data_ptr(),
                         nb, bs, L, H, D, sb, sl, sh, tb, tl, th)


class PagedVerifyAttention:
    """Batched fused paged verify/decode attention over one device pool.

    ``__call__(query, block_tables, context_lens, max_context_len, layer)``
    with query ``[B, Hq, window, D]`` (bf16/fp16/fp32, device),
    block_tables int32 ``[B, stride]`` and context_lens int32 ``[B]`` on the
    device returns ``[B, Hq, window, D]`` in the query dtype.  The workspace is
    cached and grown per shape; launches go to the current stream.
    """

    def __init__(self, pool: _lib.PagePool, device, library: _lib.CudaLibrary, status) -> None:
        self.pool = pool
        self.device = device
        self.library = library
        self.status = status
        self._workspace = None
        self._sizes: dict[tuple[int, int, int, int], int] = {}
        self._checked_device = None  # self.device with its index, set on the first call

    @classmethod
    def for_cache(cls, cache: PagedKVCache) -> "PagedVerifyAttention":
        return cls(cache.pool_desc, cache.device, cache.library, cache._status)

    def workspace_bytes(self, batch: int, query_heads: int, window: int, max_context_len: int) -> int:
        import ctypes

        key = (batch, query_heads, window, max_context_len)
        if key in self._sizes:
            return self._sizes[key]
        size = ctypes.c_size_t()
        self.library.check(self.library.handle.sdc_paged_attention_workspace_size(
            batch, query_heads, self.pool.num_heads, self.pool.head_dim, window, max_context_len,
            ctypes.byref(size)), "attention workspace sizing")
        self._sizes[key] = int(size.value)
        return int(size.value)

    def __call__(self, query, block_tables, context_lens, max_context_len: int, layer: int, *, out=None):
        import torch

        if query.dim() != 4:
            raise CudaPagedAttentionError("query must use [batch, heads, tokens, head_dim] layout")
        B, Hq, kw, D = (int(d) for d in query.shape)
        if block_tables.dtype != torch.int32 or context_lens.dtype != torch.int32:
            raise CudaPagedAttentionError("block tables and context lengths must be int32")
        if block_tables.dim() != 2 or block_tables.shape[0] != B or context_lens.shape != (B,):
            raise CudaPagedAttentionError("block tables / context lengths do not match the batch")
        if block_tables.stride(1) != 1:
            block_tables = block_tables.contiguous()
        query = query.contiguous()
        if out is None:
            out = torch.empty_like(query)
        elif out.shape != query.shape or out.dtype != query.dtype or not out.is_contiguous():
            raise CudaPagedAttentionError("out must be a contiguous tensor of the query's shape and dtype")
        device = self._checked_device
        if device is None:
            device = torch.device(self.device)
            if device.type == "cuda" and device.index is None:
                device = torch.device("cuda", torch.cuda.current_device())
            self._checked_device = device
        if query.device != device or out.device != device or block_tables.device != device or \
                context_lens.device != device:
            raise CudaPagedAttentionError("query, out, block tables and context lengths must be on the pool's device")
        need = self.workspace_bytes(B, Hq, kw, int(max_context_len))
        if self._workspace is None or self._workspace.numel() < need:
            self._workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=self.device)
        stream = torch.cuda.current_stream(self.device)
        status = self.library.handle.sdc_paged_verify_attention(
            self.pool, int(layer), query.data_ptr(), _dtype_code(query.dtype), B, Hq, kw,
            block_tables.data_ptr(), block_tables.stride(0), context_lens.data_ptr(), int(max_context_len),
            out.data_ptr(), self._workspace.data_ptr(), self._workspace.numel(), self.status.data_ptr(),
            stream.cuda_stream)
        self.library.check(status, "paged verify attention")
        return out


def paged_verify_attention(cache: PagedKVCache, query, sequence_ids: Sequence[Hashable], layer: int, *, out=None):
    """Batched attention for ``sequence_ids`` of ``cache`` (query ``[B, Hq, window, D]``)."""
    attention = getattr(cache, "_verify_attention", None)
    if attention is None:
        attention = PagedVerifyAttention.for_cache(cache)
        cache._verify_attention = attention
    tables, lens, max_len = cache.attention_inputs(sequence_ids)
    return attention(query, tables, lens, max_len, layer, out=out)


class CudaPagedKVCacheStorage:
    """Binds one sequence of a device ``PagedKVCache`` for kernel consumption."""

    def __init__(self, config: KVCacheConfig, runtime: Any, *, name: str = "paged_kv") -> None:
        if not isinstance(name, str) or not name.strip():
            raise ValueError("CUDA paged-cache storage name cannot be empty")
        self.config = config
        self.runtime = runtime
        self.name = name
        self._sequence_id: Hashable | None = None
        self._cache: PagedKVCache | None = None
        self._tokens = 0
        self._slots: tuple[int, ...] = ()
        self._blocks = 0
        self._synchronizations = 0
        self._uploaded = 0
        self._cleared = 0

    def _validate(self, cache: PagedKVCache) -> None:
        if not isinstance(cache, PagedKVCache):
            raise TypeError("cache must be a device PagedKVCache")
        if cache.config != self.config:
            raise CudaPagedKVCacheError("cache and CUDA paged-cache configurations differ")

    @property
    def stats(self) -> CudaPagedKVCacheStats:
        cfg = self.config
        return CudaPagedKVCacheStats(
            synchronizations=self._synchronizations, uploaded_tokens=self._uploaded,
            cleared_tokens=self._cleared, active_tokens=self._tokens, active_blocks=self._blocks,
            device_storage_bytes=cfg.capacity_tokens * cfg.quantized_bytes_per_token)

    def _view_of(self, cache: PagedKVCache, sequence_id: Hashable, length: int) -> CudaPagedKVCacheView:
        row = cache.table_row(sequence_id)
        nblk = (length + self.config.block_size - 1) // self.config.block_size
        return CudaPagedKVCacheView(
            keys=cache.keys_view, values=cache.values_view, key_scales=cache.key_scales_view,
            value_scales=cache.value_scales_view, block_table=cache.block_tables[row, :nblk],
            token_count=length, block_size=self.config.block_size,
            context_lens=cache.context_lens[row:row + 1])

    @property
    def view(self) -> CudaPagedKVCacheView:
        if self._cache is None or self._sequence_id is None:
            raise CudaPagedKVCacheError("storage has not been synchronized")
        return self._view_of(self._cache, self._sequence_id, self._tokens)

    def synchronize(self, cache: PagedKVCache, sequence_id: Hashable) -> Any:
        self._validate(cache)
        length = cache.sequence_length(sequence_id)
        if self._sequence_id is not None and sequence_id != self._sequence_id:
            raise CudaPagedKVCacheError("CUDA paged-cache storage is already bound to another sequence")
        stable = cache.changes_since(sequence_id, self._tokens)
        if cache is self._cache and sequence_id == self._sequence_id and stable == length == self._tokens:
            # nothing appended or rolled back since the last call: the slots
            # and block count are unchanged, nothing is uploaded or cleared
            self._synchronizations += 1
            view = self._view_of(cache, sequence_id, length)
            return self.runtime.submit_transfer(lambda: view, label=f"specdecode.transfer.{self.name}.synchronize")
        table = cache.block_table(sequence_id)
        bs = self.config.block_size
        new_slots = tuple(table[t // bs] * bs + t % bs for t in range(length))
        stale = set(self._slots[stable:]) - set(new_slots[stable:])
        self._uploaded += length - min(stable, length)
        self._cleared += len(stale)
        self._sequence_id = sequence_id
        self._cache = cache
        self._tokens = length
        self._slots = new_slots
        self._blocks = len(table)
        self._synchronizations += 1
        view = self._view_of(cache, sequence_id, length)
        return self.runtime.submit_transfer(lambda: view, label=f"specdecode.transfer.{self.name}.synchronize")


def submit_paged_attention(runtime: Any, query: Any, cache: CudaPagedKVCacheView, layer_index: int, *,
                           wait_for: Sequence[Any] = ()) -> Any:
    """Fused causal attention over one cached sequence (reference signature).

    ``query`` is ``[1, query_heads, query_tokens, head_dim]`` and stands for
    the last ``query_tokens`` cached positions.  One kernel launch on the
    target stream replaces the reference's gather/dequantize/expand/SDPA.
    """
    import torch

    if not isinstance(cache, CudaPagedKVCacheView):
        raise TypeError("cache must be a CudaPagedKVCacheView")
    if (isinstance(cache.token_count, bool) or not isinstance(cache.token_count, int) or cache.token_count < 1
            or isinstance(cache.block_size, bool) or not isinstance(cache.block_size, int)
            or cache.block_size < 1):
        raise CudaPagedAttentionError("packed cache metadata is invalid")
    query_shape = tuple(int(d) for d in query.shape)
    if len(query_shape) != 4 or query_shape[0] != 1:
        raise CudaPagedAttentionError("query must use [1, heads, tokens, head_dim] layout")
    pool = pool_from_view(cache)
    if str(query.device) != str(runtime.device):
        raise CudaPagedAttentionError("query must be on the CUDA runtime device")
    for tensor in (cache.keys, cache.values, cache.key_scales, cache.value_scales, cache.block_table):
        if str(tensor.device) != str(runtime.device):
            raise CudaPagedAttentionError("packed cache must be on the CUDA runtime device")
    if isinstance(layer_index, bool) or not isinstance(layer_index, int) or not 0 <= layer_index < pool.num_layers:
        raise CudaPagedAttentionError("layer_index is outside the packed cache")
    query_heads, query_tokens, head_dim = query_shape[1:]
    if query_heads < 1 or query_tokens < 1 or query_tokens > cache.token_count:
        raise CudaPagedAttentionError("query token count is outside the packed cache")
    if head_dim != pool.head_dim or query_heads % pool.num_heads:
        raise CudaPagedAttentionError("query heads are incompatible with packed K/V")
    active_blocks = (cache.token_count + cache.block_size - 1) // cache.block_size
    if int(cache.block_table.numel()) != active_blocks:
        raise CudaPagedAttentionError("device block table does not cover cached tokens")
    if query.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise CudaPagedAttentionError("query dtype must be bfloat16, float16 or float32")

    from . import _lib as lib

    library = lib.load_library()
    state = getattr(runtime, "_paged_attention_state", None)
    if state is None:
        state = {"status": torch.zeros(1, dtype=torch.int32, device=runtime.device), "attention": {}}
        runtime._paged_attention_state = state

    def run() -> Any:
        table = cache.block_table
        if table.dtype != torch.int32:
            table = table.to(torch.int32)
        table = table.reshape(1, -1).contiguous()
        lens = cache.context_lens
        if lens is None or lens.dtype != torch.int32:
            lens = torch.full((1,), cache.token_count, dtype=torch.int32, device=runtime.device)
        key = (pool.keys, pool.key_scales, pool.num_blocks)
        attention = state["attention"].get(key)
        if attention is None:
            attention = PagedVerifyAttention(pool, runtime.device, library, state["status"])
            state["attention"][key] = attention
        return attention(query, table, lens, cache.token_count, layer_index)

    return runtime.submit_target(run, wait_for=wait_for, label="specdecode.target.paged_attention")


def attention_bytes(context_lens: Sequence[int], query_heads: int, kv_heads: int, head_dim: int, window: int,
                    block_size: int, query_bytes: int = 2) -> int:
    """Algorithmic HBM bytes of one verify-attention launch: every cached
    token's INT8 K and V codes plus their fp32 scales for each KV head, the
    query and output, and the block-table entries."""
    per_token = 2 * kv_heads * head_dim + 2 * kv_heads * 4
    tokens = int(sum(context_lens))
    batch = len(context_lens)
    q = batch * query_heads * window * head_dim * query_bytes
    tables = sum(math.ceil(t / block_size) for t in context_lens) * 4
    return tokens * per_token + 2 * q + tables
