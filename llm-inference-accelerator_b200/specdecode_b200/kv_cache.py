"""Device-resident paged INT8 KV cache with the reference's PagedKVCache surface.

The public types and the ``PagedKVCache`` method surface follow
src/specdecode/kv_cache.py (KVCacheConfig 21-61, QuantizedVector 64-88,
KVQuantizer 91-99, PagedKVCache 201-473) so callers written against the
reference — the Hugging Face paged-cache mirror, the speculative decoder's
rollback calls — run unchanged.  What differs is where the data lives: codes
and scales are device tensors in HBM, quantization happens in the fused
quantize-and-append kernel, rollback zeroes slots with the rollback kernel,
and reads dequantize on the device.  Allocation and block tables stay on the
host (``page_table.PageTable``), with device copies of the tables kept in sync
by the same kernel launches.

Physical layout (per pool): codes ``[block][layer][head][offset][dim]`` int8
and scales ``[block][layer][head][offset]`` float32, so one (block, layer,
head) page is one contiguous run the attention kernel reads with a single
bulk copy.  ``keys_view`` etc. expose the reference's logical layout
``[block][offset][layer][head][dim]`` as a permuted view of the same memory.

Additive APIs beyond the reference: ``append_tensor`` (device tensors in,
no per-element Python), ``append_batch`` / ``truncate_batch`` (many sequences
in one launch), ``attention_inputs`` (device tables for batched attention).
"""

from __future__ import annotations

import math
import struct
from collections.abc import Hashable, Sequence
from dataclasses import dataclass
from typing import Protocol, runtime_checkable

import numpy as np

from . import _lib
from .page_table import AppendPlan, KVCacheCapacityError, KVCacheError, PageTable, TruncatePlan  # noqa: F401

__all__ = [
    "KVCacheError", "KVCacheCapacityError", "KVCacheConfig", "QuantizedVector", "KVQuantizer",
    "QuantizedKVToken", "DequantizedKVToken", "KVCacheCheckpoint", "KVCacheStats", "PagedKVCache",
    "CudaUnavailableError",
]


class CudaUnavailableError(RuntimeError):
    """Raised when the device cache is created without a usable CUDA device."""


@dataclass(frozen=True, slots=True)
class KVCacheConfig:
    """Physical cache shape and block-pool capacity."""

    num_layers: int
    num_heads: int
    head_dim: int
    block_size: int = 16
    num_blocks: int = 256

    def __post_init__(self) -> None:
        for name in ("num_layers", "num_heads", "head_dim", "block_size", "num_blocks"):
            value = getattr(self, name)
            if isinstance(value, bool) or not isinstance(value, int) or value < 1:
                raise ValueError(f"{name} must be a positive integer")

    @property
    def capacity_tokens(self) -> int:
        return self.block_size * self.num_blocks

    @property
    def fp32_bytes_per_token(self) -> int:
        return 2 * self.num_layers * self.num_heads * self.head_dim * 4

    @property
    def quantized_bytes_per_token(self) -> int:
        return 2 * self.num_layers * self.num_heads * self.head_dim + 2 * self.num_layers * self.num_heads * 4

    @property
    def theoretical_savings_ratio(self) -> float:
        return 1.0 - self.quantized_bytes_per_token / self.fp32_bytes_per_token


def _exact_float32(value: float) -> bool:
    try:
        return struct.unpack("=f", struct.pack("=f", value))[0] == value
    except OverflowError:
        return False


@dataclass(frozen=True, slots=True)
class QuantizedVector:
    """One symmetric INT8 vector and its float32-representable scale."""

    values: tuple[int, ...]
    scale: float

    def __post_init__(self) -> None:
        if not self.values:
            raise ValueError("a quantized vector cannot be empty")
        if not math.isfinite(self.scale) or self.scale < 0.0:
            raise ValueError("quantization scale must be finite and non-negative")
        if not _exact_float32(self.scale):
            raise ValueError("quantization scale must be exactly representable as float32")
        for value in self.values:
            if isinstance(value, bool) or not isinstance(value, int):
                raise TypeError("quantized values must be integers")
            if not -127 <= value <= 127:
                raise ValueError("quantized values must be inside [-127, 127]")
        if self.scale == 0.0 and any(self.values):
            raise ValueError("a zero quantization scale requires all-zero values")


@runtime_checkable
class KVQuantizer(Protocol):
    """Quantization operations a cache can be configured with."""

    name: str

    def quantize(self, values: Sequence[float]) -> QuantizedVector: ...

    def dequantize(self, vector: QuantizedVector) -> tuple[float, ...]: ...


@dataclass(frozen=True, slots=True)
class QuantizedKVToken:
    keys: tuple[tuple[QuantizedVector, ...], ...]
    values: tuple[tuple[QuantizedVector, ...], ...]


@dataclass(frozen=True, slots=True)
class DequantizedKVToken:
    keys: tuple[tuple[tuple[float, ...], ...], ...]
    values: tuple[tuple[tuple[float, ...], ...], ...]


@dataclass(frozen=True, slots=True)
class KVCacheCheckpoint:
    sequence_id: Hashable
    token_count: int


@dataclass(frozen=True, slots=True)
class KVCacheStats:
    sequences: int
    used_tokens: int
    capacity_tokens: int
    allocated_blocks: int
    free_blocks: int
    used_quantized_bytes: int
    allocated_quantized_bytes: int
    capacity_quantized_bytes: int
    fp32_equivalent_bytes: int
    block_table_bytes: int
    theoretical_savings_ratio: float


# Quantizers whose rule is the reference's per-head symmetric INT8 rule; the
# device pool applies that rule in its fused kernel.
_REFERENCE_RULE_QUANTIZERS = frozenset({"python", "native", "cuda"})


def _torch():
    import torch

    return torch


_DTYPE_CODES = None


def _dtype_code(dtype) -> int:
    global _DTYPE_CODES
    torch = _torch()
    if _DTYPE_CODES is None:
        _DTYPE_CODES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16,
                        torch.float16: _lib.DTYPE_F16, torch.float64: _lib.DTYPE_F64}
    try:
        return _DTYPE_CODES[dtype]
    except KeyError as error:
        raise TypeError(f"unsupported KV dtype {dtype}") from error


class _MetadataRing:
    """Pinned host staging + device buffers for per-call metadata (slots,
    table edits, lengths), uploaded with one asynchronous copy.

    ``upload`` fills the next ring slot, enqueues its copy and returns a
    ticket; after launching the kernel that reads it, the caller passes the
    ticket to ``release``, which records an event behind that kernel.  A slot
    is refilled only after its event has completed, so neither its pinned host
    bytes nor its device bytes are overwritten while a copy or kernel may still
    read them."""

    def __init__(self, device, depth: int = 4, initial_bytes: int = 1 << 16) -> None:
        torch = _torch()
        self.device = device
        self.depth = depth
        self.host = [torch.empty(initial_bytes, dtype=torch.uint8, pin_memory=True) for _ in range(depth)]
        self.dev = [torch.empty(initial_bytes, dtype=torch.uint8, device=device) for _ in range(depth)]
        self.events = [None] * depth
        self.busy = [False] * depth
        self.at = 0

    def upload(self, parts: Sequence[np.ndarray], stream) -> tuple[list[int], int]:
        torch = _torch()
        sizes = [int(p.nbytes) for p in parts]
        offsets, total = [], 0
        for size in sizes:
            offsets.append(total)
            total += (size + 15) // 16 * 16
        total = max(total, 16)
        slot = self.at
        self.at = (self.at + 1) % self.depth
        if self.busy[slot]:
            raise RuntimeError("metadata ring overrun: a prepared operation was never committed")
        if self.events[slot] is not None:
            self.events[slot].synchronize()
            self.events[slot] = None
        if self.host[slot].numel() < total:
            capacity = 1 << (total - 1).bit_length()
            self.host[slot] = torch.empty(capacity, dtype=torch.uint8, pin_memory=True)
            self.dev[slot] = torch.empty(capacity, dtype=torch.uint8, device=self.device)
        host = self.host[slot].numpy()
        for part, off, size in zip(parts, offsets, sizes):
            if size:
                host[off:off + size] = np.ascontiguousarray(part).view(np.uint8).reshape(-1)
        with torch.cuda.stream(stream):
            self.dev[slot][:total].copy_(self.host[slot][:total], non_blocking=True)
        self.busy[slot] = True
        base = self.dev[slot].data_ptr()
        return [base + off for off in offsets], slot

    def device_view(self, ticket: int, address: int, count: int, dtype):
        """``count`` elements of ``dtype`` at ``address`` inside ticket's
        device buffer (valid until the ticket is released)."""
        torch = _torch()
        buf = self.dev[ticket]
        start = address - buf.data_ptr()
        nbytes = count * torch.empty((), dtype=dtype).element_size()
        return buf[start:start + nbytes].view(dtype)

    def release(self, ticket: int, stream) -> None:
        torch = _torch()
        event = torch.cuda.Event()
        event.record(stream)
        self.events[ticket] = event
        self.busy[ticket] = False


@dataclass
class PendingAppend:
    """A planned append whose metadata is already on its way to the device;
    ``PagedKVCache.commit_append`` launches it."""

    plan: AppendPlan
    keys: object
    values: object
    layer_begin: int
    layers: int
    pointers: list
    ticket: int
    stream: object


@dataclass
class LayerwiseAppend:
    """Slots reserved for new tokens of every layer (``PagedKVCache.reserve``),
    filled one layer at a time by ``PagedKVCache.write_layer``."""

    plan: AppendPlan
    slots: object  # device int64 [tokens], sequence-major
    tokens: int


@dataclass
class PendingTruncate:
    plan: TruncatePlan
    pointers: list | None
    ticket: int
    stream: object
    sequence_ids: list
    counts: list


class PagedKVCache:
    """Fixed-pool paged INT8 cache resident in device memory.

    Same semantics as the reference's PagedKVCache: lowest-free-id block
    allocation, atomic appends (no partial state after a failure), rollback
    that clears discarded slots and releases whole blocks, byte accounting.
    Not thread-safe; callers serialise, as with the reference.
    """

    def __init__(self, config: KVCacheConfig, *, quantizer: KVQuantizer | None = None, device=None,
                 block_order=None, max_sequences: int = 64, max_blocks_per_sequence: int | None = None,
                 check_status: bool = True, library_path=None) -> None:
        torch = _torch()
        if not isinstance(config, KVCacheConfig):
            raise TypeError("config must be a KVCacheConfig")
        if not torch.cuda.is_available():
            raise CudaUnavailableError("the paged INT8 cache needs a CUDA device; none is available")
        if quantizer is not None:
            name = getattr(quantizer, "name", None)
            if name not in _REFERENCE_RULE_QUANTIZERS:
                raise TypeError(
                    "the device cache quantizes with the reference per-head symmetric INT8 rule; "
                    f"quantizer {name!r} is not one of {sorted(_REFERENCE_RULE_QUANTIZERS)}")
        self.config = config
        self.quantizer = quantizer
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.check_status_after_each_call = check_status
        self._lib = _lib.load_library(library_path)
        L, H, D, bs, nb = config.num_layers, config.num_heads, config.head_dim, config.block_size, config.num_blocks
        if D % 16 or D > 512:
            raise ValueError("head_dim must be a multiple of 16 and at most 512 for the device pool")
        self._pages = PageTable(nb, bs, block_order=block_order, max_sequences=max_sequences,
                                max_blocks_per_sequence=max_blocks_per_sequence)
        self.key_codes = torch.zeros((nb, L, H, bs, D), dtype=torch.int8, device=self.device)
        self.value_codes = torch.zeros_like(self.key_codes)
        self.key_scale_pages = torch.zeros((nb, L, H, bs), dtype=torch.float32, device=self.device)
        self.value_scale_pages = torch.zeros_like(self.key_scale_pages)
        self.block_tables = torch.full(self._pages.tables.shape, -1, dtype=torch.int32, device=self.device)
        self.context_lens = torch.zeros(self._pages.tables.shape[0], dtype=torch.int32, device=self.device)
        self._status = torch.zeros(1, dtype=torch.int32, device=self.device)
        # deep enough that a decoding loop planning several steps ahead of the
        # device rarely waits for a ring slot
        self._meta = _MetadataRing(self.device, depth=16)
        self.pool_desc = _lib.PagePool(
            self.key_codes.data_ptr(), self.value_codes.data_ptr(), self.key_scale_pages.data_ptr(),
            self.value_scale_pages.data_ptr(), nb, bs, L, H, D,
            L * H * bs * D, H * bs * D, bs * D, L * H * bs, H * bs, bs)
        self._low_water: dict[Hashable, int] = {}

    # -- views ----------------------------------------------------------------
    @property
    def keys_view(self):
        """Codes in the reference's ``[block, offset, layer, head, dim]`` layout."""
        return self.key_codes.permute(0, 3, 1, 2, 4)

    @property
    def values_view(self):
        return self.value_codes.permute(0, 3, 1, 2, 4)

    @property
    def key_scales_view(self):
        return self.key_scale_pages.permute(0, 3, 1, 2)

    @property
    def value_scales_view(self):
        return self.value_scale_pages.permute(0, 3, 1, 2)

    @property
    def library(self) -> _lib.CudaLibrary:
        return self._lib

    # -- device status ----------------------------------------------------------
    def _stream(self):
        return _torch().cuda.current_stream(self.device)

    def status_bits(self, *, reset: bool = True) -> int:
        """Synchronise and return (then clear) the device fault bits."""
        bits = int(self._status.item())
        if bits and reset:
            self._status.zero_()
        return bits

    def check_status(self) -> None:
        bits = self.status_bits()
        if bits:
            raise _lib.NativeBackendError(f"device fault: {_lib.fault_message(bits)}",
                                          status=_lib.STATUS_DEVICE_FAULT, faults=bits)

    def _ensure_table_rows(self) -> None:
        torch = _torch()
        rows = self._pages.capacity_rows
        if self.block_tables.shape[0] < rows:
            grown = torch.full((rows, self.block_tables.shape[1]), -1, dtype=torch.int32, device=self.device)
            grown[: self.block_tables.shape[0]].copy_(self.block_tables)
            lens = torch.zeros(rows, dtype=torch.int32, device=self.device)
            lens[: self.context_lens.shape[0]].copy_(self.context_lens)
            self.block_tables, self.context_lens = grown, lens

    def _edits(self, entries_ptr: int, n_entries: int, lengths_ptr: int, n_lengths: int) -> _lib.TableEdits:
        return _lib.TableEdits(self.block_tables.data_ptr(), self.block_tables.shape[1],
                               self.block_tables.shape[0], self.context_lens.data_ptr(),
                               entries_ptr, n_entries, lengths_ptr, n_lengths)

    # -- sequences --------------------------------------------------------------
    def create_sequence(self, sequence_id: Hashable) -> None:
        self._pages.create_sequence(sequence_id)
        self._ensure_table_rows()
        self._low_water[sequence_id] = 0

    def sequence_length(self, sequence_id: Hashable) -> int:
        return self._pages.sequence_length(sequence_id)

    def block_table(self, sequence_id: Hashable) -> tuple[int, ...]:
        return self._pages.block_table(sequence_id)

    def physical_slot(self, sequence_id: Hashable, token_index: int) -> tuple[int, int]:
        return self._pages.physical_slot(sequence_id, token_index)

    def table_row(self, sequence_id: Hashable) -> int:
        """Row of ``block_tables`` / ``context_lens`` holding this sequence."""
        return self._pages.require(sequence_id)

    # -- append -----------------------------------------------------------------
    def _as_kv_tensor(self, tensor, label: str, layers: int):
        torch = _torch()
        if not isinstance(tensor, torch.Tensor):
            raise TypeError(f"{label} must be a tensor")
        if tensor.dtype == torch.bool or not tensor.is_floating_point():
            raise TypeError("KV values must be real numbers, not booleans or integers")
        _dtype_code(tensor.dtype)
        shape = (layers, self.config.num_heads, self.config.head_dim)
        if tensor.dim() != 4 or tuple(tensor.shape[1:]) != shape:
            raise ValueError(f"{label} must have shape [tokens, {layers}, num_heads, head_dim]")
        if tensor.device != self.device:
            tensor = tensor.to(self.device, non_blocking=True)
        es = tensor.element_size()
        if (tensor.stride(3) != 1 or tensor.data_ptr() % 16 or any((tensor.stride(i) * es) % 16 for i in range(3))):
            tensor = tensor.contiguous()
        return tensor

    def _prepare_append(self, sequence_ids, keys, values, counts, layer_begin: int, layers: int) -> PendingAppend:
        plan = self._pages.plan_append(sequence_ids, counts)
        try:
            stream = self._stream()
            pointers, ticket = self._meta.upload([plan.slots, plan.table_entries, plan.new_lengths], stream)
        except Exception:
            self._pages.undo_append(plan)
            raise
        return PendingAppend(plan, keys, values, layer_begin, layers, pointers, ticket, stream)

    def commit_append(self, pending: PendingAppend) -> list[tuple[int, ...]]:
        """Launch a prepared append; returns the token indices per sequence."""
        plan, keys, values = pending.plan, pending.keys, pending.values
        slots_ptr, entries_ptr, lengths_ptr = pending.pointers
        edits = self._edits(entries_ptr, len(plan.table_entries), lengths_ptr, len(plan.new_lengths))
        n = int(plan.slots.size)
        try:
            status = self._lib.handle.sdc_quantize_append(
                self.pool_desc, pending.layer_begin, pending.layers, keys.data_ptr() if n else None,
                values.data_ptr() if n else None, _dtype_code(keys.dtype), n,
                keys.stride(0), keys.stride(1), keys.stride(2), slots_ptr, edits,
                self._status.data_ptr(), pending.stream.cuda_stream)
        finally:
            self._meta.release(pending.ticket, pending.stream)
        if status != _lib.STATUS_OK:
            self._pages.undo_append(plan)
            self._lib.check(status, "quantize-append")
        if self.check_status_after_each_call:
            bits = self.status_bits()
            if bits:
                self._undo_append(plan)
                self.status_bits()
                if bits & _lib.FAULT_NONFINITE_VALUE:
                    raise ValueError("KV values must be finite")
                if bits & _lib.FAULT_INVALID_SCALE:
                    raise ValueError("quantization scale is outside the float32 range")
                raise _lib.NativeBackendError(f"device fault: {_lib.fault_message(bits)}",
                                              status=_lib.STATUS_DEVICE_FAULT, faults=bits)
        return [tuple(range(int(s), int(s) + int(c))) for s, c in zip(plan.starts, plan.counts)]

    def _undo_append(self, plan: AppendPlan) -> None:
        """Zero the slots an append wrote and rewind the device tables."""
        stream = self._stream()
        rewind_entries = plan.table_entries.copy()
        rewind_entries[:, 2] = -1
        old_lengths = np.stack([plan.rows, plan.starts], axis=1).astype(np.int32)
        (slots_ptr, entries_ptr, lengths_ptr), ticket = self._meta.upload(
            [plan.slots, rewind_entries, old_lengths], stream)
        edits = self._edits(entries_ptr, len(rewind_entries), lengths_ptr, len(old_lengths))
        try:
            status = self._lib.handle.sdc_rollback(
                self.pool_desc, slots_ptr, int(plan.slots.size), edits, self._status.data_ptr(),
                stream.cuda_stream)
        finally:
            self._meta.release(ticket, stream)
        self._lib.check(status, "rollback")
        self._pages.undo_append(plan)

    def reserve(self, sequence_ids: Sequence[Hashable], count: int) -> LayerwiseAppend:
        """Allocate pages for ``count`` new tokens of every listed sequence and
        extend their device block tables and lengths without writing codes.
        ``write_layer`` then quantizes each layer's keys / values into the
        reserved slots, which is how a model whose layers run one after
        another (an attention hook) appends; a layer's attention over the new
        tokens is valid once that layer has been written.  Capacity is checked
        first: a failed reservation changes nothing."""
        torch = _torch()
        ids = list(sequence_ids)
        count = int(count)
        if count < 1:
            raise ValueError("reserve at least one token")
        plan = self._pages.plan_append(ids, [count] * len(ids))
        stream = self._stream()
        try:
            (slots_ptr, entries_ptr, lengths_ptr), ticket = self._meta.upload(
                [np.ascontiguousarray(plan.slots, dtype=np.int64), plan.table_entries, plan.new_lengths], stream)
            # the reservation keeps its own copy of the slots (a device-to-device
            # copy on the stream: no host synchronisation)
            with torch.cuda.stream(stream):
                slots = self._meta.device_view(ticket, slots_ptr, int(plan.slots.size), torch.int64).clone()
        except Exception:
            self._pages.undo_append(plan)
            raise
        edits = self._edits(entries_ptr, len(plan.table_entries), lengths_ptr, len(plan.new_lengths))
        try:
            status = self._lib.handle.sdc_quantize_append(
                self.pool_desc, 0, self.config.num_layers, None, None, _dtype_code(torch.float32), 0, 0, 0, 0,
                None, edits, self._status.data_ptr(), stream.cuda_stream)
        finally:
            self._meta.release(ticket, stream)
        if status != _lib.STATUS_OK:
            self._pages.undo_append(plan)
            self._lib.check(status, "slot reservation")
        return LayerwiseAppend(plan, slots, int(plan.slots.size))

    def write_layer(self, pending: LayerwiseAppend, layer: int, keys, values) -> None:
        """Quantize layer ``layer``'s keys / values ``[tokens, num_heads,
        head_dim]`` (tokens in reservation order: all of the first sequence's,
        then the next sequence's) into the slots of a reservation."""
        if not 0 <= int(layer) < self.config.num_layers:
            raise ValueError(f"layer {layer} outside the cache's {self.config.num_layers} layers")
        n = pending.tokens
        H, D = self.config.num_heads, self.config.head_dim
        if tuple(keys.shape) != (n, H, D) or tuple(values.shape) != (n, H, D):
            raise ValueError(f"keys/values must have shape [{n}, {H}, {D}]")
        k = self._as_kv_tensor(keys.reshape(n, 1, H, D), "keys", 1)
        v = self._as_kv_tensor(values.reshape(n, 1, H, D), "values", 1)
        if v.dtype != k.dtype:
            v = v.to(k.dtype)
        status = self._lib.handle.sdc_quantize_append(
            self.pool_desc, int(layer), 1, k.data_ptr(), v.data_ptr(), _dtype_code(k.dtype), n,
            k.stride(0), k.stride(1), k.stride(2), pending.slots.data_ptr(), None, self._status.data_ptr(),
            self._stream().cuda_stream)
        self._lib.check(status, "layer write")

    def append_tensor(self, sequence_id: Hashable, keys, values) -> tuple[int, ...]:
        """Atomically quantize and append ``keys``/``values`` of shape
        ``[tokens, num_layers, num_heads, head_dim]`` (float32/bf16/fp16/fp64,
        any device)."""
        self._pages.require(sequence_id)
        L = self.config.num_layers
        keys = self._as_kv_tensor(keys, "keys", L)
        values = self._as_kv_tensor(values, "values", L)
        if keys.shape[0] != values.shape[0]:
            raise ValueError("keys and values must hold the same number of tokens")
        if values.dtype != keys.dtype:
            values = values.to(keys.dtype)
        n = int(keys.shape[0])
        if n == 0:
            return ()
        return self.commit_append(self._prepare_append([sequence_id], keys, values, [n], 0, L))[0]

    def prepare_append_batch(self, sequence_ids: Sequence[Hashable], keys, values) -> PendingAppend:
        """Validate and plan an append of ``keys``/``values``
        ``[batch, tokens, layers, heads, dim]`` — the same number of tokens to
        every listed sequence — and stage its metadata; ``commit_append``
        launches it.  Allocation state changes here; a prepared append must be
        committed before the next one is prepared."""
        if keys.dim() != 5 or values.shape != keys.shape:
            raise ValueError("keys/values must have shape [batch, tokens, layers, heads, dim]")
        B, n = int(keys.shape[0]), int(keys.shape[1])
        if B != len(sequence_ids):
            raise ValueError("one key/value block per sequence is required")
        L = self.config.num_layers
        flat_k = self._as_kv_tensor(keys.reshape(B * n, *keys.shape[2:]), "keys", L)
        flat_v = self._as_kv_tensor(values.reshape(B * n, *values.shape[2:]), "values", L)
        if flat_v.dtype != flat_k.dtype:
            flat_v = flat_v.to(flat_k.dtype)
        return self._prepare_append(list(sequence_ids), flat_k, flat_v, [n] * B, 0, L)

    def append_batch(self, sequence_ids: Sequence[Hashable], keys, values) -> list[tuple[int, ...]]:
        """Append to many sequences in one launch (see ``prepare_append_batch``)."""
        return self.commit_append(self.prepare_append_batch(sequence_ids, keys, values))

    def append(self, sequence_id: Hashable, keys, values) -> int:
        return self.append_many(sequence_id, ((keys, values),))[0]

    def append_many(self, sequence_id: Hashable, entries) -> tuple[int, ...]:
        """Reference-compatible append of nested ``[layer][head][dim]`` entries
        (kv_cache.py:298-336).  Python floats are quantized from float64."""
        self._pages.require(sequence_id)
        pending = tuple(entries)
        if not pending:
            return ()
        keys = self._nested_to_tensor([k for k, _ in pending], "key")
        values = self._nested_to_tensor([v for _, v in pending], "value")
        return self.append_tensor(sequence_id, keys, values)

    def _nested_to_tensor(self, tensors, label: str):
        torch = _torch()
        L, H, D = self.config.num_layers, self.config.num_heads, self.config.head_dim
        flat: list[float] = []
        for tensor in tensors:
            if isinstance(tensor, torch.Tensor):
                if tuple(tensor.shape) != (L, H, D):
                    raise ValueError(f"{label} must contain one [num_heads, head_dim] tensor per layer")
                flat.extend(float(v) for v in tensor.detach().double().cpu().reshape(-1).tolist())
                continue
            if len(tensor) != L:
                raise ValueError(f"{label} must contain one tensor per model layer")
            for layer in tensor:
                if len(layer) != H:
                    raise ValueError(f"each {label} layer must contain num_heads vectors")
                for head in layer:
                    if len(head) != D:
                        raise ValueError(f"each {label} head must contain head_dim values")
                    for value in head:
                        if isinstance(value, bool):
                            raise TypeError("KV values must be real numbers, not booleans")
                        try:
                            converted = float(value)
                        except (TypeError, ValueError) as error:
                            raise TypeError("KV values must be real numbers") from error
                        if not math.isfinite(converted):
                            raise ValueError("KV values must be finite")
                        flat.append(converted)
        host = torch.tensor(flat, dtype=torch.float64).reshape(len(tensors), L, H, D)
        return host.pin_memory().to(self.device, non_blocking=True)

    # -- rollback ---------------------------------------------------------------
    def prepare_truncate_batch(self, sequence_ids: Sequence[Hashable], token_counts) -> PendingTruncate:
        """Plan a rollback of several sequences and stage its metadata;
        ``commit_truncate`` launches it."""
        sequence_ids, counts = list(sequence_ids), list(token_counts)
        plan = self._pages.plan_truncate(sequence_ids, counts)
        stream = self._stream()
        if plan.cleared_slots.size == 0 and plan.table_entries.size == 0:
            return PendingTruncate(plan, None, -1, stream, sequence_ids, counts)
        pointers, ticket = self._meta.upload([plan.cleared_slots, plan.table_entries, plan.new_lengths], stream)
        return PendingTruncate(plan, pointers, ticket, stream, sequence_ids, counts)

    def commit_truncate(self, pending: PendingTruncate) -> list[int]:
        plan = pending.plan
        if pending.pointers is not None:  # otherwise nothing was discarded
            slots_ptr, entries_ptr, lengths_ptr = pending.pointers
            edits = self._edits(entries_ptr, len(plan.table_entries), lengths_ptr, len(plan.new_lengths))
            try:
                status = self._lib.handle.sdc_rollback(
                    self.pool_desc, slots_ptr, int(plan.cleared_slots.size), edits, self._status.data_ptr(),
                    pending.stream.cuda_stream)
            finally:
                self._meta.release(pending.ticket, pending.stream)
            self._lib.check(status, "rollback")
        for seq, count in zip(pending.sequence_ids, pending.counts):
            self._low_water[seq] = min(self._low_water.get(seq, int(count)), int(count))
        return [int(r) for r in plan.released]

    def truncate(self, sequence_id: Hashable, token_count: int) -> int:
        """Discard a suffix; returns the number of physical blocks released
        (kv_cache.py:395-420)."""
        return self.commit_truncate(self.prepare_truncate_batch([sequence_id], [token_count]))[0]

    def truncate_batch(self, sequence_ids: Sequence[Hashable], token_counts) -> list[int]:
        return self.commit_truncate(self.prepare_truncate_batch(sequence_ids, token_counts))

    def checkpoint(self, sequence_id: Hashable) -> KVCacheCheckpoint:
        return KVCacheCheckpoint(sequence_id, self.sequence_length(sequence_id))

    def rollback(self, sequence_id: Hashable, checkpoint: KVCacheCheckpoint) -> int:
        if checkpoint.sequence_id != sequence_id:
            raise ValueError("checkpoint belongs to a different sequence")
        return self.truncate(sequence_id, checkpoint.token_count)

    def remove_sequence(self, sequence_id: Hashable) -> int:
        released = self.truncate(sequence_id, 0)
        self._pages.drop_sequence(sequence_id)
        self._low_water.pop(sequence_id, None)
        return released

    # -- reads --------------------------------------------------------------------
    def _gather(self, slots: np.ndarray, dtype, layer_begin: int = 0, layers: int | None = None):
        """Dequantize the listed slots on the device: ``(keys, values)`` of
        shape ``[n, layers, heads, dim]`` in ``dtype``."""
        torch = _torch()
        layers = self.config.num_layers if layers is None else layers
        n = int(slots.size)
        shape = (n, layers, self.config.num_heads, self.config.head_dim)
        out_k = torch.empty(shape, dtype=dtype, device=self.device)
        out_v = torch.empty(shape, dtype=dtype, device=self.device)
        if n == 0:
            return out_k, out_v
        stream = self._stream()
        (slots_ptr,), ticket = self._meta.upload([slots.astype(np.int64)], stream)
        try:
            status = self._lib.handle.sdc_gather_dequantize(
                self.pool_desc, layer_begin, layers, slots_ptr, n, out_k.data_ptr(), out_v.data_ptr(),
                _dtype_code(dtype), out_k.stride(0), out_k.stride(1), out_k.stride(2),
                self._status.data_ptr(), stream.cuda_stream)
        finally:
            self._meta.release(ticket, stream)
        self._lib.check(status, "gather-dequantize")
        return out_k, out_v

    def read_quantized_token(self, sequence_id: Hashable, token_index: int) -> QuantizedKVToken:
        block, offset = self.physical_slot(sequence_id, token_index)
        k = self.key_codes[block, :, :, offset].cpu().tolist()
        v = self.value_codes[block, :, :, offset].cpu().tolist()
        ks = self.key_scale_pages[block, :, :, offset].cpu().tolist()
        vs = self.value_scale_pages[block, :, :, offset].cpu().tolist()

        def build(codes, scales):
            return tuple(tuple(QuantizedVector(tuple(int(c) for c in codes[l][h]), float(scales[l][h]))
                               for h in range(len(codes[l]))) for l in range(len(codes)))

        return QuantizedKVToken(keys=build(k, ks), values=build(v, vs))

    def read_token(self, sequence_id: Hashable, token_index: int) -> DequantizedKVToken:
        block, offset = self.physical_slot(sequence_id, token_index)
        return self._dequantized_tokens(np.array([block * self.config.block_size + offset]))[0]

    def read_sequence(self, sequence_id: Hashable) -> tuple[DequantizedKVToken, ...]:
        length = self.sequence_length(sequence_id)
        if length == 0:
            return ()
        return self._dequantized_tokens(self._pages.slots_of(sequence_id, 0, length))

    def _dequantized_tokens(self, slots: np.ndarray) -> tuple[DequantizedKVToken, ...]:
        torch = _torch()
        k, v = self._gather(slots, torch.float64)
        k, v = k.cpu().tolist(), v.cpu().tolist()

        def nest(t):
            return tuple(tuple(tuple(head) for head in layer) for layer in t)

        return tuple(DequantizedKVToken(keys=nest(k[i]), values=nest(v[i])) for i in range(len(k)))

    def gather_slots(self, slots, dtype, *, layer_begin: int = 0, layers: int | None = None, out=None):
        """Dequantize the physical slots held in the device int64 tensor
        ``slots`` (``block * block_size + offset`` per token, as
        ``physical_slot`` gives): ``(keys, values)`` ``[n, layers, heads,
        dim]`` in ``dtype``, written into ``out`` when given.  No host copy:
        the slot list is already on the device (for example built from the
        block tables by the caller)."""
        torch = _torch()
        layers = self.config.num_layers if layers is None else layers
        if not isinstance(slots, torch.Tensor) or slots.dtype != torch.int64 or slots.dim() != 1:
            raise TypeError("slots must be a 1-D int64 tensor")
        if slots.device != torch.device(self.device):
            raise ValueError("slots must be on the cache's device")
        n = int(slots.numel())
        shape = (n, layers, self.config.num_heads, self.config.head_dim)
        if out is None:
            out = (torch.empty(shape, dtype=dtype, device=self.device),
                   torch.empty(shape, dtype=dtype, device=self.device))
        out_k, out_v = out
        if out_k.shape != shape or out_v.shape != shape or out_k.dtype != dtype or out_v.dtype != dtype:
            raise ValueError("output tensors must be [n, layers, heads, dim] in the requested dtype")
        if out_k.stride() != out_v.stride() or out_k.stride(3) != 1:
            raise ValueError("output tensors must share strides with contiguous head vectors")
        if n == 0:
            return out_k, out_v
        slots = slots.contiguous()
        stream = self._stream()
        self._lib.check(self._lib.handle.sdc_gather_dequantize(
            self.pool_desc, layer_begin, layers, slots.data_ptr(), n, out_k.data_ptr(), out_v.data_ptr(),
            _dtype_code(dtype), out_k.stride(0), out_k.stride(1), out_k.stride(2),
            self._status.data_ptr(), stream.cuda_stream), "gather-dequantize")
        return out_k, out_v

    def gather_sequence(self, sequence_id: Hashable, dtype, *, layer_begin: int = 0, layers: int | None = None):
        """Device tensors ``[T, layers, heads, dim]`` of dequantized K and V."""
        length = self.sequence_length(sequence_id)
        return self._gather(self._pages.slots_of(sequence_id, 0, length), dtype, layer_begin, layers)

    # -- attention inputs -------------------------------------------------------------
    def attention_inputs(self, sequence_ids: Sequence[Hashable]):
        """``(block_tables int32 [B, stride], context_lens int32 [B], max_len)``
        on the device for the listed sequences (a view when rows are
        consecutive)."""
        torch = _torch()
        rows = [self._pages.require(s) for s in sequence_ids]
        max_len = max((int(self._pages.lengths[r]) for r in rows), default=0)
        first = rows[0] if rows else 0
        if rows == list(range(first, first + len(rows))):
            return self.block_tables[first:first + len(rows)], self.context_lens[first:first + len(rows)], max_len
        index = torch.tensor(rows, dtype=torch.long, device=self.device)
        return self.block_tables.index_select(0, index), self.context_lens.index_select(0, index), max_len

    def changes_since(self, sequence_id: Hashable, old_length: int) -> int:
        """Length of the prefix unchanged since a reader saw ``old_length``
        tokens (used for incremental-sync accounting)."""
        stable = min(old_length, self._low_water.get(sequence_id, old_length))
        self._low_water[sequence_id] = self.sequence_length(sequence_id)
        return stable

    # -- accounting -----------------------------------------------------------------
    def stats(self) -> KVCacheStats:
        cfg = self.config
        rows = list(self._pages.rows.values())
        used = int(self._pages.lengths[rows].sum()) if rows else 0
        allocated = int(self._pages.nblocks[rows].sum()) if rows else 0
        per_token = cfg.quantized_bytes_per_token
        return KVCacheStats(
            sequences=len(rows), used_tokens=used, capacity_tokens=cfg.capacity_tokens,
            allocated_blocks=allocated, free_blocks=self._pages.free_blocks(),
            used_quantized_bytes=used * per_token,
            allocated_quantized_bytes=allocated * cfg.block_size * per_token,
            capacity_quantized_bytes=cfg.capacity_tokens * per_token,
            fp32_equivalent_bytes=used * cfg.fp32_bytes_per_token, block_table_bytes=allocated * 4,
            theoretical_savings_ratio=cfg.theoretical_savings_ratio)

    def validate_invariants(self) -> None:
        self._pages.validate_invariants()

    @property
    def page_table(self) -> PageTable:
        return self._pages

    def device_memory_bytes(self) -> int:
        tensors = (self.key_codes, self.value_codes, self.key_scale_pages, self.value_scale_pages)
        return sum(t.numel() * t.element_size() for t in tensors)

    def __repr__(self) -> str:  # pragma: no cover - debugging aid
        c = self.config
        return (f"PagedKVCache(L={c.num_layers}, H={c.num_heads}, D={c.head_dim}, bs={c.block_size}, "
                f"nb={c.num_blocks}, device={self.device})")
