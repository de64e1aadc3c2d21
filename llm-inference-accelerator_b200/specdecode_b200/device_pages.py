"""A paged INT8 cache whose block tables, lengths and free set live on the
device (csrc/page_alloc.cu).

``PagedKVCache`` plans every append and rollback on the host (its
``PageTable`` mirrors the reference's allocator, src/specdecode/kv_cache.py:
220-427) and ships the table edits to the kernels.  ``DevicePagedCache``
keeps that state on the device instead, so a decoding loop appends, rolls
back and forks sequences with kernel launches only -- no host planning and
no host-to-device table copies:

* ``reserve`` / ``append``: new blocks are the lowest free heap ids, taken in
  row order, so the tables equal the reference allocator's for the same
  operations (``block_order`` relabels heap ids to physical blocks, as in
  ``PagedKVCache``); ``append`` then quantizes into the reserved slots with
  kernel (a);
* ``truncate`` / ``release``: blocks past the new length return to the free
  set with their pages zeroed, and the removed rows of an unshared, partly
  kept last page are zeroed, as the reference's rollback leaves released
  slots;
* ``fork``: prefix sharing, which the reference defers
  (docs/kv-cache.md:105-108): an empty row takes another row's blocks and
  length, each block reference-counted, and the first append into a shared,
  partly filled last block copies it first (copy-on-write).

The host keeps only an upper bound of every row's length (for grid sizes and
the attention's ``max_context_len``).  Faults (a pool short of blocks, a row
or length out of range) are bits in a device status word that
``check_status`` reads; a faulted call changes nothing on the device.
"""

from __future__ import annotations

import ctypes
from collections.abc import Sequence

import numpy as np

from . import _lib
from .kv_cache import CudaUnavailableError, KVCacheCapacityError, KVCacheConfig, KVCacheError, _dtype_code


def _torch():
    import torch

    return torch


class _Staging:
    """Pinned host rows for the small per-call arrays (rows, counts,
    lengths), copied to the device asynchronously.  A pageable copy would
    wait for the stream to drain; a ring of pinned slots lets the host queue
    many calls ahead.  A slot is reused only after its copy has run."""

    def __init__(self, device, width: int, depth: int = 64) -> None:
        torch = _torch()
        self.host = torch.empty((depth, 2, width), dtype=torch.int32, pin_memory=True)
        self.dev = torch.empty((depth, 2, width), dtype=torch.int32, device=device)
        self.events = [None] * depth
        self.next = 0
        self.device = device

    def put(self, first: Sequence[int], second: Sequence[int] | None = None):
        torch = _torch()
        k = self.next
        self.next = (k + 1) % len(self.events)
        if self.events[k] is not None:
            self.events[k].synchronize()
        n = len(first)
        view = self.host[k].numpy()
        view[0, :n] = first
        if second is not None:
            view[1, :n] = second
        self.dev[k, :, :n].copy_(self.host[k, :, :n], non_blocking=True)
        event = torch.cuda.Event()
        event.record(torch.cuda.current_stream(self.device))
        self.events[k] = event
        return self.dev[k, 0, :n], self.dev[k, 1, :n]


class DevicePagedCache:
    """Device pool plus device-resident allocator state for ``max_rows`` rows."""

    def __init__(self, config: KVCacheConfig, *, max_rows: int = 64, max_blocks_per_row: int | None = None,
                 block_order=None, device=None, library_path=None) -> None:
        torch = _torch()
        if not torch.cuda.is_available():
            raise CudaUnavailableError("the device page allocator needs a CUDA device; none is available")
        self.config = config
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self._lib = _lib.load_library(library_path)
        L, H, D, bs, nb = config.num_layers, config.num_heads, config.head_dim, config.block_size, config.num_blocks
        if D % 16 or D > 512:
            raise ValueError("head_dim must be a multiple of 16 and at most 512 for the device pool")
        if max_rows < 1:
            raise ValueError("max_rows must be positive")
        stride = int(max_blocks_per_row) if max_blocks_per_row is not None else nb
        if stride < 1:
            raise ValueError("max_blocks_per_row must be positive")
        order = np.arange(nb, dtype=np.int64) if block_order is None else np.asarray(block_order, dtype=np.int64)
        if order.shape != (nb,) or not np.array_equal(np.sort(order), np.arange(nb)):
            raise ValueError("block_order must be a permutation of the block ids")
        heap_of = np.empty(nb, dtype=np.int64)
        heap_of[order] = np.arange(nb)
        words = np.zeros((nb + 31) // 32, dtype=np.uint32)
        full, rest = divmod(nb, 32)
        words[:full] = 0xFFFFFFFF
        if rest:
            words[full] = (1 << rest) - 1
        dev = self.device
        self.key_codes = torch.zeros((nb, L, H, bs, D), dtype=torch.int8, device=dev)
        self.value_codes = torch.zeros_like(self.key_codes)
        self.key_scale_pages = torch.zeros((nb, L, H, bs), dtype=torch.float32, device=dev)
        self.value_scale_pages = torch.zeros_like(self.key_scale_pages)
        self.free_bits = torch.from_numpy(words.view(np.int32)).to(dev)
        self.refcount = torch.zeros(nb, dtype=torch.int32, device=dev)
        self.high_water = torch.zeros(nb, dtype=torch.int32, device=dev)
        self.block_order = torch.from_numpy(order.astype(np.int32)).to(dev)
        self.heap_of = torch.from_numpy(heap_of.astype(np.int32)).to(dev)
        self.block_tables = torch.full((max_rows, stride), -1, dtype=torch.int32, device=dev)
        self.context_lens = torch.zeros(max_rows, dtype=torch.int32, device=dev)
        self._status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.pool_desc = _lib.PagePool(
            self.key_codes.data_ptr(), self.value_codes.data_ptr(), self.key_scale_pages.data_ptr(),
            self.value_scale_pages.data_ptr(), nb, bs, L, H, D,
            L * H * bs * D, H * bs * D, bs * D, L * H * bs, H * bs, bs)
        self.allocator_desc = _lib.PageAllocator(
            self.free_bits.data_ptr(), self.refcount.data_ptr(), self.high_water.data_ptr(),
            self.block_order.data_ptr(),
            self.heap_of.data_ptr(), self.block_tables.data_ptr(), self.context_lens.data_ptr(), nb, bs,
            max_rows, stride)
        self.length_bound = np.zeros(max_rows, dtype=np.int64)
        self._workspace = torch.empty(0, dtype=torch.uint8, device=dev)
        self._staging = _Staging(dev, max(max_rows, 1))

    @property
    def library(self) -> _lib.CudaLibrary:
        return self._lib

    @property
    def max_rows(self) -> int:
        return int(self.block_tables.shape[0])

    @property
    def status(self):
        """The device fault word (int32 [1]) every call of this cache ORs into."""
        return self._status

    def attention(self):
        """Kernel (c) over this pool: ``attention(query, block_tables,
        context_lens, max_context_len, layer)`` with rows of this cache's
        tables and lengths."""
        from .cuda_kv_cache import PagedVerifyAttention

        return PagedVerifyAttention(self.pool_desc, self.device, self._lib, self._status)

    def _stream(self) -> int:
        return _torch().cuda.current_stream(self.device).cuda_stream

    def _rows(self, rows: Sequence[int], *, distinct: bool = True) -> list[int]:
        rows = [int(r) for r in rows]
        if not rows:
            raise ValueError("at least one row is required")
        if distinct and len(set(rows)) != len(rows):
            raise ValueError("rows must be distinct")
        if min(rows) < 0 or max(rows) >= self.max_rows:
            raise IndexError("row outside the table")
        return rows

    # -- status -----------------------------------------------------------------
    def status_bits(self, *, reset: bool = True) -> int:
        bits = int(self._status.item())
        if bits and reset:
            self._status.zero_()
        return bits

    def check_status(self) -> None:
        """Raises if any call since the last check faulted; the faulted calls
        changed nothing, and the host's length bounds are re-read."""
        bits = self.status_bits()
        if not bits:
            return
        self.length_bound = self.context_lens.cpu().numpy().astype(np.int64)
        message = _lib.fault_message(bits)
        if bits & _lib.FAULT_CAPACITY:
            raise KVCacheCapacityError(message)
        raise KVCacheError(f"device page allocator fault: {message}")

    # -- operations ---------------------------------------------------------------
    def reserve(self, rows: Sequence[int], counts: Sequence[int]):
        """Room for counts[i] more tokens in each of ``rows``; returns the
        slots of the new tokens (device int64, row order then token order)."""
        torch = _torch()
        rows = self._rows(rows)
        counts = [int(c) for c in counts]
        if len(counts) != len(rows) or min(counts) < 0:
            raise ValueError("one non-negative count per row is required")
        if len(rows) > 1024:
            raise ValueError("at most 1024 rows per call")
        total = sum(counts)
        size = ctypes.c_size_t()
        self._lib.check(self._lib.handle.sdc_pages_append_workspace_size(len(rows), total, self.config.block_size,
                                                                         ctypes.byref(size)), "page workspace")
        if self._workspace.numel() < size.value:
            self._workspace = torch.empty(max(size.value, 1 << 16), dtype=torch.uint8, device=self.device)
        slots = torch.empty(total, dtype=torch.int64, device=self.device)
        rows_t, counts_t = self._staging.put(rows, counts)
        self._lib.check(self._lib.handle.sdc_pages_append(
            self.allocator_desc, self.pool_desc, rows_t.data_ptr(), counts_t.data_ptr(), len(rows), total,
            slots.data_ptr() if total else None, self._workspace.data_ptr(), self._workspace.numel(),
            self._status.data_ptr(), self._stream()), "page reservation")
        for r, c in zip(rows, counts):
            self.length_bound[r] += c
        return slots

    def append(self, rows: Sequence[int], keys, values):
        """Quantizes ``keys`` / ``values`` ``[len(rows), n, layers, heads,
        head_dim]`` (float32/bf16/f16/f64) into n new slots of every row."""
        c = self.config
        if keys.dim() != 5 or tuple(keys.shape[2:]) != (c.num_layers, c.num_heads, c.head_dim) \
                or keys.shape[0] != len(rows) or values.shape != keys.shape:
            raise ValueError("keys/values must be [rows, tokens, num_layers, num_heads, head_dim]")
        n = int(keys.shape[1])
        slots = self.reserve(rows, [n] * len(rows))
        if n == 0:
            return slots
        k = keys.to(self.device).reshape(len(rows) * n, c.num_layers, c.num_heads, c.head_dim).contiguous()
        v = values.to(self.device, dtype=k.dtype).reshape(k.shape).contiguous()
        self._lib.check(self._lib.handle.sdc_quantize_append(
            self.pool_desc, 0, c.num_layers, k.data_ptr(), v.data_ptr(), _dtype_code(k.dtype), k.shape[0],
            k.stride(0), k.stride(1), k.stride(2), slots.data_ptr(), None, self._status.data_ptr(),
            self._stream()), "quantize-append")
        return slots

    def truncate(self, rows: Sequence[int], new_lengths: Sequence[int]) -> None:
        """Rolls ``rows`` back to ``new_lengths`` tokens."""
        rows = self._rows(rows)
        lengths = [int(n) for n in new_lengths]
        if len(lengths) != len(rows) or min(lengths) < 0:
            raise ValueError("one non-negative length per row is required")
        removed = max(max(int(self.length_bound[r]) - n, 0) for r, n in zip(rows, lengths))
        rows_t, lengths_t = self._staging.put(rows, lengths)
        self._lib.check(self._lib.handle.sdc_pages_truncate(
            self.allocator_desc, self.pool_desc, rows_t.data_ptr(), lengths_t.data_ptr(), len(rows), removed,
            self._status.data_ptr(), self._stream()), "page truncation")
        for r, n in zip(rows, lengths):
            if n <= self.length_bound[r]:  # a longer length faults on the device and changes nothing
                self.length_bound[r] = n

    def release(self, rows: Sequence[int]) -> None:
        """Empties ``rows`` (their blocks return to the free set once no other
        row shares them)."""
        self.truncate(rows, [0] * len(list(rows)))

    def fork(self, sources: Sequence[int], destinations: Sequence[int]) -> None:
        """Each (empty) destination row shares its source row's blocks; a
        source may be forked more than once."""
        src = self._rows(sources, distinct=False)
        dst = self._rows(destinations)
        if len(src) != len(dst) or set(src) & set(dst):
            raise ValueError("sources and destinations must pair up and be different rows")
        src_t, dst_t = self._staging.put(src, dst)
        self._lib.check(self._lib.handle.sdc_pages_fork(
            self.allocator_desc, src_t.data_ptr(), dst_t.data_ptr(), len(src), self._status.data_ptr(),
            self._stream()), "page fork")
        for s, d in zip(src, dst):
            self.length_bound[d] = self.length_bound[s]

    # -- inspection ---------------------------------------------------------------
    def snapshot(self) -> dict:
        """Host copies of the allocator state (synchronises)."""
        words = self.free_bits.cpu().numpy().view(np.uint32)
        nb = self.config.num_blocks
        heap_free = ((words[np.arange(nb) // 32] >> (np.arange(nb) % 32)) & 1).astype(bool)
        return {
            "tables": self.block_tables.cpu().numpy(),
            "lengths": self.context_lens.cpu().numpy(),
            "refcount": self.refcount.cpu().numpy(),
            "free": heap_free,  # indexed by heap id
            "heap_of": self.heap_of.cpu().numpy(),
        }

    def validate_invariants(self) -> None:
        """Every block is free exactly when no table entry references it, and
        its reference count equals the entries that do."""
        snap = self.snapshot()
        bs = self.config.block_size
        counts = np.zeros(self.config.num_blocks, dtype=np.int64)
        for row, length in enumerate(snap["lengths"]):
            used = -(-int(length) // bs)
            entries = snap["tables"][row, :used]
            if (entries < 0).any() or (snap["tables"][row, used:] != -1).any():
                raise AssertionError(f"row {row}: table entries disagree with its length")
            np.add.at(counts, entries, 1)
        if not np.array_equal(counts, snap["refcount"]):
            raise AssertionError("reference counts differ from the table entries")
        free_phys = np.zeros(self.config.num_blocks, dtype=bool)
        free_phys[self.block_order.cpu().numpy()[snap["free"]]] = True
        if not np.array_equal(free_phys, counts == 0):
            raise AssertionError("the free set differs from the unreferenced blocks")

