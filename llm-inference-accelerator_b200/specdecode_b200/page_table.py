"""Host-side page-table bookkeeping for the device-resident paged cache.

This is the allocator and block-table state machine of the reference's
``PagedKVCache`` (src/specdecode/kv_cache.py:201-473), kept on the host
because allocation order is part of the contract: a new block is always the
lowest free block id (the min-heap of kv_cache.py:220-221, :327, :418).  The
free set is a boolean mask over heap ids, so "the k lowest free ids" is one
vectorised scan and a batched append over many sequences allocates in the
same order as the sequential per-sequence appends it replaces.

``block_order`` optionally relabels heap ids to physical block ids
(``physical = block_order[heap_id]``): the allocator keeps lowest-id-first
semantics while pages land at scattered physical addresses, which is how a
randomized free list is reproduced deterministically.

Nothing here touches the GPU; the device pool turns the plans returned by
``plan_append`` / ``plan_truncate`` into kernel launches.
"""

from __future__ import annotations

from collections.abc import Hashable, Sequence
from dataclasses import dataclass

import numpy as np


class KVCacheError(RuntimeError):
    """Base error for paged KV-cache operations."""


class KVCacheCapacityError(KVCacheError):
    """Raised when an append cannot be satisfied by the physical block pool."""


@dataclass
class AppendPlan:
    rows: np.ndarray          # int64 [B] table row of each sequence
    starts: np.ndarray        # int64 [B] length before the append
    counts: np.ndarray        # int64 [B] tokens appended per sequence
    slots: np.ndarray         # int64 [sum(counts)] physical slot per token, sequence-major
    new_heap_ids: np.ndarray  # int64 heap ids popped, in allocation order
    table_entries: np.ndarray  # int32 [E, 3] (row, logical block, physical block)
    new_lengths: np.ndarray   # int32 [B, 2] (row, length)


@dataclass
class TruncatePlan:
    rows: np.ndarray
    cleared_slots: np.ndarray  # int64 slots whose codes/scales are zeroed
    table_entries: np.ndarray  # int32 [E, 3] (row, logical block, -1)
    new_lengths: np.ndarray    # int32 [B, 2]
    released: np.ndarray       # int64 [B] blocks released per sequence


def _check_int(value, name: str) -> int:
    if isinstance(value, bool) or not isinstance(value, (int, np.integer)):
        raise TypeError(f"{name} must be an integer")
    return int(value)


class PageTable:
    """Sequences, block tables, lengths and the free-block set."""

    def __init__(self, num_blocks: int, block_size: int, *, block_order=None,
                 max_sequences: int = 64, max_blocks_per_sequence: int | None = None) -> None:
        self.num_blocks = int(num_blocks)
        self.block_size = int(block_size)
        if block_order is None:
            self.block_order = np.arange(self.num_blocks, dtype=np.int64)
        else:
            order = np.asarray(block_order, dtype=np.int64)
            if order.shape != (self.num_blocks,) or not np.array_equal(np.sort(order), np.arange(self.num_blocks)):
                raise ValueError("block_order must be a permutation of range(num_blocks)")
            self.block_order = order
        self.heap_id_of = np.empty(self.num_blocks, dtype=np.int64)
        self.heap_id_of[self.block_order] = np.arange(self.num_blocks, dtype=np.int64)
        self.max_blocks = int(max_blocks_per_sequence or self.num_blocks)
        self.free = np.ones(self.num_blocks, dtype=bool)           # indexed by heap id
        self.occupied = np.zeros((self.num_blocks, self.block_size), dtype=bool)  # by physical id
        self.tables = np.full((max(1, max_sequences), self.max_blocks), -1, dtype=np.int32)
        self.nblocks = np.zeros(max(1, max_sequences), dtype=np.int64)
        self.lengths = np.zeros(max(1, max_sequences), dtype=np.int64)
        self.row_free = np.ones(max(1, max_sequences), dtype=bool)
        self.rows: dict[Hashable, int] = {}

    # -- sequences ----------------------------------------------------------
    @property
    def capacity_rows(self) -> int:
        return self.tables.shape[0]

    def grow_rows(self, new_rows: int) -> None:
        old = self.tables.shape[0]
        if new_rows <= old:
            return
        self.tables = np.concatenate([self.tables, np.full((new_rows - old, self.max_blocks), -1, np.int32)])
        self.nblocks = np.concatenate([self.nblocks, np.zeros(new_rows - old, np.int64)])
        self.lengths = np.concatenate([self.lengths, np.zeros(new_rows - old, np.int64)])
        self.row_free = np.concatenate([self.row_free, np.ones(new_rows - old, bool)])

    def require(self, sequence_id: Hashable) -> int:
        try:
            row = self.rows.get(sequence_id)
        except TypeError as error:
            raise TypeError("sequence_id must be hashable") from error
        if row is None:
            raise KeyError(f"unknown sequence: {sequence_id!r}")
        return row

    def create_sequence(self, sequence_id: Hashable) -> int:
        try:
            if sequence_id in self.rows:
                raise ValueError(f"sequence already exists: {sequence_id!r}")
            hash(sequence_id)
        except TypeError as error:
            raise TypeError("sequence_id must be hashable") from error
        free_rows = np.flatnonzero(self.row_free)
        if free_rows.size == 0:
            self.grow_rows(2 * self.capacity_rows)
            free_rows = np.flatnonzero(self.row_free)
        row = int(free_rows[0])
        self.row_free[row] = False
        self.rows[sequence_id] = row
        self.tables[row] = -1
        self.nblocks[row] = 0
        self.lengths[row] = 0
        return row

    def drop_sequence(self, sequence_id: Hashable) -> int:
        row = self.require(sequence_id)
        if self.lengths[row] or self.nblocks[row]:
            raise AssertionError("sequence must be truncated to zero before it is dropped")
        del self.rows[sequence_id]
        self.row_free[row] = True
        return row

    def sequence_length(self, sequence_id: Hashable) -> int:
        return int(self.lengths[self.require(sequence_id)])

    def block_table(self, sequence_id: Hashable) -> tuple[int, ...]:
        row = self.require(sequence_id)
        return tuple(int(b) for b in self.tables[row, : self.nblocks[row]])

    def physical_slot(self, sequence_id: Hashable, token_index) -> tuple[int, int]:
        row = self.require(sequence_id)
        index = _check_int(token_index, "token_index")
        if not 0 <= index < self.lengths[row]:
            raise IndexError("token_index is outside the cached sequence")
        block, offset = divmod(index, self.block_size)
        return int(self.tables[row, block]), offset

    def slots_of(self, sequence_id: Hashable, start: int, stop: int) -> np.ndarray:
        row = self.require(sequence_id)
        t = np.arange(start, stop, dtype=np.int64)
        return self.tables[row, t // self.block_size].astype(np.int64) * self.block_size + t % self.block_size

    def free_blocks(self) -> int:
        return int(self.free.sum())

    # -- append ---------------------------------------------------------------
    def plan_append(self, sequence_ids: Sequence[Hashable], counts) -> AppendPlan:
        """Allocate blocks and slots for appending ``counts[i]`` tokens to
        ``sequence_ids[i]``, in order.  Raises before mutating anything when
        the pool cannot hold them (kv_cache.py:310-319)."""
        rows = np.array([self.require(s) for s in sequence_ids], dtype=np.int64)
        if len(set(rows.tolist())) != len(rows):
            raise ValueError("a sequence appears twice in one batched append")
        counts = np.asarray(counts, dtype=np.int64).reshape(-1)
        if counts.shape != rows.shape or (counts < 0).any():
            raise ValueError("counts must give one non-negative token count per sequence")
        bs = self.block_size
        starts = self.lengths[rows].copy()
        finals = starts + counts
        required = (finals + bs - 1) // bs
        additional = np.maximum(required - self.nblocks[rows], 0)
        total_new = int(additional.sum())
        if (required > self.max_blocks).any():
            raise KVCacheCapacityError("append exceeds the per-sequence block-table capacity")
        free_ids = np.flatnonzero(self.free)
        if total_new > free_ids.size:
            raise KVCacheCapacityError(
                f"append requires {total_new} new blocks but only {free_ids.size} are free")
        new_heap = free_ids[:total_new].astype(np.int64)
        new_phys = self.block_order[new_heap]
        # state mutation starts here
        self.free[new_heap] = False
        entries = np.empty((total_new, 3), dtype=np.int32)
        at = 0
        for i in np.flatnonzero(additional):
            row, n_new, first = int(rows[i]), int(additional[i]), int(self.nblocks[rows[i]])
            self.tables[row, first:first + n_new] = new_phys[at:at + n_new]
            entries[at:at + n_new, 0] = row
            entries[at:at + n_new, 1] = np.arange(first, first + n_new)
            entries[at:at + n_new, 2] = new_phys[at:at + n_new]
            self.nblocks[row] += n_new
            at += n_new
        total = int(counts.sum())
        seq_of = np.repeat(np.arange(rows.size), counts)
        t = starts[seq_of] + (np.arange(total) - np.repeat(np.cumsum(counts) - counts, counts))
        blocks = self.tables[rows[seq_of], t // bs].astype(np.int64)
        slots = blocks * bs + t % bs
        if self.occupied[blocks, t % bs].any():
            raise AssertionError("cache slot was unexpectedly occupied")
        self.occupied[blocks, t % bs] = True
        self.lengths[rows] = finals
        new_lengths = np.stack([rows, finals], axis=1).astype(np.int32)
        return AppendPlan(rows, starts, counts, slots, new_heap, entries, new_lengths)

    def undo_append(self, plan: AppendPlan) -> None:
        """Revert ``plan`` (used when the device rejected the appended data)."""
        bs = self.block_size
        blocks = plan.slots // bs
        self.occupied[blocks, plan.slots % bs] = False
        for row, logical, _ in plan.table_entries:
            self.tables[row, logical] = -1
        for i, row in enumerate(plan.rows):
            self.lengths[row] = plan.starts[i]
            self.nblocks[row] = (plan.starts[i] + bs - 1) // bs
        self.free[plan.new_heap_ids] = True

    # -- truncate -------------------------------------------------------------
    def plan_truncate(self, sequence_ids: Sequence[Hashable], token_counts) -> TruncatePlan:
        """Discard suffixes (kv_cache.py:395-420): clear slots ``[count, len)``,
        release blocks past ``ceil(count / block_size)``."""
        rows = np.array([self.require(s) for s in sequence_ids], dtype=np.int64)
        counts = []
        for value in token_counts:
            counts.append(_check_int(value, "token_count"))
        counts = np.asarray(counts, dtype=np.int64).reshape(-1)
        if counts.shape != rows.shape:
            raise ValueError("one token count per sequence is required")
        if len(set(rows.tolist())) != len(rows):
            raise ValueError("a sequence appears twice in one batched truncate")
        current = self.lengths[rows]
        if ((counts < 0) | (counts > current)).any():
            raise ValueError("token_count must be between zero and the sequence length")
        bs = self.block_size
        removed = current - counts
        total = int(removed.sum())
        seq_of = np.repeat(np.arange(rows.size), removed)
        t = counts[seq_of] + (np.arange(total) - np.repeat(np.cumsum(removed) - removed, removed))
        blocks = self.tables[rows[seq_of], t // bs].astype(np.int64)
        slots = blocks * bs + t % bs
        self.occupied[blocks, t % bs] = False
        kept = (counts + bs - 1) // bs
        released = self.nblocks[rows] - kept
        entries = []
        for i in np.flatnonzero(released):
            row = int(rows[i])
            ids = self.tables[row, kept[i]:self.nblocks[row]].astype(np.int64)
            if self.occupied[ids].any():
                raise AssertionError("released cache block still contains live entries")
            self.free[self.heap_id_of[ids]] = True
            for logical in range(int(kept[i]), int(self.nblocks[row])):
                entries.append((row, logical, -1))
            self.tables[row, kept[i]:self.nblocks[row]] = -1
            self.nblocks[row] = kept[i]
        self.lengths[rows] = counts
        table_entries = np.asarray(entries, dtype=np.int32).reshape(-1, 3)
        new_lengths = np.stack([rows, counts], axis=1).astype(np.int32)
        return TruncatePlan(rows, slots, table_entries, new_lengths, released.astype(np.int64))

    # -- audit ----------------------------------------------------------------
    def validate_invariants(self) -> None:
        """Raise ``AssertionError`` when allocator or table state is corrupt
        (kv_cache.py:449-473)."""
        live_rows = np.array(sorted(self.rows.values()), dtype=np.int64)
        allocated = [self.tables[r, : self.nblocks[r]].astype(np.int64) for r in live_rows]
        allocated = np.concatenate(allocated) if allocated else np.zeros(0, np.int64)
        if allocated.size != np.unique(allocated).size:
            raise AssertionError("a physical block is owned by multiple logical blocks")
        if (allocated < 0).any() or (allocated >= self.num_blocks).any():
            raise AssertionError("a block table holds an id outside the pool")
        allocated_heap = self.heap_id_of[allocated]
        if (self.free[allocated_heap]).any():
            raise AssertionError("a physical block is both allocated and free")
        if allocated.size + int(self.free.sum()) != self.num_blocks:
            raise AssertionError("physical block ownership is incomplete")
        bs = self.block_size
        for r in live_rows:
            length, n = int(self.lengths[r]), int(self.nblocks[r])
            if n != (length + bs - 1) // bs:
                raise AssertionError("logical block-table length is inconsistent")
            if (self.tables[r, n:] != -1).any():
                raise AssertionError("block table holds entries past its length")
            if n:
                occ = self.occupied[self.tables[r, :n].astype(np.int64)].reshape(-1)
                expected = np.arange(n * bs) < length
                if not np.array_equal(occ, expected):
                    raise AssertionError("physical block occupancy is inconsistent")
        free_phys = self.block_order[np.flatnonzero(self.free)]
        if self.occupied[free_phys].any():
            raise AssertionError("a free physical block contains cached entries")
