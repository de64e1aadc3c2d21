"""ORACLE — the paged INT8 cache state machine restated on the CPU.

Test infrastructure only.  Follows src/specdecode/kv_cache.py:201-473
(PagedKVCache) for allocation, append, truncate and accounting, and the
device-storage rule of src/specdecode/cuda_kv_cache.py:333-354 that released
slots hold zero codes and zero scales.

Storage uses the reference's kernel-facing logical layout
(src/specdecode/cuda_kv_cache.py:21-37): codes ``[block, offset, layer, head,
dim]`` int8 and scales ``[block, offset, layer, head]`` float32.

``block_order`` is an optional relabelling of physical block ids: the
allocator still pops the lowest free *heap id* (kv_cache.py:220-221, :327,
:418) and stores ``block_order[heap_id]`` in the block table.  With the
identity order this is exactly the reference allocator; a seeded permutation
gives the "randomized free list" of the append benchmark while staying
deterministic on both sides.
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass

import numpy as np

from .quant import CQuantizer, quantize_rows


class OracleCapacityError(RuntimeError):
    pass


@dataclass
class OracleStats:
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


class PagedCacheOracle:
    def __init__(self, num_layers, num_heads, head_dim, block_size, num_blocks,
                 *, block_order=None, use_c=True) -> None:
        self.L, self.H, self.D = num_layers, num_heads, head_dim
        self.bs, self.nb = block_size, num_blocks
        self.keys = np.zeros((num_blocks, block_size, num_layers, num_heads, head_dim), np.int8)
        self.values = np.zeros_like(self.keys)
        self.key_scales = np.zeros((num_blocks, block_size, num_layers, num_heads), np.float32)
        self.value_scales = np.zeros_like(self.key_scales)
        self.occupied = np.zeros((num_blocks, block_size), bool)
        self._heap = list(range(num_blocks))
        heapq.heapify(self._heap)
        self.block_order = (np.arange(num_blocks, dtype=np.int64) if block_order is None
                            else np.asarray(block_order, dtype=np.int64))
        self._heap_id_of = {int(p): h for h, p in enumerate(self.block_order)}
        self.tables: dict = {}
        self.lengths: dict = {}
        self._c = CQuantizer() if use_c else None

    # -- kv_cache.py:233-259 -------------------------------------------------
    def create_sequence(self, seq) -> None:
        if seq in self.lengths:
            raise ValueError(f"sequence already exists: {seq!r}")
        self.tables[seq] = []
        self.lengths[seq] = 0

    def sequence_length(self, seq) -> int:
        return self.lengths[seq]

    def block_table(self, seq) -> tuple[int, ...]:
        return tuple(self.tables[seq])

    def physical_slot(self, seq, index) -> tuple[int, int]:
        if not 0 <= index < self.lengths[seq]:
            raise IndexError("token_index is outside the cached sequence")
        block, offset = divmod(index, self.bs)
        return self.tables[seq][block], offset

    def _quantize(self, x):
        if self._c is not None:
            return self._c.quantize_rows(x)
        return quantize_rows(x)

    # -- kv_cache.py:298-336 -------------------------------------------------
    def append_many(self, seq, keys: np.ndarray, values: np.ndarray) -> tuple[int, ...]:
        """keys/values: ``[n, L, H, D]`` real arrays (any float dtype)."""
        n = int(keys.shape[0])
        if n == 0:
            return ()
        start = self.lengths[seq]
        table = self.tables[seq]
        final = start + n
        required = (final + self.bs - 1) // self.bs
        additional = required - len(table)
        if additional > len(self._heap):
            raise OracleCapacityError(
                f"append requires {additional} new blocks but only {len(self._heap)} are free")
        kq, ks, kst = self._quantize(keys)
        vq, vs, vst = self._quantize(values)
        if (kst != 0).any() or (vst != 0).any():
            raise ValueError("non-finite KV values or invalid scale")
        for _ in range(additional):
            table.append(int(self.block_order[heapq.heappop(self._heap)]))
        for i in range(n):
            t = start + i
            block, offset = table[t // self.bs], t % self.bs
            assert not self.occupied[block, offset]
            self.keys[block, offset] = kq[i]
            self.values[block, offset] = vq[i]
            self.key_scales[block, offset] = ks[i]
            self.value_scales[block, offset] = vs[i]
            self.occupied[block, offset] = True
        self.lengths[seq] = final
        return tuple(range(start, final))

    # -- kv_cache.py:395-427 + cuda_kv_cache.py:336-342 -----------------------
    def truncate(self, seq, count: int) -> int:
        current = self.lengths[seq]
        if not 0 <= count <= current:
            raise ValueError("token_count must be between zero and the sequence length")
        if count == current:
            return 0
        table = self.tables[seq]
        for t in range(count, current):
            block, offset = table[t // self.bs], t % self.bs
            self.keys[block, offset] = 0
            self.values[block, offset] = 0
            self.key_scales[block, offset] = 0
            self.value_scales[block, offset] = 0
            self.occupied[block, offset] = False
        kept = (count + self.bs - 1) // self.bs
        released = table[kept:]
        del table[kept:]
        for block in released:
            assert not self.occupied[block].any()
            heapq.heappush(self._heap, self._heap_id_of[block])
        self.lengths[seq] = count
        return len(released)

    def remove_sequence(self, seq) -> int:
        released = self.truncate(seq, 0)
        del self.tables[seq]
        del self.lengths[seq]
        return released

    def free_blocks(self) -> int:
        return len(self._heap)

    # -- kv_cache.py:43-61, 429-447 -------------------------------------------
    def stats(self) -> OracleStats:
        fp32_per_token = 2 * self.L * self.H * self.D * 4
        q_per_token = 2 * self.L * self.H * self.D + 2 * self.L * self.H * 4
        used = sum(self.lengths.values())
        allocated = sum(len(t) for t in self.tables.values())
        return OracleStats(
            sequences=len(self.lengths), used_tokens=used,
            capacity_tokens=self.bs * self.nb, allocated_blocks=allocated,
            free_blocks=len(self._heap), used_quantized_bytes=used * q_per_token,
            allocated_quantized_bytes=allocated * self.bs * q_per_token,
            capacity_quantized_bytes=self.bs * self.nb * q_per_token,
            fp32_equivalent_bytes=used * fp32_per_token, block_table_bytes=allocated * 4,
            theoretical_savings_ratio=1.0 - q_per_token / fp32_per_token)

    # -- read path ------------------------------------------------------------
    def gather(self, seq, layer: int):
        """Codes/scales of one layer for every cached token of ``seq``:
        ``(k [T, H, D] int8, v, ks [T, H] f32, vs)``."""
        T = self.lengths[seq]
        idx = np.arange(T)
        blocks = np.asarray(self.tables[seq], dtype=np.int64)[idx // self.bs] if T else np.zeros(0, np.int64)
        offs = idx % self.bs
        return (self.keys[blocks, offs, layer], self.values[blocks, offs, layer],
                self.key_scales[blocks, offs, layer], self.value_scales[blocks, offs, layer])
