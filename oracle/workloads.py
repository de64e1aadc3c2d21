"""ORACLE — seeded synthetic workloads with the benchmark configurations' shapes.

Test infrastructure only.  There is no public dataset for this path; every
input is drawn from ``numpy.random.default_rng(seed)`` so that the script that
runs the reference (tests/golden/make_golden.py) and the GPU tests see
bit-identical inputs on any machine.

``speculative_events`` is the CPU-runnable reference workload: sequences are
prefilled, then each speculative round appends a window of tokens to every
sequence and keeps the prefix accepted by per-token Bernoulli(p) draws up to
the first rejection, rolling the rest back.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class SpeculativeShape:
    num_layers: int = 16
    num_heads: int = 8
    head_dim: int = 64
    block_size: int = 16
    num_blocks: int = 4096
    sequences: int = 4
    prefill: int = 512
    rounds: int = 64
    window: int = 5
    accept_p: float = 0.7


FULL_SPECULATIVE = SpeculativeShape()
SMALL_SPECULATIVE = SpeculativeShape(num_layers=2, num_heads=2, head_dim=16, block_size=4,
                                     num_blocks=96, sequences=3, prefill=13, rounds=12,
                                     window=5, accept_p=0.7)


def speculative_events(shape: SpeculativeShape, seed: int):
    """Yield ``("append", seq, keys, values)`` with float32 ``[n, L, H, D]``
    arrays and ``("truncate", seq, token_count)``."""
    rng = np.random.default_rng(seed)
    dims = (shape.num_layers, shape.num_heads, shape.head_dim)
    lengths = {s: 0 for s in range(shape.sequences)}
    for s in range(shape.sequences):
        k = rng.standard_normal((shape.prefill, *dims), dtype=np.float32)
        v = rng.standard_normal((shape.prefill, *dims), dtype=np.float32)
        lengths[s] += shape.prefill
        yield ("append", s, k, v)
    for _ in range(shape.rounds):
        for s in range(shape.sequences):
            start = lengths[s]
            k = rng.standard_normal((shape.window, *dims), dtype=np.float32)
            v = rng.standard_normal((shape.window, *dims), dtype=np.float32)
            yield ("append", s, k, v)
            accepted = 0
            while accepted < shape.window and rng.random() < shape.accept_p:
                accepted += 1
            lengths[s] = start + accepted
            yield ("truncate", s, start + accepted)


def state_digest(tables: dict, lengths: dict, keys, values, key_scales, value_scales) -> str:
    """sha256 over block tables, lengths and the full logical-layout storage
    (codes ``[nb, bs, L, H, D]`` int8, scales ``[nb, bs, L, H]`` float32 bit
    patterns; released slots must hold zeros)."""
    h = hashlib.sha256()
    for seq in sorted(tables):
        h.update(np.asarray(tables[seq], dtype=np.int64).tobytes())
        h.update(np.int64(lengths[seq]).tobytes())
    h.update(np.ascontiguousarray(keys, dtype=np.int8).tobytes())
    h.update(np.ascontiguousarray(values, dtype=np.int8).tobytes())
    h.update(np.ascontiguousarray(key_scales, dtype=np.float32).view(np.uint32).tobytes())
    h.update(np.ascontiguousarray(value_scales, dtype=np.float32).view(np.uint32).tobytes())
    return h.hexdigest()


@dataclass(frozen=True)
class VerifyShape:
    batch: int = 32
    query_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    window: int = 5
    block_size: int = 16
    min_context: int = 1024
    max_context: int = 8192


VERIFY_8B = VerifyShape()
VERIFY_70B = VerifyShape(batch=8, query_heads=64, kv_heads=8, head_dim=128, window=5,
                         block_size=16, min_context=131072, max_context=131072)


def verify_inputs(shape: VerifyShape, seed: int):
    """Context lengths, per-sequence block tables over a randomly permuted
    pool, and query values (float32 draws, to be rounded to bf16).

    Returns ``(context_lens int64 [B], tables list[np.ndarray int64],
    num_blocks, query float32 [B, Hq, kw, D])``.
    """
    rng = np.random.default_rng(seed)
    lens = rng.integers(shape.min_context, shape.max_context + 1, size=shape.batch)
    blocks_per_seq = (lens + shape.block_size - 1) // shape.block_size
    num_blocks = int(blocks_per_seq.sum())
    perm = rng.permutation(num_blocks)
    tables, at = [], 0
    for n in blocks_per_seq:
        tables.append(perm[at:at + n].astype(np.int64))
        at += n
    query = rng.standard_normal((shape.batch, shape.query_heads, shape.window, shape.head_dim),
                                dtype=np.float32)
    return lens.astype(np.int64), tables, num_blocks, query
