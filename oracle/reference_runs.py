"""ORACLE — the reference's own CPU path, run and timed.  Test infrastructure only.

The CPU baseline of the benchmark is the reference's code itself, unchanged:
its Python package (``src/specdecode``) copied into ``oracle/_ref/specdecode/``
and its C++ quantizer library compiled from ``native/src/native.cpp`` into
``oracle/_ref/libspecdecode_native.so``, both by ``make -C oracle ref``.
Nothing here imports the product package or loads its CUDA library, so a
process that runs only this module (``bench.py --impl reference``) executes
the reference's code and the oracle's C / numpy restatements, nothing else.
Only ``bench.py``'s CPU-baseline legs and ``tests/`` call this module.

Legs, each on a bounded sample of the benchmark's workloads:

* ``time_submit_paged_attention`` — the reference's unfused paged attention
  (``src/specdecode/cuda_kv_cache.py:370-503``: gather pages, dequantize in
  the query dtype, expand GQA heads, boolean causal mask, SDPA) on CPU torch
  through a runtime shim that runs the submitted closure inline, one sequence
  per call (its API is batch 1), all host threads.
* ``time_reconstruct_attention`` — the reference's CPU reconstruct path:
  ``HuggingFacePagedCacheMirror.materialize_legacy_cache``
  (``src/specdecode/hf_paged_cache.py:247-313``: ``read_sequence``
  dequantizes every head vector through ``sd_dequantize_symmetric_int8_f64``
  and rebuilds ``[1, heads, T, head_dim]`` tensors from Python lists), then
  the GQA expansion and CPU SDPA a Hugging Face attention layer runs on the
  rebuilt cache.  The mirror is filled first through its ``synchronize``
  (``hf_paged_cache.py:204-232``: ``.tolist()`` per token and layer, then
  ``PagedKVCache.append_many`` with ``NativeKVQuantizer``), timed apart.
* ``time_append_rollback`` — ``PagedKVCache.append_many`` and ``truncate``
  (``src/specdecode/kv_cache.py:290-336``, ``:395-420``) with
  ``NativeKVQuantizer`` over the reference's library: the speculative
  append / rollback step of a workload, for a subsample of its sequences and
  steps.
"""

from __future__ import annotations

import math
import os
import sys
import time
from pathlib import Path

import numpy as np

REF_DIR = Path(__file__).resolve().parent / "_ref"
NATIVE_LIBRARY = REF_DIR / "libspecdecode_native.so"


class ReferenceUnavailable(RuntimeError):
    """The reference's package or library is not in oracle/_ref/."""


def reference_package():
    """The reference's ``specdecode`` package, imported from oracle/_ref/."""
    if not (REF_DIR / "specdecode" / "__init__.py").is_file() or not NATIVE_LIBRARY.is_file():
        raise ReferenceUnavailable("oracle/_ref/ lacks the reference's package or library; run `make -C oracle ref`")
    path = str(REF_DIR)
    if path not in sys.path:
        sys.path.insert(0, path)
    import specdecode

    where = Path(specdecode.__file__).resolve()
    if REF_DIR not in where.parents:
        raise ReferenceUnavailable(f"a different specdecode package was imported: {where}")
    return specdecode


def native_quantizer():
    """The reference's ``NativeKVQuantizer`` over its own compiled library."""
    reference_package()
    from specdecode.native import NativeKVQuantizer

    return NativeKVQuantizer.load(str(NATIVE_LIBRARY))


class CpuRuntime:
    """The part of the reference's ``CudaExecutionRuntime`` that
    ``submit_paged_attention`` uses (``device``, ``torch_module``,
    ``submit_target``), on the CPU: the closure runs inline."""

    def __init__(self) -> None:
        import torch

        self.device = torch.device("cpu")
        self.torch_module = torch

    def submit_target(self, operation, *, wait_for=(), label=""):
        class _Done:
            pass

        task = _Done()
        task.result = operation()
        return task


def bf16_values(x: np.ndarray) -> np.ndarray:
    """float32 array rounded to the nearest bfloat16 values (still float32)."""
    import torch

    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def verify_pool(num_blocks: int, kv_heads: int, head_dim: int, block_size: int, seed: int, layers: int = 1):
    """An INT8 page pool in the reference's kernel-facing layout: codes
    ``[block, offset, layer, head, dim]`` and fp32 scales ``[block, offset,
    layer, head]`` (``cuda_kv_cache.py:21-37``), quantized from N(0,1)
    bf16-valued keys and values by the reference rule.  Quantization goes
    through the oracle's C restatement, which the tests hold bit-exact to the
    reference's quantizers."""
    from oracle.quant import CQuantizer

    import torch

    quantizer = CQuantizer()
    gen = torch.Generator().manual_seed(seed)
    shape = (num_blocks, block_size, layers, kv_heads, head_dim)
    out = {}
    for name in ("keys", "values"):
        codes = np.empty(shape, np.int8)
        scales = np.empty(shape[:-1], np.float32)
        step = 1024
        for b0 in range(0, num_blocks, step):
            b1 = min(num_blocks, b0 + step)
            x = torch.randn((b1 - b0,) + shape[1:], generator=gen).to(torch.bfloat16).float().numpy()
            c, s, status = quantizer.quantize_rows(x)
            if status.any():
                raise RuntimeError("the pool's synthetic values failed to quantize")
            codes[b0:b1] = c
            scales[b0:b1] = s
        out[name] = codes
        out[name[:-1] + "_scales"] = scales
    return out


def host_threads() -> int:
    """Use every host core for torch's CPU ops; returns the thread count."""
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    return torch.get_num_threads()


def time_submit_paged_attention(pool, lens, table, query, block_size: int, budget_s: float, *, layer: int = 0,
                                min_passes: int = 1):
    """Run the reference's ``submit_paged_attention`` once per sequence over
    whole passes of the batch until ``budget_s`` of timed work (at least
    ``min_passes`` passes).  ``query`` is float32 ``[B, Hq, window, D]``; it
    is cast to bf16 as the benchmark's query.  Returns (the timed sequence
    indices in call order, the seconds of each call, the last output of
    every sequence)."""
    import torch

    reference_package()
    from specdecode.cuda_kv_cache import CudaPagedKVCacheView, submit_paged_attention

    host_threads()
    runtime = CpuRuntime()
    tensors = {k: torch.from_numpy(v) for k, v in pool.items()}
    q = torch.from_numpy(np.ascontiguousarray(query, dtype=np.float32)).to(torch.bfloat16)
    views = []
    for b, T in enumerate(lens):
        T = int(T)
        nblk = (T + block_size - 1) // block_size
        views.append(CudaPagedKVCacheView(
            keys=tensors["keys"], values=tensors["values"], key_scales=tensors["key_scales"],
            value_scales=tensors["value_scales"], block_table=torch.from_numpy(table[b, :nblk].astype(np.int64)),
            token_count=T, block_size=block_size))
    order, seconds, passes = [], [], 0
    outputs = [None] * len(views)
    while passes < min_passes or sum(seconds) < budget_s:
        for b, view in enumerate(views):
            t0 = time.perf_counter()
            outputs[b] = submit_paged_attention(runtime, q[b:b + 1], view, layer).result
            seconds.append(time.perf_counter() - t0)
            order.append(b)
            # after the required whole passes, stop as soon as the budget is spent
            if passes >= min_passes and sum(seconds) >= budget_s:
                break
        passes += 1
    return order, seconds, outputs


def time_reconstruct_attention(lens, query, kv_heads: int, head_dim: int, block_size: int, budget_s: float,
                               seed: int):
    """The reference's CPU reconstruct path for as many of the batch's
    sequences as fit in ``budget_s`` of timed work (at least one).  Per
    sequence: a mirror over a ``PagedKVCache`` with the reference's
    ``NativeKVQuantizer`` is filled by ``synchronize`` from N(0,1) bf16 keys
    and values (timed apart), then ``materialize_legacy_cache`` plus GQA
    expansion, causal mask and CPU SDPA in bf16 are timed.  Returns a dict of
    the timed seconds, sequences, cached tokens and the synchronize time."""
    import torch

    reference_package()
    from specdecode.hf_paged_cache import HuggingFacePagedCacheMirror
    from specdecode.kv_cache import KVCacheConfig, PagedKVCache

    threads = host_threads()
    native = native_quantizer()
    rng = np.random.default_rng(seed)
    elapsed, sync_s, sequences, tokens = 0.0, 0.0, 0, 0
    for b, T in enumerate(lens):
        T = int(T)
        nblk = (T + block_size - 1) // block_size
        mirror = HuggingFacePagedCacheMirror(PagedKVCache(
            KVCacheConfig(1, kv_heads, head_dim, block_size=block_size, num_blocks=nblk), quantizer=native))
        k = torch.from_numpy(rng.standard_normal((1, kv_heads, T, head_dim), dtype=np.float32)).to(torch.bfloat16)
        v = torch.from_numpy(rng.standard_normal((1, kv_heads, T, head_dim), dtype=np.float32)).to(torch.bfloat16)
        legacy = ((k, v),)
        t0 = time.perf_counter()
        mirror.synchronize(legacy)
        sync_s += time.perf_counter() - t0
        q = torch.from_numpy(np.ascontiguousarray(query[b:b + 1], dtype=np.float32)).to(torch.bfloat16)
        window = q.shape[2]
        groups = q.shape[1] // kv_heads
        t0 = time.perf_counter()
        keys, values = mirror.materialize_legacy_cache(torch, template=legacy)[0]
        keys = keys.repeat_interleave(groups, dim=1)
        values = values.repeat_interleave(groups, dim=1)
        mask = torch.arange(T - window, T).unsqueeze(1) >= torch.arange(T).unsqueeze(0)
        torch.nn.functional.scaled_dot_product_attention(q, keys, values, attn_mask=mask, dropout_p=0.0)
        elapsed += time.perf_counter() - t0
        sequences += 1
        tokens += T
        del mirror, keys, values
        if elapsed >= budget_s:
            break
    return {"seconds": elapsed, "sequences": sequences, "tokens": tokens, "synchronize_seconds": sync_s,
            "threads": threads}


def nested(x: np.ndarray):
    """A ``[tokens, layers, heads, dim]`` array as the reference's append
    entries: per token a pair of nested ``[layer][head][dim]`` float lists."""
    return [row.tolist() for row in x]


def time_append_rollback(layers: int, kv_heads: int, head_dim: int, block_size: int, num_blocks: int,
                         events, budget_s: float):
    """Drive the reference's ``PagedKVCache`` with ``NativeKVQuantizer``
    through ``events`` until ``budget_s`` of timed work: each event is
    ``("append", seq, keys, values)`` with ``[tokens, layers, heads, dim]``
    arrays, or ``("truncate", seq, new_length)``.  Only the reference's
    ``append_many`` / ``truncate`` calls are timed; building the nested
    input lists is not.  Returns a dict of token counts and seconds."""
    reference_package()
    from specdecode.kv_cache import KVCacheConfig, PagedKVCache

    cache = PagedKVCache(KVCacheConfig(layers, kv_heads, head_dim, block_size=block_size, num_blocks=num_blocks),
                         quantizer=native_quantizer())
    created = set()
    append_s = truncate_s = 0.0
    appended = rolled = events_done = 0
    for event in events:
        if event[0] == "append":
            _, seq, keys, values = event
            if seq not in created:
                cache.create_sequence(seq)
                created.add(seq)
            entries = list(zip(nested(keys), nested(values)))
            t0 = time.perf_counter()
            cache.append_many(seq, entries)
            append_s += time.perf_counter() - t0
            appended += len(entries)
        else:
            _, seq, count = event
            before = cache.sequence_length(seq)
            t0 = time.perf_counter()
            cache.truncate(seq, int(count))
            truncate_s += time.perf_counter() - t0
            rolled += before - int(count)
        events_done += 1
        if append_s + truncate_s >= budget_s:
            break
    return {"append_seconds": append_s, "truncate_seconds": truncate_s, "appended_tokens": appended,
            "rolled_back_tokens": rolled, "events": events_done, "sequences": len(created)}


def gb_per_s(nbytes: float, seconds: float) -> float:
    return nbytes / seconds / 1e9 if seconds > 0 else math.nan
