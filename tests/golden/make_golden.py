"""Generate the golden fixtures in tests/golden/ by running the reference itself.

Run in a checkout that has the reference at /root/reference (read-only) and
its C++ quantizer built by ``make -C oracle ref``::

    python tests/golden/make_golden.py

It imports the reference's Python package from /root/reference/src and loads
its native library from oracle/_ref/, then records:

* kat_quant.json        the reference tests' known-answer quantization vectors,
                        the round-half-away tie vector, error cases, and random
                        float32/bf16-valued vectors; Python and C++ quantizers
                        must agree and both results are stored
* small_speculative.npz a small speculative append/rollback workload run through
                        the reference PagedKVCache: final storage in the
                        kernel-facing layout, block tables after every step,
                        lengths and stats
* full_speculative.json the full CPU-runnable workload (16 layers, 8 heads,
                        head_dim 64, 4 x 512 prefill, 64 rounds x 5) reduced to
                        a sha256 of tables, lengths and storage
* attention_small.npz   the reference's unfused paged attention
                        (submit_paged_attention) run on CPU torch in bf16 and
                        fp32 for small random caches

Nothing at test time reads /root/reference; tests only read these fixtures.
"""

from __future__ import annotations

import json
import math
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
REFERENCE_SRC = Path("/root/reference/src")
sys.path.insert(0, str(REFERENCE_SRC))
sys.path.insert(0, str(REPO))

import torch  # noqa: E402

from specdecode import cuda_kv_cache as ref_cuda  # noqa: E402
from specdecode.kv_cache import KVCacheConfig, PagedKVCache, PythonKVQuantizer  # noqa: E402
from specdecode.native import NativeBackendError, NativeKVQuantizer  # noqa: E402

from oracle.workloads import (  # noqa: E402
    FULL_SPECULATIVE,
    SMALL_SPECULATIVE,
    speculative_events,
    state_digest,
)

OUT = Path(__file__).resolve().parent
NATIVE_LIB = REPO / "oracle" / "_ref" / "libspecdecode_native.so"


def _bf16_values(rng, n):
    x = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).to(torch.bfloat16)
    return [float(v) for v in x.float().tolist()]


def _tie_vector(rng, n):
    """Values that are exact half-integer multiples of their own scale."""
    target_scale = float(np.float32(rng.uniform(0.01, 3.0)))
    # choose m = 127 * s exactly representable; quantizer recomputes s from m
    m = float(np.float32(127.0 * target_scale))
    s = float(np.float32(m / 127.0))
    vals = [m]
    for _ in range(n - 1):
        k = int(rng.integers(-126, 126))
        vals.append(float(np.float32((k + 0.5) * s)))
    return vals


def kat_quant(python_q, native_q) -> dict:
    rng = np.random.default_rng(1234)
    cases = {
        "reference_kat": [-1.0, -0.5, 0.0, 0.5, 1.0],
        "zero": [0.0, 0.0, 0.0],
        "native_parity": [0.001, -12.5, 3.25, 99.0],
        "tie": [127.0, 0.5, 1.5, 2.5, -2.5, -0.5],
        "single": [3.0],
        "negative_zero": [-0.0, 0.0, -0.0],
        "tiny": [1e-30, -2e-30, 5e-31],
        "huge": [3.0e38, -1.0e38, 2.5e37],
    }
    for i in range(24):
        cases[f"f32_random_{i}"] = [float(v) for v in rng.standard_normal(64).astype(np.float32)]
    for i in range(24):
        cases[f"bf16_random_{i}"] = _bf16_values(rng, 128)
    for i in range(24):
        cases[f"tie_random_{i}"] = _tie_vector(rng, 64)
    results = {}
    for name, vec in cases.items():
        p = python_q.quantize(vec)
        n = native_q.quantize(vec)
        assert p == n, name
        results[name] = {"input": vec, "codes": list(p.values), "scale": p.scale,
                         "dequantized": list(native_q.dequantize(n))}
    errors = {}
    for name, vec in {"empty": [], "nan": [1.0, math.nan], "inf": [math.inf, 1.0],
                      "neg_inf": [-math.inf]}.items():
        try:
            native_q.quantize(vec)
            status = 0
        except NativeBackendError as error:
            status = error.status
        errors[name] = {"input": [repr(v) for v in vec], "status": status}
    return {"vectors": results, "errors": errors}


def run_reference_workload(shape, seed, quantizer, snapshot_tables=False):
    config = KVCacheConfig(shape.num_layers, shape.num_heads, shape.head_dim,
                           block_size=shape.block_size, num_blocks=shape.num_blocks)
    cache = PagedKVCache(config, quantizer=quantizer)
    for s in range(shape.sequences):
        cache.create_sequence(s)
    snapshots = []
    for event in speculative_events(shape, seed):
        if event[0] == "append":
            _, seq, k, v = event
            entries = [(k[i].tolist(), v[i].tolist()) for i in range(k.shape[0])]
            cache.append_many(seq, entries)
        else:
            _, seq, count = event
            cache.truncate(seq, count)
        cache.validate_invariants()
        if snapshot_tables:
            snapshots.append([list(cache.block_table(s)) for s in range(shape.sequences)])
    return cache, snapshots


def logical_storage(cache, shape):
    L, H, D = shape.num_layers, shape.num_heads, shape.head_dim
    keys = np.zeros((shape.num_blocks, shape.block_size, L, H, D), np.int8)
    values = np.zeros_like(keys)
    kscale = np.zeros((shape.num_blocks, shape.block_size, L, H), np.float32)
    vscale = np.zeros_like(kscale)
    for b, block in enumerate(cache._blocks):  # read-only inspection of reference state
        for o, token in enumerate(block):
            if token is None:
                continue
            for layer in range(L):
                for h in range(H):
                    keys[b, o, layer, h] = token.keys[layer][h].values
                    values[b, o, layer, h] = token.values[layer][h].values
                    kscale[b, o, layer, h] = token.keys[layer][h].scale
                    vscale[b, o, layer, h] = token.values[layer][h].scale
    tables = {s: list(cache.block_table(s)) for s in range(shape.sequences)}
    lengths = {s: cache.sequence_length(s) for s in range(shape.sequences)}
    return tables, lengths, keys, values, kscale, vscale


class _CpuRuntime:
    """Just enough of CudaExecutionRuntime for submit_paged_attention on CPU."""

    def __init__(self):
        self.device = torch.device("cpu")
        self.torch_module = torch

    def submit_target(self, operation, *, wait_for=(), label=""):
        class _Task:
            pass

        task = _Task()
        task.result = operation()
        return task


def attention_cases() -> dict:
    rng = np.random.default_rng(99)
    runtime = _CpuRuntime()
    arrays = {}
    specs = [
        # (Hq, Hkv, D, kw, T, bs, L, layer, nb)
        (4, 2, 16, 3, 37, 4, 2, 1, 16),
        (8, 2, 32, 5, 70, 16, 1, 0, 8),
        (2, 1, 8, 1, 9, 2, 1, 0, 8),
        (8, 8, 16, 5, 5, 4, 3, 2, 4),
        (32, 8, 128, 5, 100, 16, 1, 0, 8),
    ]
    for index, (hq, hkv, d, kw, T, bs, L, layer, nb) in enumerate(specs):
        nblk = (T + bs - 1) // bs
        table = rng.permutation(nb)[:nblk].astype(np.int64)
        keys = rng.integers(-127, 128, size=(nb, bs, L, hkv, d)).astype(np.int8)
        values = rng.integers(-127, 128, size=(nb, bs, L, hkv, d)).astype(np.int8)
        kscale = rng.uniform(0.001, 0.05, size=(nb, bs, L, hkv)).astype(np.float32)
        vscale = rng.uniform(0.001, 0.05, size=(nb, bs, L, hkv)).astype(np.float32)
        q32 = rng.standard_normal((1, hq, kw, d)).astype(np.float32)
        view = ref_cuda.CudaPagedKVCacheView(
            keys=torch.from_numpy(keys), values=torch.from_numpy(values),
            key_scales=torch.from_numpy(kscale), value_scales=torch.from_numpy(vscale),
            block_table=torch.from_numpy(table), token_count=T, block_size=bs)
        outs = {}
        for name, dtype in (("bf16", torch.bfloat16), ("f32", torch.float32)):
            q = torch.from_numpy(q32).to(dtype)
            task = ref_cuda.submit_paged_attention(runtime, q, view, layer)
            outs[name] = task.result.float().numpy()
        prefix = f"case{index}_"
        arrays.update({
            prefix + "spec": np.array([hq, hkv, d, kw, T, bs, L, layer, nb], np.int64),
            prefix + "table": table, prefix + "keys": keys, prefix + "values": values,
            prefix + "key_scales": kscale, prefix + "value_scales": vscale,
            prefix + "query_f32": q32,
            prefix + "query_bf16_bits": torch.from_numpy(q32).to(torch.bfloat16).view(torch.int16).numpy(),
            prefix + "out_bf16": outs["bf16"], prefix + "out_f32": outs["f32"],
        })
    arrays["num_cases"] = np.array([len(specs)], np.int64)
    return arrays


def main() -> None:
    python_q = PythonKVQuantizer()
    native_q = NativeKVQuantizer.load(str(NATIVE_LIB))

    kat = kat_quant(python_q, native_q)
    (OUT / "kat_quant.json").write_text(json.dumps(kat, indent=0, sort_keys=True))
    print("kat_quant.json:", len(kat["vectors"]), "vectors")

    shape = SMALL_SPECULATIVE
    cache, snapshots = run_reference_workload(shape, 7, python_q, snapshot_tables=True)
    tables, lengths, keys, values, ks, vs = logical_storage(cache, shape)
    width = max(len(t) for snap in snapshots for t in snap)
    snap_arr = np.full((len(snapshots), shape.sequences, width), -1, np.int64)
    for i, snap in enumerate(snapshots):
        for s, t in enumerate(snap):
            snap_arr[i, s, :len(t)] = t
    stats = cache.stats()
    np.savez_compressed(
        OUT / "small_speculative.npz", keys=keys, values=values, key_scales=ks, value_scales=vs,
        lengths=np.array([lengths[s] for s in range(shape.sequences)], np.int64),
        table_snapshots=snap_arr,
        stats=np.array([stats.sequences, stats.used_tokens, stats.capacity_tokens,
                        stats.allocated_blocks, stats.free_blocks, stats.used_quantized_bytes,
                        stats.allocated_quantized_bytes, stats.capacity_quantized_bytes,
                        stats.fp32_equivalent_bytes, stats.block_table_bytes], np.int64),
        seed=np.array([7], np.int64))
    print("small_speculative.npz: digest", state_digest(tables, lengths, keys, values, ks, vs))

    start = time.perf_counter()
    full_cache, _ = run_reference_workload(FULL_SPECULATIVE, 11, native_q)
    elapsed = time.perf_counter() - start
    tables, lengths, keys, values, ks, vs = logical_storage(full_cache, FULL_SPECULATIVE)
    digest = state_digest(tables, lengths, keys, values, ks, vs)
    (OUT / "full_speculative.json").write_text(json.dumps({
        "seed": 11, "digest": digest, "lengths": [lengths[s] for s in sorted(lengths)],
        "tables_sha256_only": True, "reference_seconds": round(elapsed, 1),
        "quantizer": "NativeKVQuantizer (reference C++ built from native/src/native.cpp)",
    }, indent=1))
    print("full_speculative.json:", digest, f"{elapsed:.1f}s")

    np.savez_compressed(OUT / "attention_small.npz", **attention_cases())
    print("attention_small.npz written")


if __name__ == "__main__":
    main()
