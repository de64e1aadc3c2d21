"""Device PagedKVCache (quantize-append and rollback kernels) against the
reference: bit-exact codes, scale bits, block tables, lengths, stats, and
zeroed released slots."""

from __future__ import annotations

import json
import math

import numpy as np
import pytest

from gpu_helpers import make_cache, read_logical
from oracle.paged_cache import PagedCacheOracle
from oracle.quant import bits_f32
from oracle.workloads import FULL_SPECULATIVE, SMALL_SPECULATIVE, speculative_events, state_digest

pytestmark = pytest.mark.gpu


def replay(cache, shape, seed, snapshots=None):
    import torch

    for s in range(shape.sequences):
        cache.create_sequence(s)
    for step, event in enumerate(speculative_events(shape, seed)):
        if event[0] == "append":
            k = torch.from_numpy(event[2]).to(cache.device)
            v = torch.from_numpy(event[3]).to(cache.device)
            cache.append_tensor(event[1], k, v)
        else:
            cache.truncate(event[1], event[2])
        if snapshots is not None:
            snap = snapshots[step]
            for s in range(shape.sequences):
                assert list(cache.block_table(s)) == [b for b in snap[s].tolist() if b >= 0], (step, s)
    cache.validate_invariants()


def test_small_workload_matches_reference_fixture(device, golden_dir):
    golden = np.load(golden_dir / "small_speculative.npz")
    shape = SMALL_SPECULATIVE
    cache = make_cache(device, shape.num_layers, shape.num_heads, shape.head_dim, shape.block_size,
                       shape.num_blocks)
    replay(cache, shape, int(golden["seed"][0]), golden["table_snapshots"])
    keys, values, ks, vs = read_logical(cache)
    assert np.array_equal(keys, golden["keys"])
    assert np.array_equal(values, golden["values"])
    assert np.array_equal(bits_f32(ks), bits_f32(golden["key_scales"]))
    assert np.array_equal(bits_f32(vs), bits_f32(golden["value_scales"]))
    assert [cache.sequence_length(s) for s in range(shape.sequences)] == golden["lengths"].tolist()
    st = cache.stats()
    assert [st.sequences, st.used_tokens, st.capacity_tokens, st.allocated_blocks, st.free_blocks,
            st.used_quantized_bytes, st.allocated_quantized_bytes, st.capacity_quantized_bytes,
            st.fp32_equivalent_bytes, st.block_table_bytes] == golden["stats"].tolist()
    assert cache.status_bits() == 0


def test_full_cpu_reference_workload_digest(device, golden_dir):
    """16 layers, 8 heads, head_dim 64: 4 x 512 prefill and 64 speculative
    rounds of 5 tokens with Bernoulli(0.7) acceptance, rolled back."""
    expected = json.loads((golden_dir / "full_speculative.json").read_text())
    shape = FULL_SPECULATIVE
    cache = make_cache(device, shape.num_layers, shape.num_heads, shape.head_dim, shape.block_size,
                       shape.num_blocks, check_status=False)
    replay(cache, shape, expected["seed"])
    assert cache.status_bits() == 0
    keys, values, ks, vs = read_logical(cache)
    tables = {s: list(cache.block_table(s)) for s in range(shape.sequences)}
    lengths = {s: cache.sequence_length(s) for s in range(shape.sequences)}
    assert [lengths[s] for s in range(shape.sequences)] == expected["lengths"]
    assert state_digest(tables, lengths, keys, values, ks, vs) == expected["digest"]


@pytest.mark.parametrize("src_dtype", ["float32", "bfloat16", "float16"])
def test_batched_append_and_rollback_match_oracle(device, src_dtype):
    """Append-benchmark shape in small: many sequences, 5-token windows,
    0..5 tokens rolled back each, randomly relabelled physical blocks."""
    import torch

    rng = np.random.default_rng(31)
    L, H, D, bs, nb, B = 3, 4, 128, 16, 512, 24
    order = rng.permutation(nb)
    cache = make_cache(device, L, H, D, bs, nb, block_order=order, check_status=False)
    oracle = PagedCacheOracle(L, H, D, bs, nb, block_order=order)
    seqs = list(range(B))
    for s in seqs:
        cache.create_sequence(s)
        oracle.create_sequence(s)
    dtype = getattr(torch, src_dtype)
    for step in range(12):
        factors = np.exp(rng.uniform(np.log(0.1), np.log(10.0), size=(1, 1, 1, H, 1)))
        k = torch.from_numpy(rng.standard_normal((B, 5, L, H, D)) * factors).to(dtype)
        v = torch.from_numpy(rng.standard_normal((B, 5, L, H, D)) * factors).to(dtype)
        cache.append_batch(seqs, k.to(device), v.to(device))
        k64, v64 = k.double().numpy(), v.double().numpy()
        for i, s in enumerate(seqs):
            oracle.append_many(s, k64[i], v64[i])
        rolled = rng.integers(0, 6, size=B)
        counts = [cache.sequence_length(s) - int(r) for s, r in zip(seqs, rolled)]
        released = cache.truncate_batch(seqs, counts)
        assert released == [oracle.truncate(s, c) for s, c in zip(seqs, counts)]
        for s in seqs:
            assert cache.block_table(s) == oracle.block_table(s)
    assert cache.status_bits() == 0
    keys, values, ks, vs = read_logical(cache)
    assert np.array_equal(keys, oracle.keys)
    assert np.array_equal(values, oracle.values)
    assert np.array_equal(bits_f32(ks), bits_f32(oracle.key_scales))
    assert np.array_equal(bits_f32(vs), bits_f32(oracle.value_scales))
    # device tables and lengths mirror the host state
    rows = [cache.table_row(s) for s in seqs]
    dev_tables = cache.block_tables.cpu().numpy()
    dev_lens = cache.context_lens.cpu().numpy()
    for s, r in zip(seqs, rows):
        t = cache.block_table(s)
        assert dev_tables[r, : len(t)].tolist() == list(t)
        assert (dev_tables[r, len(t):] == -1).all()
        assert dev_lens[r] == cache.sequence_length(s)
    cache.validate_invariants()


def _entry(L, H, D, base):
    keys = tuple(tuple(tuple(base + l * 0.7 + h * 0.2 + d * 0.05 for d in range(D)) for h in range(H))
                 for l in range(L))
    values = tuple(tuple(tuple(-base - 0.25 + l * 0.7 + h * 0.2 + d * 0.05 for d in range(D)) for h in range(H))
                   for l in range(L))
    return keys, values


def test_reference_api_cases(device):
    """tests/test_kv_cache.py:61-208 of the reference, with head_dim 16."""
    from specdecode_b200.kv_cache import KVCacheCapacityError, QuantizedVector

    L, H, D = 2, 2, 16
    cache = make_cache(device, L, H, D, 2, 4)
    cache.create_sequence("request-a")
    assert cache.append_many("request-a", [_entry(L, H, D, float(i + 1)) for i in range(3)]) == (0, 1, 2)
    assert cache.block_table("request-a") == (0, 1)
    assert cache.physical_slot("request-a", 2) == (1, 0)
    # read path equals the oracle quantizer + double dequantization
    from oracle.quant import dequantize_vector, quantize_vector

    token = cache.read_quantized_token("request-a", 1)
    restored = cache.read_token("request-a", 1)
    keys, _ = _entry(L, H, D, 2.0)
    for l in range(L):
        for h in range(H):
            codes, scale = quantize_vector(keys[l][h])
            assert token.keys[l][h] == QuantizedVector(codes, scale)
            assert restored.keys[l][h] == dequantize_vector(codes, scale)
            for x, y in zip(keys[l][h], restored.keys[l][h]):
                assert abs(x - y) <= scale / 2 + 1e-14
    assert len(cache.read_sequence("request-a")) == 3
    # rollback releases the suffix block and reuses slot (1, 1)
    checkpoint = cache.checkpoint("request-a")
    cache.append_many("request-a", [_entry(L, H, D, float(i)) for i in range(4, 7)])
    assert cache.rollback("request-a", checkpoint) == 1
    assert cache.block_table("request-a") == (0, 1)
    cache.append("request-a", *_entry(L, H, D, 9.0))
    assert cache.physical_slot("request-a", 3) == (1, 1)
    # capacity failure is atomic
    with pytest.raises(KVCacheCapacityError):
        cache.append_many("request-a", [_entry(L, H, D, 1.0)] * 5)
    assert cache.sequence_length("request-a") == 4
    # malformed entry is rejected before anything is written
    with pytest.raises(ValueError):
        cache.append_many("request-a", [_entry(L, H, D, 1.0), ((((1.0, 2.0),),), _entry(L, H, D, 1.0)[1])])
    with pytest.raises(TypeError):
        cache.append("request-a", ((((True,) * D,) * H),) * L, _entry(L, H, D, 1.0)[1])
    assert cache.sequence_length("request-a") == 4
    cache.create_sequence("b")
    with pytest.raises(ValueError):
        cache.rollback("b", checkpoint)
    assert cache.remove_sequence("request-a") == 2
    cache.validate_invariants()
    stats = cache.stats()
    assert stats.used_tokens == 0 and stats.free_blocks == 4


def test_nonfinite_append_is_atomic_and_leaves_zeroed_slots(device):
    import torch

    L, H, D = 2, 2, 32
    cache = make_cache(device, L, H, D, 4, 8)
    cache.create_sequence("a")
    good = torch.randn(3, L, H, D, device=device)
    cache.append_tensor("a", good, good)
    before = [t.clone() for t in (cache.key_codes, cache.value_codes, cache.key_scale_pages, cache.value_scale_pages)]
    bad = torch.randn(6, L, H, D, device=device)
    bad[4, 1, 0, 7] = float("nan")
    with pytest.raises(ValueError):
        cache.append_tensor("a", bad, bad)
    assert cache.sequence_length("a") == 3
    assert cache.block_table("a") == (0,)
    after = (cache.key_codes, cache.value_codes, cache.key_scale_pages, cache.value_scale_pages)
    for x, y in zip(before, after):
        assert torch.equal(x, y)
    assert cache.context_lens[cache.table_row("a")].item() == 3
    cache.validate_invariants()


def test_device_fault_bits_for_bad_slots(device):
    """A slot outside the pool is skipped and reported, never written."""
    import ctypes

    import torch

    from specdecode_b200 import _lib

    cache = make_cache(device, 1, 1, 16, 2, 2, check_status=False)
    lib = cache.library
    src = torch.ones(1, 1, 1, 16, device=device)
    slots = torch.tensor([99], dtype=torch.int64, device=device)
    rc = lib.handle.sdc_quantize_append(ctypes.byref(cache.pool_desc), 0, 1, src.data_ptr(), src.data_ptr(),
                                        _lib.DTYPE_F32, 1, 16, 16, 16, slots.data_ptr(), None,
                                        cache._status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    assert cache.status_bits() == _lib.FAULT_SLOT_RANGE
    assert int(cache.key_codes.abs().sum()) == 0


def test_float64_entries_take_the_double_path(device):
    """Python floats quantize exactly as the reference's double arithmetic."""
    from oracle.quant import quantize_vector

    cache = make_cache(device, 1, 1, 16, 4, 4)
    cache.create_sequence(0)
    vec = [0.1 * (i - 7) + 1e-17 * i for i in range(16)]
    cache.append(0, ((vec,),), ((vec[::-1],),))
    token = cache.read_quantized_token(0, 0)
    codes, scale = quantize_vector(vec)
    assert token.keys[0][0].values == codes and token.keys[0][0].scale == scale
    assert math.isfinite(token.values[0][0].scale)


@pytest.mark.parametrize("layers,sequences,window", [(7, 64, 10), (32, 8, 5)])
def test_rollback_spans_of_layers_match_oracle(device, layers, sequences, window):
    """Rollbacks whose blocks clear several layers each (many rolled slots
    over 7 layers: spans of 4 and a last span of 3; few slots over 32
    layers: spans of 2): every released slot holds zeros, codes and scales,
    and the kept ones are untouched."""
    import torch

    rng = np.random.default_rng(layers * 100 + sequences)
    H, D, bs, nb = 2, 64, 16, 512
    order = rng.permutation(nb)
    cache = make_cache(device, layers, H, D, bs, nb, block_order=order, check_status=False)
    oracle = PagedCacheOracle(layers, H, D, bs, nb, block_order=order)
    seqs = list(range(sequences))
    for s in seqs:
        cache.create_sequence(s)
        oracle.create_sequence(s)
    for step in range(4):
        k = torch.from_numpy(rng.standard_normal((sequences, window, layers, H, D))).to(torch.bfloat16)
        v = torch.from_numpy(rng.standard_normal((sequences, window, layers, H, D))).to(torch.bfloat16)
        cache.append_batch(seqs, k.to(device), v.to(device))
        k64, v64 = k.double().numpy(), v.double().numpy()
        for i, s in enumerate(seqs):
            oracle.append_many(s, k64[i], v64[i])
        rolled = rng.integers(0, window + 1, size=sequences)
        counts = [cache.sequence_length(s) - int(r) for s, r in zip(seqs, rolled)]
        assert cache.truncate_batch(seqs, counts) == [oracle.truncate(s, c) for s, c in zip(seqs, counts)]
    assert cache.status_bits() == 0
    keys, values, ks, vs = read_logical(cache)
    assert np.array_equal(keys, oracle.keys)
    assert np.array_equal(values, oracle.values)
    assert np.array_equal(bits_f32(ks), bits_f32(oracle.key_scales))
    assert np.array_equal(bits_f32(vs), bits_f32(oracle.value_scales))


def test_gather_slots_equals_gather_sequence(device):
    """The device-slot gather returns the same dequantized rows as the
    sequence gather, for slots listed in any order."""
    import torch

    rng = np.random.default_rng(5)
    L, H, D, bs, nb = 2, 4, 128, 16, 64
    cache = make_cache(device, L, H, D, bs, nb, block_order=rng.permutation(nb))
    cache.create_sequence("a")
    k = torch.from_numpy(rng.standard_normal((150, L, H, D))).to(torch.bfloat16).to(device)
    v = torch.from_numpy(rng.standard_normal((150, L, H, D))).to(torch.bfloat16).to(device)
    cache.append_tensor("a", k, v)
    want_k, want_v = cache.gather_sequence("a", torch.float32)
    slots = [b * bs + o for b, o in (cache.physical_slot("a", t) for t in range(150))]
    perm = rng.permutation(150)
    got_k, got_v = cache.gather_slots(torch.tensor([slots[i] for i in perm], device=device), torch.float32)
    assert torch.equal(got_k, want_k[torch.from_numpy(perm).to(device)])
    assert torch.equal(got_v, want_v[torch.from_numpy(perm).to(device)])
    with pytest.raises(TypeError):
        cache.gather_slots(torch.tensor(slots, dtype=torch.int32, device=device), torch.float32)
