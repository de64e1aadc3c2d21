"""The device-resident page allocator (csrc/page_alloc.cu, DevicePagedCache).

* Without sharing, every block table, length and pool byte equals the
  oracle's restatement of the reference allocator (lowest free block first,
  src/specdecode/kv_cache.py:220-427) after each step of a seeded sequence of
  batched appends, rollbacks and releases, with and without a permuted
  block order; attention over the device tables matches the oracle.
* Prefix sharing: forked rows read their source's tokens, appends copy a
  shared partly filled block first, concurrent appends by every holder of a
  block leave one holder with it, and releasing everything returns every
  block with all-zero pages.
* Faulted calls (a pool short of blocks, a rollback past the length, a fork
  into a non-empty row) change nothing.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

L, H, D, BS = 2, 2, 32, 4


def _cache(device, nb, rows, block_order=None):
    from specdecode_b200.device_pages import DevicePagedCache
    from specdecode_b200.kv_cache import KVCacheConfig

    return DevicePagedCache(KVCacheConfig(L, H, D, block_size=BS, num_blocks=nb), max_rows=rows,
                            max_blocks_per_row=nb, block_order=block_order, device=device)


def _pool(cache):
    """Device pool in the oracle's [block, offset, layer, head, dim] layout."""
    return (cache.key_codes.permute(0, 3, 1, 2, 4).contiguous().cpu().numpy(),
            cache.value_codes.permute(0, 3, 1, 2, 4).contiguous().cpu().numpy(),
            cache.key_scale_pages.permute(0, 3, 1, 2).contiguous().cpu().numpy(),
            cache.value_scale_pages.permute(0, 3, 1, 2).contiguous().cpu().numpy())


def _same_tables(cache, oracle, rows):
    snap = cache.snapshot()
    for r in rows:
        n = oracle.sequence_length(r)
        assert snap["lengths"][r] == n, r
        used = -(-n // BS)
        assert list(snap["tables"][r, :used]) == list(oracle.block_table(r)), r
        assert (snap["tables"][r, used:] == -1).all(), r


@pytest.mark.parametrize("permuted", [False, True])
def test_tables_and_pool_follow_the_reference_allocator(device, permuted):
    import torch

    from oracle.paged_cache import PagedCacheOracle

    nb, R = 96, 6
    rng = np.random.default_rng(7 + permuted)
    order = rng.permutation(nb) if permuted else None
    cache = _cache(device, nb, R, order)
    oracle = PagedCacheOracle(L, H, D, BS, nb, block_order=order, use_c=False)
    for r in range(R):
        oracle.create_sequence(r)
    for step in range(40):
        rows = [int(r) for r in rng.permutation(R)[: rng.integers(1, R + 1)]]
        if step % 3 != 2:
            n = int(rng.integers(0, 12))
            keys = rng.standard_normal((len(rows), n, L, H, D)).astype(np.float32)
            values = rng.standard_normal((len(rows), n, L, H, D)).astype(np.float32)
            room = sum(-(-(oracle.sequence_length(r) + n) // BS) - -(-oracle.sequence_length(r) // BS)
                       for r in rows)
            if room > oracle.free_blocks():
                continue
            cache.append(rows, torch.from_numpy(keys), torch.from_numpy(values))
            for i, r in enumerate(rows):
                oracle.append_many(r, keys[i], values[i])
        else:
            lengths = [int(rng.integers(0, oracle.sequence_length(r) + 1)) for r in rows]
            if step % 9 == 8:
                lengths = [0] * len(rows)
            cache.truncate(rows, lengths)
            for r, n in zip(rows, lengths):
                oracle.truncate(r, n)
        cache.check_status()
        _same_tables(cache, oracle, range(R))
        if step % 10 == 9:
            cache.validate_invariants()
    k, v, ks, vs = _pool(cache)
    assert np.array_equal(k, oracle.keys) and np.array_equal(v, oracle.values)
    assert np.array_equal(ks.view(np.uint32), oracle.key_scales.view(np.uint32))
    assert np.array_equal(vs.view(np.uint32), oracle.value_scales.view(np.uint32))

    # attention over the device tables and lengths
    from oracle.attention import attention_fp64

    live = [r for r in range(R) if oracle.sequence_length(r) >= 2]
    if live:
        attention = cache.attention()
        q = torch.randn((len(live), 4, 2, D), generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
        idx = torch.tensor(live, device=device)
        out = attention(q.to(device), cache.block_tables[idx].contiguous(), cache.context_lens[idx].contiguous(),
                        int(max(oracle.sequence_length(r) for r in live)), 1).float().cpu().numpy()
        cache.check_status()
        for i, r in enumerate(live):
            exact = attention_fp64(q[i].float().numpy(), *oracle.gather(r, 1))
            assert np.abs(out[i] - exact).max() <= 1e-2


def _read_tokens(cache, row):
    """(codes, scales) of a row's cached tokens, read through its table."""
    snap = cache.snapshot()
    n = int(snap["lengths"][row])
    k, v, ks, vs = _pool(cache)
    idx = np.arange(n)
    blocks = snap["tables"][row][idx // BS]
    return k[blocks, idx % BS], v[blocks, idx % BS], ks[blocks, idx % BS], vs[blocks, idx % BS]


def test_fork_shares_blocks_and_copies_on_write(device):
    import torch

    from oracle.quant import quantize_rows

    nb = 32
    cache = _cache(device, nb, 4)
    rng = np.random.default_rng(11)

    def tokens(n):
        return (rng.standard_normal((1, n, L, H, D)).astype(np.float32),
                rng.standard_normal((1, n, L, H, D)).astype(np.float32))

    expected = {}

    def append(rows, n):
        ks, vs = zip(*[tokens(n) for _ in rows])
        keys, values = np.concatenate(ks), np.concatenate(vs)
        cache.append(rows, torch.from_numpy(keys), torch.from_numpy(values))
        for i, r in enumerate(rows):
            expected[r] = expected.get(r, []) + list(zip(keys[i], values[i]))

    def check(row):
        k, v, ksc, vsc = _read_tokens(cache, row)
        want = expected.get(row, [])
        assert k.shape[0] == len(want)
        for t, (wk, wv) in enumerate(want):
            ck, cs, _ = quantize_rows(wk)
            cv, vsc_want, _ = quantize_rows(wv)
            assert np.array_equal(k[t], ck) and np.array_equal(v[t], cv), (row, t)
            assert np.array_equal(ksc[t].view(np.uint32), cs.view(np.uint32)), (row, t)
            assert np.array_equal(vsc[t].view(np.uint32), vsc_want.view(np.uint32)), (row, t)

    append([0], 10)  # blocks 0, 1 and 2 (two rows of block 2)
    free_before = int(cache.snapshot()["free"].sum())
    cache.fork([0, 0], [1, 2])
    expected[1] = list(expected[0])
    expected[2] = list(expected[0])
    cache.check_status()
    snap = cache.snapshot()
    assert int(snap["free"].sum()) == free_before  # sharing takes no block
    assert list(snap["refcount"][:3]) == [3, 3, 3]
    for r in (0, 1, 2):
        check(r)
    append([1], 3)  # copies block 2 first
    cache.check_status()
    snap = cache.snapshot()
    assert snap["refcount"][2] == 2 and snap["tables"][1, 2] != 2
    for r in (0, 1, 2):
        check(r)
    append([0, 2], 5)  # both remaining holders of block 2: one copies, one keeps it
    cache.check_status()
    cache.validate_invariants()
    snap = cache.snapshot()
    assert snap["refcount"][2] == 1
    assert sorted([snap["tables"][0, 2] == 2, snap["tables"][2, 2] == 2]) == [False, True]
    for r in (0, 1, 2):
        check(r)
    cache.truncate([1], [5])
    expected[1] = expected[1][:5]
    cache.check_status()
    cache.validate_invariants()
    for r in (0, 1, 2):
        check(r)
    cache.release([0, 1, 2])
    cache.check_status()
    cache.validate_invariants()
    snap = cache.snapshot()
    assert snap["free"].all() and (snap["refcount"] == 0).all()
    k, v, ks, vs = _pool(cache)
    assert not k.any() and not v.any() and not ks.any() and not vs.any()


def test_faulted_calls_change_nothing(device):
    import torch

    from specdecode_b200.kv_cache import KVCacheCapacityError, KVCacheError

    nb = 8
    cache = _cache(device, nb, 3)
    x = torch.randn((1, 9, L, H, D))
    cache.append([0], x, x)  # 3 blocks
    cache.check_status()
    before = cache.snapshot()
    pool_before = _pool(cache)

    def unchanged():
        after = cache.snapshot()
        for key in before:
            assert np.array_equal(before[key], after[key]), key
        for a, b in zip(pool_before, _pool(cache)):
            assert np.array_equal(a, b)

    y = torch.randn((2, 12, L, H, D))
    cache.append([1, 2], y, y)  # 6 more blocks: the pool has 5
    with pytest.raises(KVCacheCapacityError):
        cache.check_status()
    unchanged()
    cache.truncate([1], [4])  # row 1 is empty
    with pytest.raises(KVCacheError):
        cache.check_status()
    unchanged()
    cache.fork([1], [0])  # row 0 is not empty
    with pytest.raises(KVCacheError):
        cache.check_status()
    unchanged()
    with pytest.raises(ValueError):
        cache.reserve([0, 0], [1, 1])


def test_truncate_zeroing_in_layer_spans_follows_the_reference(device):
    """Enough rows and removed tokens that each zeroing block clears several
    layers (nine layers in spans of three): the pool after every step equals
    the reference allocator's, freed slots all zero."""
    import torch

    from oracle.paged_cache import PagedCacheOracle
    from specdecode_b200.device_pages import DevicePagedCache
    from specdecode_b200.kv_cache import KVCacheConfig

    layers, nb, R = 9, 512, 64
    rng = np.random.default_rng(17)
    order = rng.permutation(nb)
    cache = DevicePagedCache(KVCacheConfig(layers, H, D, block_size=BS, num_blocks=nb), max_rows=R,
                             max_blocks_per_row=32, block_order=order, device=device)
    oracle = PagedCacheOracle(layers, H, D, BS, nb, block_order=order, use_c=False)
    rows = list(range(R))
    for r in rows:
        oracle.create_sequence(r)
    for step in range(4):
        keys = rng.standard_normal((R, 12, layers, H, D)).astype(np.float32)
        values = rng.standard_normal((R, 12, layers, H, D)).astype(np.float32)
        cache.append(rows, torch.from_numpy(keys), torch.from_numpy(values))
        for i, r in enumerate(rows):
            oracle.append_many(r, keys[i], values[i])
        lengths = [max(0, oracle.sequence_length(r) - int(rng.integers(0, 13))) for r in rows]
        cache.truncate(rows, lengths)
        for r, n in zip(rows, lengths):
            oracle.truncate(r, n)
        cache.check_status()
    cache.validate_invariants()
    k = cache.key_codes.permute(0, 3, 1, 2, 4).contiguous().cpu().numpy()
    v = cache.value_codes.permute(0, 3, 1, 2, 4).contiguous().cpu().numpy()
    ks = cache.key_scale_pages.permute(0, 3, 1, 2).contiguous().cpu().numpy()
    vs = cache.value_scale_pages.permute(0, 3, 1, 2).contiguous().cpu().numpy()
    assert np.array_equal(k, oracle.keys) and np.array_equal(v, oracle.values)
    assert np.array_equal(ks.view(np.uint32), oracle.key_scales.view(np.uint32))
    assert np.array_equal(vs.view(np.uint32), oracle.value_scales.view(np.uint32))
