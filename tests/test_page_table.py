"""Host page-table bookkeeping against the reference semantics (CPU only).

Mirrors the block-table, rollback, isolation and accounting cases of the
reference's tests/test_kv_cache.py:61-208 and replays seeded speculative
workloads against the oracle's restatement of PagedKVCache."""

from __future__ import annotations

import numpy as np
import pytest

from oracle.paged_cache import OracleCapacityError, PagedCacheOracle
from oracle.workloads import SMALL_SPECULATIVE, speculative_events
from specdecode_b200.page_table import KVCacheCapacityError, PageTable


def test_block_table_and_physical_slots():  # test_kv_cache.py:81-92
    pages = PageTable(num_blocks=4, block_size=2)
    pages.create_sequence("request-a")
    plan = pages.plan_append(["request-a"], [3])
    assert plan.slots.tolist() == [0, 1, 2]
    assert pages.block_table("request-a") == (0, 1)
    assert pages.physical_slot("request-a", 2) == (1, 0)
    pages.validate_invariants()


def test_rollback_releases_suffix_and_reuses_slot():  # test_kv_cache.py:150-168
    pages = PageTable(num_blocks=4, block_size=2)
    pages.create_sequence("a")
    pages.plan_append(["a"], [3])
    pages.plan_append(["a"], [3])
    plan = pages.plan_truncate(["a"], [3])
    assert plan.released.tolist() == [1]
    assert sorted(plan.cleared_slots.tolist()) == [3, 4, 5]
    assert pages.block_table("a") == (0, 1)
    again = pages.plan_append(["a"], [1])
    assert again.slots.tolist() == [3]
    assert pages.physical_slot("a", 3) == (1, 1)
    pages.validate_invariants()


def test_isolation_and_lowest_id_reuse():  # test_kv_cache.py:177-190
    pages = PageTable(num_blocks=4, block_size=2)
    for s in ("a", "b"):
        pages.create_sequence(s)
    pages.plan_append(["a"], [1])
    pages.plan_append(["b"], [1])
    assert pages.block_table("a") == (0,) and pages.block_table("b") == (1,)
    pages.plan_truncate(["a"], [0])
    pages.drop_sequence("a")
    pages.create_sequence("c")
    pages.plan_append(["c"], [1])
    assert pages.block_table("c") == (0,)
    pages.validate_invariants()


def test_capacity_failure_leaves_state_untouched():  # test_kv_cache.py:135-148
    pages = PageTable(num_blocks=1, block_size=2)
    pages.create_sequence("limited")
    with pytest.raises(KVCacheCapacityError):
        pages.plan_append(["limited"], [3])
    assert pages.sequence_length("limited") == 0
    assert pages.free_blocks() == 1
    pages.validate_invariants()


def test_errors_follow_reference_types():
    pages = PageTable(num_blocks=4, block_size=2)
    pages.create_sequence("a")
    with pytest.raises(ValueError):
        pages.create_sequence("a")
    with pytest.raises(KeyError):
        pages.sequence_length("missing")
    with pytest.raises(TypeError):
        pages.create_sequence(["unhashable"])
    with pytest.raises(TypeError):
        pages.plan_truncate(["a"], [True])
    with pytest.raises(ValueError):
        pages.plan_truncate(["a"], [1])
    with pytest.raises(IndexError):
        pages.physical_slot("a", 0)


def test_undo_append_restores_everything():
    pages = PageTable(num_blocks=8, block_size=2)
    pages.create_sequence("a")
    pages.plan_append(["a"], [3])
    before = (pages.block_table("a"), pages.sequence_length("a"), pages.free.copy(), pages.occupied.copy())
    plan = pages.plan_append(["a"], [4])
    pages.undo_append(plan)
    assert (pages.block_table("a"), pages.sequence_length("a")) == before[:2]
    assert np.array_equal(pages.free, before[2]) and np.array_equal(pages.occupied, before[3])
    pages.validate_invariants()


def test_invariant_audit_detects_corruption():
    pages = PageTable(num_blocks=4, block_size=2)
    pages.create_sequence("a")
    pages.plan_append(["a"], [2])
    pages.free[0] = True  # block 0 both allocated and free
    with pytest.raises(AssertionError):
        pages.validate_invariants()


@pytest.mark.parametrize("relabel", [False, True])
def test_speculative_workload_tables_match_oracle(relabel):
    shape = SMALL_SPECULATIVE
    order = np.random.default_rng(3).permutation(shape.num_blocks) if relabel else None
    pages = PageTable(shape.num_blocks, shape.block_size, block_order=order)
    oracle = PagedCacheOracle(shape.num_layers, shape.num_heads, shape.head_dim, shape.block_size,
                              shape.num_blocks, block_order=order, use_c=False)
    for s in range(shape.sequences):
        pages.create_sequence(s)
        oracle.create_sequence(s)
    for event in speculative_events(shape, 21):
        if event[0] == "append":
            n = event[2].shape[0]
            plan = pages.plan_append([event[1]], [n])
            start = oracle.sequence_length(event[1])
            oracle.append_many(event[1], event[2], event[3])
            expected = [oracle.physical_slot(event[1], t) for t in range(start, start + n)]
            assert plan.slots.tolist() == [b * shape.block_size + o for b, o in expected]
        else:
            released = pages.plan_truncate([event[1]], [event[2]]).released.tolist()
            assert released == [oracle.truncate(event[1], event[2])]
        for s in range(shape.sequences):
            assert pages.block_table(s) == oracle.block_table(s)
        pages.validate_invariants()
    assert pages.free_blocks() == oracle.free_blocks()


def test_batched_plans_equal_sequential_plans():
    rng = np.random.default_rng(8)
    batched = PageTable(num_blocks=200, block_size=4)
    sequential = PageTable(num_blocks=200, block_size=4)
    seqs = list(range(10))
    for s in seqs:
        batched.create_sequence(s)
        sequential.create_sequence(s)
    for _ in range(20):
        plan = batched.plan_append(seqs, [5] * len(seqs))
        slots = np.concatenate([sequential.plan_append([s], [5]).slots for s in seqs])
        assert np.array_equal(plan.slots, slots)
        keep = rng.integers(0, 6, size=len(seqs))
        counts = [sequential.sequence_length(s) - 5 + int(k) for s, k in zip(seqs, keep)]
        tplan = batched.plan_truncate(seqs, counts)
        cleared = np.concatenate([sequential.plan_truncate([s], [c]).cleared_slots for s, c in zip(seqs, counts)])
        assert np.array_equal(np.sort(tplan.cleared_slots), np.sort(cleared))
        for s in seqs:
            assert batched.block_table(s) == sequential.block_table(s)
    batched.validate_invariants()


def test_batched_capacity_error_is_atomic():
    pages = PageTable(num_blocks=3, block_size=2)
    for s in ("a", "b"):
        pages.create_sequence(s)
    with pytest.raises(KVCacheCapacityError):
        pages.plan_append(["a", "b"], [4, 4])
    assert pages.free_blocks() == 3
    assert pages.sequence_length("a") == pages.sequence_length("b") == 0


def test_oracle_capacity_error_matches():
    oracle = PagedCacheOracle(1, 1, 16, 2, 1, use_c=False)
    oracle.create_sequence("x")
    with pytest.raises(OracleCapacityError):
        oracle.append_many("x", np.zeros((3, 1, 1, 16), np.float32), np.zeros((3, 1, 1, 16), np.float32))
