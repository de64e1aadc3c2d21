"""Placement over ranks: request partitioning and KV-head tensor parallelism.

The tensor-parallel test runs two gloo ranks on the CPU; each computes its
head shard of the attention with the float64 oracle and the all-gather must
rebuild exactly the unsharded result.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from specdecode_b200.sharding import HeadShard, TensorParallelVerifyAttention, head_shard, lpt_partition


def test_lpt_partition_is_balanced_and_complete():
    rng = np.random.default_rng(3)
    lengths = rng.integers(1024, 8193, size=37).tolist()
    for world in (1, 2, 4, 8):
        parts = lpt_partition(lengths, world)
        assert sorted(i for p in parts for i in p) == list(range(len(lengths)))
        loads = [sum(lengths[i] for i in p) for p in parts]
        # LPT bound: no rank exceeds the mean by more than the longest job
        assert max(loads) - sum(loads) / world <= max(lengths)
        assert parts == lpt_partition(lengths, world)


def test_lpt_partition_small_cases():
    assert lpt_partition([5, 1, 4], 2) == [[0], [1, 2]]
    assert lpt_partition([], 3) == [[], [], []]
    with pytest.raises(ValueError):
        lpt_partition([1], 0)


def test_head_shard_ranges_and_validation():
    s = head_shard(1, 4, 8, 64)
    assert isinstance(s, HeadShard)
    assert list(s.kv_range) == [2, 3] and list(s.q_range) == list(range(16, 32))
    # query heads of the shard read exactly the shard's KV heads
    group = 64 // 8
    assert {h // group for h in s.q_range} == set(s.kv_range)
    with pytest.raises(ValueError):
        head_shard(0, 3, 8, 64)
    with pytest.raises(ValueError):
        head_shard(4, 4, 8, 64)


def _free_port() -> int:
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _tp_rank(rank: int, world: int, port: int, out_dir: str) -> None:
    import torch
    import torch.distributed as dist

    from oracle.attention import attention_fp64

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(11)
        B, Hq, Hkv, D, kw = 3, 16, 4, 32, 3
        lens = [40, 7, 65]
        k_codes = [rng.integers(-127, 128, size=(T, Hkv, D)).astype(np.int8) for T in lens]
        v_codes = [rng.integers(-127, 128, size=(T, Hkv, D)).astype(np.int8) for T in lens]
        k_sc = [rng.uniform(0.005, 0.05, size=(T, Hkv)).astype(np.float32) for T in lens]
        v_sc = [rng.uniform(0.005, 0.05, size=(T, Hkv)).astype(np.float32) for T in lens]
        q = rng.standard_normal((B, Hq, kw, D))
        shard = head_shard(rank, world, Hkv, Hq)
        kv = slice(shard.kv_range.start, shard.kv_range.stop)

        def local_attention(query_shard, tables, context_lens, max_len, layer):
            out = [attention_fp64(query_shard[b].numpy(), k_codes[b][:, kv], v_codes[b][:, kv], k_sc[b][:, kv],
                                  v_sc[b][:, kv]) for b in range(B)]
            return torch.from_numpy(np.stack(out))

        tp = TensorParallelVerifyAttention(local_attention, shard)
        full = tp(torch.from_numpy(q), None, None, max(lens), 0).numpy()
        want = np.stack([attention_fp64(q[b], k_codes[b], v_codes[b], k_sc[b], v_sc[b]) for b in range(B)])
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), np.array([np.abs(full - want).max()]))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_heads_gather_to_the_unsharded_result(tmp_path):
    import torch.multiprocessing as mp

    world = 2
    mp.spawn(_tp_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for rank in range(world):
        assert float(np.load(tmp_path / f"rank{rank}.npy")[0]) == 0.0
