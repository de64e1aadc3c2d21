"""KV-head tensor-parallel verify attention with the all-gather fused into
the attention launch (``sdc_paged_verify_attention_gather``,
``sharding.PeerHeadGather``).

* Two ranks emulated on one GPU: rank 0's call, then rank 1's, each storing
  its heads' rows into both ranks' gathered buffers.  Rank 1's completion
  flag in rank 0's buffer is raised by the host beforehand (rank 1 has not
  run yet), so no launch ever waits on another launch of the same GPU.
  Afterwards both buffers hold the same bytes, every flag reads the epoch,
  and each sequence's rows are within the attention tolerance of exact
  float64 attention over all heads.  Covers the tensor-core kernel with its
  combine launch (40 rows per KV head), its direct-write path (one chunk
  per sequence) and the CUDA-core kernel (head_dim 256).
* A flag nothing raises: the completion wait gives up after the test limit
  and reports SDC_FAULT_WAIT_TIMEOUT, with this rank's rows already stored.
* Two processes on two GPUs (skipped with fewer): PeerHeadGather over real
  inter-process mappings, several calls (epochs), every rank's gathered
  output equal across ranks and within tolerance of exact attention.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest

from gpu_helpers import gather_oracle, load_logical, make_cache, random_pool, tables_tensor
from oracle.attention import attention_fp64

pytestmark = pytest.mark.gpu

CASES = {
    # name: (query heads, KV heads, head_dim, window, context lengths)
    "tc_combine": (64, 8, 128, 5, [2000, 3100, 500]),
    "tc_direct": (32, 8, 128, 2, [150 + 7 * i for i in range(80)]),
    "simt": (16, 4, 256, 3, [700, 90]),
}


def _shard_pool(keys, values, ks, vs, rank, world):
    H = keys.shape[3]
    hs = slice(rank * H // world, (rank + 1) * H // world)
    return keys[:, :, :, hs].copy(), values[:, :, :, hs].copy(), ks[:, :, :, hs].copy(), vs[:, :, :, hs].copy()


def _problem(seed, hq, hkv, d, window, lens, bs=16):
    rng = np.random.default_rng(seed)
    blocks = [(T + bs - 1) // bs for T in lens]
    nb = int(sum(blocks))
    keys, values, ks, vs = random_pool(rng, nb, bs, 1, hkv, d)
    perm = rng.permutation(nb)
    tables, at = [], 0
    for n in blocks:
        tables.append(perm[at:at + n].tolist())
        at += n
    q = rng.standard_normal((len(lens), hq, window, d)).astype(np.float32)
    return keys, values, ks, vs, tables, q


def _exact_rows(keys, values, ks, vs, tables, lens, qf, bs=16):
    return [attention_fp64(qf[b], *gather_oracle(keys, values, ks, vs, tables[b], T, bs, 0))
            for b, T in enumerate(lens)]


def _gather_call(cache, q_local, tables, lens, max_len, outs, flags, world, rank, epoch):
    import torch

    from specdecode_b200 import _lib

    lib = cache.library.handle
    B, hq, kw, D = (int(x) for x in q_local.shape)
    size = ctypes.c_size_t()
    assert lib.sdc_paged_attention_workspace_size(B, hq, cache.config.num_heads, D, kw, max_len,
                                                  ctypes.byref(size)) == 0
    ws = torch.empty(max(int(size.value), 256), dtype=torch.uint8, device=cache.device)
    out_arr = (ctypes.c_void_p * world)(*[o.data_ptr() for o in outs])
    flag_arr = (ctypes.c_void_p * world)(*[f.data_ptr() for f in flags])
    return lib.sdc_paged_verify_attention_gather(
        cache.pool_desc, 0, q_local.data_ptr(), _lib.DTYPE_BF16, B, hq, kw, tables.data_ptr(), tables.stride(0),
        lens.data_ptr(), max_len, out_arr, flag_arr, world, rank, epoch, ws.data_ptr(), ws.numel(),
        cache._status.data_ptr(), torch.cuda.current_stream(cache.device).cuda_stream)


@pytest.mark.parametrize("case", sorted(CASES))
def test_two_ranks_emulated_on_one_gpu(device, case):
    import torch

    hq, hkv, d, window, lens = CASES[case]
    world, bs = 2, 16
    keys, values, ks, vs, tables, q = _problem(11, hq, hkv, d, window, lens)
    qt = torch.from_numpy(q).to(torch.bfloat16).to(device)
    tab = tables_tensor(tables, device)
    ctx = torch.tensor(lens, dtype=torch.int32, device=device)
    outs = [torch.zeros_like(qt) for _ in range(world)]
    flags = [torch.zeros(world, dtype=torch.int32, device=device) for _ in range(world)]
    flags[0][1] = 1  # rank 1's completion, raised ahead: it runs after rank 0 here
    caches = []
    for rank in range(world):
        cache = make_cache(device, 1, hkv // world, d, bs, keys.shape[0])
        load_logical(cache, *_shard_pool(keys, values, ks, vs, rank, world))
        caches.append(cache)
        part = hq // world
        q_local = qt[:, rank * part:(rank + 1) * part].contiguous()
        assert _gather_call(cache, q_local, tab, ctx, max(lens), outs, flags, world, rank, 1) == 0
    torch.cuda.synchronize()
    assert [c.status_bits() for c in caches] == [0, 0]
    assert torch.equal(outs[0], outs[1])
    assert [f.tolist() for f in flags] == [[1, 1], [1, 1]]
    got = outs[0].float().cpu().numpy()
    exact = _exact_rows(keys, values, ks, vs, tables, lens, qt.float().cpu().numpy())
    for b in range(len(lens)):
        bound = 2.0 ** -8 * np.abs(exact[b]) + 6e-3
        assert (np.abs(got[b] - exact[b]) <= bound).all(), (case, b, float(np.abs(got[b] - exact[b]).max()))


def test_completion_wait_gives_up_and_reports(device):
    """Rank 0 of two, and rank 1 never signals: the completion launch waits
    out the test limit (about 8 ms), reports SDC_FAULT_WAIT_TIMEOUT and
    returns; rank 0's rows are in both buffers and its own flag is raised in
    both."""
    import torch

    from specdecode_b200 import _lib

    hq, hkv, d, window, lens = CASES["tc_combine"]
    world, bs = 2, 16
    keys, values, ks, vs, tables, q = _problem(12, hq, hkv, d, window, lens)
    qt = torch.from_numpy(q).to(torch.bfloat16).to(device)
    outs = [torch.zeros_like(qt) for _ in range(world)]
    flags = [torch.zeros(world, dtype=torch.int32, device=device) for _ in range(world)]
    cache = make_cache(device, 1, hkv // world, d, bs, keys.shape[0])
    load_logical(cache, *_shard_pool(keys, values, ks, vs, 0, world))
    hooks = cache.library.handle.sdc_test_attention_waits
    assert hooks(1 << 24, 0) == 0
    try:
        st = _gather_call(cache, qt[:, : hq // 2].contiguous(), tables_tensor(tables, device),
                          torch.tensor(lens, dtype=torch.int32, device=device), max(lens), outs, flags, world, 0, 7)
        torch.cuda.synchronize()
    finally:
        assert hooks(0, 0) == 0
    assert st == 0
    assert cache.status_bits() == _lib.FAULT_WAIT_TIMEOUT
    assert [f.tolist() for f in flags] == [[7, 0], [7, 0]]
    assert torch.equal(outs[0], outs[1])
    assert int(torch.count_nonzero(outs[0][:, : hq // 2])) > 0
    assert int(torch.count_nonzero(outs[0][:, hq // 2:])) == 0


def _two_process_worker(rank, world, port, result_dir):
    import torch
    import torch.distributed as dist

    from specdecode_b200.sharding import PeerHeadGather, head_shard

    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    hq, hkv, d, window, lens = CASES["tc_combine"]
    bs = 16
    keys, values, ks, vs, tables, _ = _problem(13, hq, hkv, d, window, lens)
    cache = make_cache(device, 1, hkv // world, d, bs, keys.shape[0])
    load_logical(cache, *_shard_pool(keys, values, ks, vs, rank, world))
    gather = PeerHeadGather(cache, head_shard(rank, world, hkv, hq), len(lens), window)
    tab = tables_tensor(tables, device)
    ctx = torch.tensor(lens, dtype=torch.int32, device=device)
    report = []
    for call in range(3):
        q = np.random.default_rng(100 + call).standard_normal((len(lens), hq, window, d)).astype(np.float32)
        qt = torch.from_numpy(q).to(torch.bfloat16).to(device)
        out = gather(qt, tab, ctx, max(lens), 0).float().cpu().numpy()
        exact = _exact_rows(keys, values, ks, vs, tables, lens, qt.float().cpu().numpy())
        worst = max(float((np.abs(out[b] - exact[b]) - 2.0 ** -8 * np.abs(exact[b])).max())
                    for b in range(len(lens)))
        report.append((worst, float(np.abs(out).sum())))
    bits = cache.status_bits()
    gather.close()
    dist.destroy_process_group()
    np.save(os.path.join(result_dir, f"rank{rank}.npy"), np.array([[bits, w, s] for w, s in report]))


def test_peer_gather_two_processes(tmp_path):
    import socket

    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_two_process_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.terminate()
            p.join(timeout=30)
    assert [p.exitcode for p in procs] == [0, 0]
    results = [np.load(tmp_path / f"rank{r}.npy") for r in range(2)]
    for res in results:
        assert (res[:, 0] == 0).all()  # no fault bits
        assert (res[:, 1] <= 6e-3).all()  # within tolerance of exact attention
    assert np.array_equal(results[0][:, 2], results[1][:, 2])  # both ranks hold the same gathered rows
