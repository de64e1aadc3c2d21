"""The no-allocation attention entry point against the regular one.

sdc_paged_verify_attention_no_alloc serves callers that may not allocate
device memory (a serving loop whose memory another allocator reserved up
front, a plugin host that hands over only its inputs and outputs, a callback
that must not synchronize the device the way cudaMalloc / cudaFree can): its
workspace is a fixed 16 MiB device array inside the library.  Two calls in a
row, with different shapes and layers so the second one runs over whatever
the first left in that array, must equal sdc_paged_verify_attention (which
uses a caller workspace) bit for bit: both run the same deterministic
kernels on the same inputs, and only the workspace's address differs.  A
shape whose workspace exceeds the array is refused before anything is
launched.

This file sorts last so that a run stopping at its first failure has already
run every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from gpu_helpers import load_logical, make_cache, tables_tensor

pytestmark = pytest.mark.gpu

BS, L, HKV, HQ, D, WINDOW = 16, 2, 8, 32, 128, 5


def _pool(rng, nb):
    """Codes and scales quantized (by the reference rule) from N(0,1) K/V."""
    from oracle.quant import quantize_rows

    k = rng.standard_normal((nb, BS, L, HKV, D))
    v = rng.standard_normal((nb, BS, L, HKV, D))
    kq, ks, _ = quantize_rows(k)
    vq, vs, _ = quantize_rows(v)
    return kq, vq, ks, vs


def _no_alloc(cache, query, tables, lens, max_len, layer, out):
    import torch

    from specdecode_b200.kv_cache import _dtype_code

    lib = cache.library
    status = lib.handle.sdc_paged_verify_attention_no_alloc(
        ctypes.byref(cache.pool_desc), int(layer), query.data_ptr(), _dtype_code(query.dtype), query.shape[0],
        query.shape[1], query.shape[2], tables.data_ptr(), tables.stride(0), lens.data_ptr(), int(max_len),
        out.data_ptr(), cache._status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return status


def test_no_alloc_matches_workspace_entry_point(device):
    import torch

    from specdecode_b200.cuda_kv_cache import PagedVerifyAttention

    rng = np.random.default_rng(2031)
    lens_all = [1500, 333, 2048, 777, 1024, 96]
    nb = sum((t + BS - 1) // BS for t in lens_all) + 8
    keys, values, ks, vs = _pool(rng, nb)
    cache = make_cache(device, L, HKV, D, BS, nb)
    load_logical(cache, keys, values, ks, vs)
    order = rng.permutation(nb)
    tables, start = [], 0
    for t in lens_all:
        n = (t + BS - 1) // BS
        tables.append(order[start:start + n].tolist())
        start += n
    regular = PagedVerifyAttention.for_cache(cache)

    # two calls in a row: different batch, context lengths and layer
    for batch, layer in ((len(lens_all), 0), (3, 1)):
        lens = lens_all[:batch]
        tt = tables_tensor(tables[:batch], device)
        lt = torch.tensor(lens, dtype=torch.int32, device=device)
        q = torch.from_numpy(rng.standard_normal((batch, HQ, WINDOW, D))).to(torch.bfloat16).to(device)
        want = regular(q, tt, lt, max(lens), layer)
        got = torch.full_like(q, float("nan"))
        status = _no_alloc(cache, q, tt, lt, max(lens), layer, got)
        torch.cuda.synchronize()
        assert status == 0, cache.library.status_string(status)
        assert cache.status_bits() == 0
        assert torch.isfinite(got.float()).all()
        assert torch.equal(got, want), (batch, layer, float((got.float() - want.float()).abs().max()))


def test_no_alloc_refuses_shapes_beyond_its_scratch(device):
    import torch

    from specdecode_b200 import _lib

    cache = make_cache(device, 1, HKV, D, BS, 4)
    batch, max_len = 512, 4096  # partial slots for 4096 KV heads: about 40 MiB
    need = ctypes.c_size_t()
    assert cache.library.handle.sdc_paged_attention_workspace_size(batch, HQ, HKV, D, WINDOW, max_len,
                                                                   ctypes.byref(need)) == 0
    assert need.value > 16 << 20
    q = torch.zeros((batch, HQ, WINDOW, D), dtype=torch.bfloat16, device=device)
    tt = torch.zeros((batch, 1), dtype=torch.int32, device=device)
    lt = torch.full((batch,), WINDOW, dtype=torch.int32, device=device)
    out = torch.empty_like(q)
    status = _no_alloc(cache, q, tt, lt, max_len, 0, out)
    assert status == _lib.STATUS_SCRATCH_EXCEEDED
    assert "scratch" in cache.library.status_string(status)
