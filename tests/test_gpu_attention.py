"""Fused paged verify attention against the oracle and the reference outputs.

Tolerances: for caches quantized from N(0,1) data (the benchmark
distribution) the output must be within max-abs 2e-2 and mean-abs 2e-3 of
the reference's dequantize-then-SDPA computation in bf16; against exact
float64 arithmetic on the same bf16 query it must be within one bf16
rounding of the exact value plus 2e-3 (|out - exact| <= 2^-8 |exact| + 2e-3).
For the reference fixture's uniformly random codes (values up to ~6) the
bounds scale with the largest dequantized value."""

from __future__ import annotations

import numpy as np
import pytest

from gpu_helpers import gather_oracle, load_logical, make_cache, random_pool, tables_tensor
from oracle.attention import attention_fp64, attention_reference_torch_flat

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def assert_near_exact(out, exact, label, scale=1.0):
    bound = 2.0 ** -8 * np.abs(exact) + 2e-3 * scale
    excess = np.abs(out - exact) - bound
    assert excess.max() <= 0, (label, float(np.abs(out - exact).max()))


def _attention(cache):
    from specdecode_b200.cuda_kv_cache import PagedVerifyAttention

    return PagedVerifyAttention.for_cache(cache)


def run_case(device, keys, values, ks, vs, tables, lens, q, layer, qdtype="bfloat16"):
    import torch

    nb, bs, L, H, D = keys.shape
    cache = make_cache(device, L, H, D, bs, nb)
    load_logical(cache, keys, values, ks, vs)
    qt = torch.from_numpy(q).to(getattr(torch, qdtype)).to(device)
    out = _attention(cache)(qt, tables_tensor(tables, device), torch.tensor(lens, dtype=torch.int32, device=device),
                            max(lens), layer)
    torch.cuda.synchronize()
    assert cache.status_bits() == 0
    return out.float().cpu().numpy(), qt.float().cpu().numpy()


def test_reference_fixture_cases(device, golden_dir):
    golden = np.load(golden_dir / "attention_small.npz")
    for index in range(int(golden["num_cases"][0])):
        p = f"case{index}_"
        hq, hkv, d, kw, T, bs, L, layer, nb = golden[p + "spec"].tolist()
        if d % 16:
            continue
        keys, values = golden[p + "keys"], golden[p + "values"]
        ks, vs = golden[p + "key_scales"], golden[p + "value_scales"]
        table = golden[p + "table"]
        out, q_used = run_case(device, keys, values, ks, vs, [table], [T], golden[p + "query_f32"], layer)
        gathered = gather_oracle(keys, values, ks, vs, table, T, bs, layer)
        exact = attention_fp64(q_used[0], *gathered)
        vmax = float(np.abs(values.astype(np.float64) * vs[..., None]).max())
        assert_near_exact(out[0], exact, index, vmax)
        ref = golden[p + "out_bf16"][0]
        assert np.abs(out[0] - ref).max() < MAX_ABS * vmax, index
        assert np.abs(out[0] - ref).mean() < MEAN_ABS * vmax, index


def _normal_pool(rng, nb, bs, L, H, D):
    """Pool quantized (per the reference rule) from N(0,1) K/V."""
    from oracle.quant import quantize_rows

    k = rng.standard_normal((nb, bs, L, H, D))
    v = rng.standard_normal((nb, bs, L, H, D))
    kq, ks, _ = quantize_rows(k)
    vq, vs, _ = quantize_rows(v)
    return kq, vq, ks, vs


CASES = [
    # (Hq, Hkv, D, window, bs, L, layer, lens)
    (32, 8, 128, 5, 16, 1, 0, [1024, 3000, 5, 17, 512, 513]),
    (8, 8, 64, 1, 16, 2, 1, [1, 2, 33, 700]),
    (16, 2, 128, 3, 8, 1, 0, [3, 8, 9, 1023, 1025]),
    (64, 8, 128, 5, 16, 1, 0, [5, 129, 2048]),
    (4, 1, 256, 8, 32, 1, 0, [8, 40, 600]),
    (16, 4, 64, 5, 16, 3, 2, [100, 1537]),
    # more than 32 query rows per KV head: split over two items per chunk
    (64, 8, 128, 8, 16, 1, 0, [8, 300, 4100]),
    (24, 8, 128, 11, 16, 2, 1, [11, 777, 2500]),
    # at least two (sequence, KV head) items per SM: one chunk per sequence,
    # the items write the output rows themselves (no combine launch).  The
    # shortest contexts (a row seeing one key, whose output is a raw value up
    # to ~4, where one bf16 step is 0.03) are left to the cases above: there
    # two independent bf16 roundings can differ by more than the 2e-2 bound
    (32, 8, 128, 5, 16, 1, 0, [40 + 37 * i for i in range(40)]),
    (16, 8, 64, 1, 16, 1, 0, [40 + 29 * i for i in range(40)]),
]


@pytest.mark.parametrize("case", CASES, ids=[f"hq{c[0]}-hkv{c[1]}-d{c[2]}-w{c[3]}-bs{c[4]}" for c in CASES])
def test_matches_oracle_and_reference_computation(device, case):
    import torch

    hq, hkv, d, kw, bs, L, layer, lens = case
    rng = np.random.default_rng(100 + CASES.index(case))
    blocks = [(t + bs - 1) // bs for t in lens]
    nb = sum(blocks) + 3
    keys, values, ks, vs = _normal_pool(rng, nb, bs, L, hkv, d)
    perm = rng.permutation(nb)
    tables, at = [], 0
    for n in blocks:
        tables.append(perm[at:at + n])
        at += n
    q = rng.standard_normal((len(lens), hq, kw, d)).astype(np.float32)
    out, q_used = run_case(device, keys, values, ks, vs, tables, lens, q, layer)
    for b, T in enumerate(lens):
        gathered = gather_oracle(keys, values, ks, vs, tables[b], T, bs, layer)
        exact = attention_fp64(q_used[b], *gathered)
        assert_near_exact(out[b], exact, (b, T))
        ref = attention_reference_torch_flat(
            torch.from_numpy(q_used[b]).to(torch.bfloat16), *[torch.from_numpy(x) for x in gathered]
        ).float().numpy()
        err = np.abs(out[b] - ref)
        assert err.max() < MAX_ABS and err.mean() < MEAN_ABS, (b, T)


@pytest.mark.parametrize("qdtype", ["float16", "float32"])
def test_other_query_dtypes(device, qdtype):
    rng = np.random.default_rng(4)
    keys, values, ks, vs = _normal_pool(rng, 40, 16, 1, 4, 128)
    tables = [rng.permutation(40)[:20]]
    q = rng.standard_normal((1, 16, 5, 128)).astype(np.float32)
    out, q_used = run_case(device, keys, values, ks, vs, tables, [317], q, 0, qdtype=qdtype)
    exact = attention_fp64(q_used[0], *gather_oracle(keys, values, ks, vs, tables[0], 317, 16, 0))
    assert_near_exact(out[0], exact, qdtype)


def test_full_verify_shape_subset_and_properties(device):
    """8B verify shape (32 sequences, contexts U[1024, 8192], window 5):
    four sequences against float64, all sequences against the unfused
    reference computation run with torch on the device."""
    import torch

    from oracle.workloads import VERIFY_8B, verify_inputs

    shape = VERIFY_8B
    lens, tables, nb, q = verify_inputs(shape, seed=2024)
    gen = torch.Generator(device=device).manual_seed(7)
    cache = make_cache(device, 1, shape.kv_heads, shape.head_dim, shape.block_size, nb)
    # fill the pool with codes quantized from N(0,1) by the append kernel
    k = torch.randn((nb * shape.block_size, 1, shape.kv_heads, shape.head_dim), generator=gen, device=device)
    v = torch.randn((nb * shape.block_size, 1, shape.kv_heads, shape.head_dim), generator=gen, device=device)
    cache.create_sequence("fill")
    cache.append_tensor("fill", k, v)
    qt = torch.from_numpy(q).to(torch.bfloat16).to(device)
    tt = tables_tensor(tables, device)
    lt = torch.tensor(lens, dtype=torch.int32, device=device)
    out = _attention(cache)(qt, tt, lt, int(lens.max()), 0).float()
    torch.cuda.synchronize()
    assert cache.status_bits() == 0
    keys_v = cache.keys_view[:, :, 0]
    vals_v = cache.values_view[:, :, 0]
    ks_v = cache.key_scales_view[:, :, 0]
    vs_v = cache.value_scales_view[:, :, 0]
    worst_max, worst_mean = 0.0, 0.0
    for b in range(shape.batch):
        T = int(lens[b])
        t = torch.arange(T, device=device)
        blk = torch.from_numpy(tables[b]).to(device)[t // shape.block_size]
        off = t % shape.block_size
        gk, gv, gks, gvs = keys_v[blk, off], vals_v[blk, off], ks_v[blk, off], vs_v[blk, off]
        ref = attention_reference_torch_flat(qt[b], gk, gv, gks, gvs).float()
        err = (out[b] - ref).abs()
        worst_max = max(worst_max, float(err.max()))
        worst_mean = max(worst_mean, float(err.mean()))
        if b < 4:
            exact = attention_fp64(qt[b].float().cpu().numpy(), gk.cpu().numpy(), gv.cpu().numpy(),
                                   gks.cpu().numpy(), gvs.cpu().numpy())
            assert_near_exact(out[b].cpu().numpy(), exact, b)
    assert worst_max < MAX_ABS and worst_mean < MEAN_ABS
    # physical placement does not matter: relabel the pool, same answer
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(1)).to(device)
    inverse = torch.empty_like(perm)
    inverse[perm] = torch.arange(nb, device=device)
    for t in (cache.key_codes, cache.value_codes, cache.key_scale_pages, cache.value_scale_pages):
        t.copy_(t[inverse])
    tt2 = perm[tt.long().clamp(min=0)].to(torch.int32).masked_fill(tt < 0, -1)
    out2 = _attention(cache)(qt, tt2, lt, int(lens.max()), 0).float()
    assert torch.equal(out, out2)


def test_long_context_70b_shape(device):
    """Llama-3.1-70B long-context verify (8 sequences x 131072 tokens, 64
    query / 8 KV heads, window 5: 40 query rows per KV head, served as two
    20-row splits) against the unfused reference computation run with torch
    on the device, every sequence."""
    import torch

    from oracle.workloads import VERIFY_70B, verify_inputs

    shape = VERIFY_70B
    lens, tables, nb, q = verify_inputs(shape, seed=77)
    gen = torch.Generator(device=device).manual_seed(70)
    cache = make_cache(device, 1, shape.kv_heads, shape.head_dim, shape.block_size, nb)
    cache.create_sequence("fill")
    step = 1 << 16
    for start in range(0, nb * shape.block_size, step):
        n = min(step, nb * shape.block_size - start)
        k = torch.randn((n, 1, shape.kv_heads, shape.head_dim), generator=gen, device=device, dtype=torch.bfloat16)
        v = torch.randn((n, 1, shape.kv_heads, shape.head_dim), generator=gen, device=device, dtype=torch.bfloat16)
        cache.append_tensor("fill", k, v)
    qt = torch.from_numpy(q).to(torch.bfloat16).to(device)
    tt = tables_tensor(tables, device)
    lt = torch.tensor(lens, dtype=torch.int32, device=device)
    out = _attention(cache)(qt, tt, lt, int(lens.max()), 0).float()
    torch.cuda.synchronize()
    assert cache.status_bits() == 0
    keys_v, vals_v = cache.keys_view[:, :, 0], cache.values_view[:, :, 0]
    ks_v, vs_v = cache.key_scales_view[:, :, 0], cache.value_scales_view[:, :, 0]
    for b in range(shape.batch):
        T = int(lens[b])
        t = torch.arange(T, device=device)
        blk = torch.from_numpy(tables[b]).to(device)[t // shape.block_size]
        off = t % shape.block_size
        ref = attention_reference_torch_flat(qt[b], keys_v[blk, off], vals_v[blk, off], ks_v[blk, off],
                                             vs_v[blk, off]).float()
        err = (out[b] - ref).abs()
        assert float(err.max()) < MAX_ABS and float(err.mean()) < MEAN_ABS, (b, float(err.max()))


def test_faults_are_reported_not_trapped(device):
    import torch

    from specdecode_b200 import _lib

    rng = np.random.default_rng(0)
    keys, values, ks, vs = random_pool(rng, 8, 16, 1, 2, 64)
    cache = make_cache(device, 1, 2, 64, 16, 8, check_status=False)
    load_logical(cache, keys, values, ks, vs)
    q = torch.randn((2, 4, 5, 64), device=device).to(torch.bfloat16)
    tables = tables_tensor([[0, 1], [2, 99]], device)  # block 99 is outside the pool
    lens = torch.tensor([3, 20], dtype=torch.int32, device=device)  # 3 < window 5
    out = _attention(cache)(q, tables, lens, 20, 0)
    torch.cuda.synchronize()
    bits = cache.status_bits()
    assert bits & _lib.FAULT_CONTEXT_RANGE and bits & _lib.FAULT_BLOCK_RANGE
    assert torch.count_nonzero(out[0]) == 0


@pytest.mark.parametrize("hq,window,d", [(32, 5, 128), (32, 5, 64), (48, 4, 128)],
                         ids=["rows20_d128", "rows20_d64", "rows24_d128"])
def test_pipeline_wait_gives_up_and_reports(device, hq, window, d):
    """The item kernel's bounded waits: with the test hook, the softmax warps
    wait on a barrier that nothing completes, so the wait gives up after the
    limit.  The launch reports SDC_FAULT_WAIT_TIMEOUT in the status word,
    writes no output row and returns (its copies and MMAs drained, tensor
    memory freed), and the next launch in the same context is correct.
    Covers the three-warpgroup kernel (20 rows per KV head, head_dim 128 and
    64) and the two-warpgroup one (24 rows)."""
    import torch

    from specdecode_b200 import _lib

    rng = np.random.default_rng(77)
    hkv, bs, T, nb = 8, 16, 100, 8
    keys, values, ks, vs = random_pool(rng, nb, bs, 1, hkv, d)
    cache = make_cache(device, 1, hkv, d, bs, nb)
    load_logical(cache, keys, values, ks, vs)
    table = rng.permutation(nb)[: (T + bs - 1) // bs].tolist()
    q = torch.from_numpy(rng.standard_normal((1, hq, window, d)).astype(np.float32)).to(torch.bfloat16).to(device)
    tables = tables_tensor([table], device)
    lens = torch.tensor([T], dtype=torch.int32, device=device)
    attention = _attention(cache)
    hooks = cache.library.handle.sdc_test_attention_waits
    out = torch.zeros_like(q)
    assert hooks(1 << 20, 1) == 0  # about half a millisecond
    try:
        attention(q, tables, lens, T, 0, out=out)
        torch.cuda.synchronize()
    finally:
        assert hooks(0, 0) == 0
    assert cache.status_bits() == _lib.FAULT_WAIT_TIMEOUT
    assert int(torch.count_nonzero(out)) == 0
    again = attention(q, tables, lens, T, 0)
    torch.cuda.synchronize()
    assert cache.status_bits() == 0
    exact = attention_fp64(q[0].float().cpu().numpy(), *gather_oracle(keys, values, ks, vs, table, T, bs, 0))
    assert_near_exact(again[0].float().cpu().numpy(), exact, "after a timed-out launch", scale=3.0)


def test_bad_output_or_device_is_refused_before_launch(device):
    """An output buffer of another shape or dtype, or inputs left on the
    host, raise before anything is launched (the kernel would otherwise write
    past the buffer or read host addresses)."""
    import torch

    from specdecode_b200.cuda_kv_cache import CudaPagedAttentionError

    rng = np.random.default_rng(3)
    keys, values, ks, vs = random_pool(rng, 8, 16, 1, 8, 128)
    cache = make_cache(device, 1, 8, 128, 16, 8)
    load_logical(cache, keys, values, ks, vs)
    q = torch.randn((1, 32, 5, 128), device=device).to(torch.bfloat16)
    tables = tables_tensor([[0, 1, 2]], device)
    lens = torch.tensor([40], dtype=torch.int32, device=device)
    attention = _attention(cache)
    for bad in (torch.empty((1, 32, 4, 128), dtype=torch.bfloat16, device=device),
                torch.empty((1, 32, 5, 128), dtype=torch.float32, device=device),
                torch.empty((1, 32, 5, 128), dtype=torch.bfloat16)):
        with pytest.raises(CudaPagedAttentionError):
            attention(q, tables, lens, 40, 0, out=bad)
    with pytest.raises(CudaPagedAttentionError):
        attention(q, tables.cpu(), lens, 40, 0)
    torch.cuda.synchronize()
    assert cache.status_bits() == 0
    out = attention(q, tables, lens, 40, 0)
    torch.cuda.synchronize()
    assert cache.status_bits() == 0 and out.shape == q.shape
