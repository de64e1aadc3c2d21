"""Pin the oracle to the reference: every restatement in oracle/ must
reproduce the fixtures that tests/golden/make_golden.py recorded by running
the reference's own Python package and C++ library."""

from __future__ import annotations

import json
import math

import numpy as np
import pytest

from oracle.attention import attention_fp64, attention_reference_torch
from oracle.paged_cache import PagedCacheOracle
from oracle.quant import (
    STATUS_INVALID_SIZE,
    STATUS_NONFINITE_VALUE,
    bits_f32,
    dequantize_vector,
    quantize_rows,
    quantize_vector,
)
from oracle.workloads import SMALL_SPECULATIVE, speculative_events, state_digest


@pytest.fixture(scope="module")
def kat(golden_dir):
    return json.loads((golden_dir / "kat_quant.json").read_text())


def test_reference_known_answers_are_in_the_fixture(kat):
    # test_kv_cache.py:31-41 and native_tests.cpp:135-156 of the reference
    vec = kat["vectors"]["reference_kat"]
    assert vec["codes"] == [-127, -64, 0, 64, 127]
    assert vec["scale"] == float(np.float32(1.0 / 127.0))
    # round half away from zero, not half to even
    assert kat["vectors"]["tie"]["codes"] == [127, 1, 2, 3, -3, -1]
    assert kat["vectors"]["tie"]["scale"] == 1.0
    assert kat["vectors"]["zero"]["scale"] == 0.0


def test_scalar_oracle_matches_every_reference_vector(kat):
    for name, case in kat["vectors"].items():
        codes, scale = quantize_vector(case["input"])
        assert list(codes) == case["codes"], name
        assert scale == case["scale"], name
        assert list(dequantize_vector(codes, scale)) == case["dequantized"], name


def test_c_oracle_matches_every_reference_vector(kat, oracle_c):
    for name, case in kat["vectors"].items():
        status, codes, scale = oracle_c.quantize(case["input"])
        assert status == 0, name
        assert list(codes) == case["codes"], name
        assert scale == case["scale"], name


def test_numpy_oracle_matches_reference_rows(kat):
    for name, case in kat["vectors"].items():
        codes, scales, status = quantize_rows(np.array([case["input"]], dtype=np.float64))
        assert status[0] == 0, name
        assert codes[0].tolist() == case["codes"], name
        assert float(scales[0]) == case["scale"], name


def test_error_statuses_match_reference(kat, oracle_c):
    expected = {name: e["status"] for name, e in kat["errors"].items()}
    assert expected == {"empty": STATUS_INVALID_SIZE, "nan": STATUS_NONFINITE_VALUE,
                        "inf": STATUS_NONFINITE_VALUE, "neg_inf": STATUS_NONFINITE_VALUE}
    assert oracle_c.quantize([])[0] == STATUS_INVALID_SIZE
    assert oracle_c.quantize([1.0, math.nan])[0] == STATUS_NONFINITE_VALUE
    assert oracle_c.quantize([math.inf, 1.0])[0] == STATUS_NONFINITE_VALUE
    _, _, status = quantize_rows(np.array([[1.0, math.nan], [0.0, 0.0]]))
    assert status.tolist() == [STATUS_NONFINITE_VALUE, 0]


def test_numpy_and_c_oracles_agree_on_random_rows(oracle_c):
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((2000, 64)) * rng.uniform(1e-3, 1e3, size=(2000, 1))).astype(np.float32)
    c_codes, c_scales, c_status = oracle_c.quantize_rows(x)
    n_codes, n_scales, n_status = quantize_rows(x.astype(np.float64))
    assert np.array_equal(c_codes, n_codes)
    assert np.array_equal(bits_f32(c_scales), bits_f32(n_scales))
    assert (c_status == 0).all() and (n_status == 0).all()


def test_cache_oracle_replays_reference_workload(golden_dir):
    golden = np.load(golden_dir / "small_speculative.npz")
    shape = SMALL_SPECULATIVE
    cache = PagedCacheOracle(shape.num_layers, shape.num_heads, shape.head_dim, shape.block_size,
                             shape.num_blocks)
    for s in range(shape.sequences):
        cache.create_sequence(s)
    for step, event in enumerate(speculative_events(shape, int(golden["seed"][0]))):
        if event[0] == "append":
            cache.append_many(event[1], event[2], event[3])
        else:
            cache.truncate(event[1], event[2])
        snap = golden["table_snapshots"][step]
        for s in range(shape.sequences):
            expected = [b for b in snap[s].tolist() if b >= 0]
            assert list(cache.block_table(s)) == expected, (step, s)
    assert np.array_equal(cache.keys, golden["keys"])
    assert np.array_equal(cache.values, golden["values"])
    assert np.array_equal(bits_f32(cache.key_scales), bits_f32(golden["key_scales"]))
    assert np.array_equal(bits_f32(cache.value_scales), bits_f32(golden["value_scales"]))
    assert [cache.sequence_length(s) for s in range(shape.sequences)] == golden["lengths"].tolist()
    st = cache.stats()
    assert [st.sequences, st.used_tokens, st.capacity_tokens, st.allocated_blocks, st.free_blocks,
            st.used_quantized_bytes, st.allocated_quantized_bytes, st.capacity_quantized_bytes,
            st.fp32_equivalent_bytes, st.block_table_bytes] == golden["stats"].tolist()
    digest = state_digest(cache.tables, cache.lengths, cache.keys, cache.values, cache.key_scales,
                          cache.value_scales)
    assert digest == "425e468e7eb5deb10bb5885748d4a9d0ab25431c50edd1fc0f13b2a3801ab66b"


def _attention_case(golden, index):
    p = f"case{index}_"
    hq, hkv, d, kw, T, bs, L, layer, nb = golden[p + "spec"].tolist()
    return dict(hq=hq, hkv=hkv, d=d, kw=kw, T=T, bs=bs, L=L, layer=layer, nb=nb,
                table=golden[p + "table"], keys=golden[p + "keys"], values=golden[p + "values"],
                ks=golden[p + "key_scales"], vs=golden[p + "value_scales"], q32=golden[p + "query_f32"],
                out_bf16=golden[p + "out_bf16"], out_f32=golden[p + "out_f32"])


def _gather(case):
    t = np.arange(case["T"])
    blocks = case["table"][t // case["bs"]]
    off = t % case["bs"]
    layer = case["layer"]
    return (case["keys"][blocks, off, layer], case["values"][blocks, off, layer],
            case["ks"][blocks, off, layer], case["vs"][blocks, off, layer])


def test_attention_oracles_match_reference_outputs(golden_dir):
    import torch

    golden = np.load(golden_dir / "attention_small.npz")
    for index in range(int(golden["num_cases"][0])):
        case = _attention_case(golden, index)
        exact = attention_fp64(case["q32"][0], *_gather(case))
        # fp32 reference SDPA vs exact arithmetic
        assert np.abs(case["out_f32"][0] - exact).max() < 1e-4, index
        # restated torch op reproduces the reference bit for bit on CPU
        args = [torch.from_numpy(case[k]) for k in ("keys", "values", "ks", "vs")]
        table = torch.from_numpy(case["table"])
        for name, dtype in (("bf16", torch.bfloat16), ("f32", torch.float32)):
            q = torch.from_numpy(case["q32"]).to(dtype)
            out = attention_reference_torch(q, *args, table, case["T"], case["layer"]).float().numpy()
            assert np.array_equal(out, case["out_" + name]), (index, name)
