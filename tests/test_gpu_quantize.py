"""Quantizer kernels against the oracle: bit-exact codes and scale bits."""

from __future__ import annotations

import json
import math

import numpy as np
import pytest

from oracle.quant import bits_f32, quantize_rows

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def native():
    from specdecode_b200.native import NativeKVQuantizer

    return NativeKVQuantizer.load()


def test_per_vector_abi_matches_reference_fixture(device, native, golden_dir):
    kat = json.loads((golden_dir / "kat_quant.json").read_text())
    for name, case in kat["vectors"].items():
        q = native.quantize(case["input"])
        assert list(q.values) == case["codes"], name
        assert q.scale == case["scale"], name
        assert list(native.dequantize(q)) == case["dequantized"], name


def test_per_vector_abi_errors(device, native):
    from specdecode_b200.native import NativeBackendError

    with pytest.raises(NativeBackendError) as info:
        native.quantize(())
    assert info.value.status == 2
    with pytest.raises(NativeBackendError) as info:
        native.quantize((1.0, math.nan))
    assert info.value.status == 3
    with pytest.raises(NativeBackendError) as info:
        native.quantize((math.inf,))
    assert info.value.status == 3
    with pytest.raises(TypeError):
        native.quantize((True,))


def _tie_rows(rng, n_rows, width):
    rows = []
    for _ in range(n_rows):
        s = np.float32(rng.uniform(1e-3, 10.0))
        m = np.float32(127.0) * s
        s = np.float32(np.float64(m) / 127.0)
        ks = rng.integers(-127, 127, size=width - 1)
        vals = [(k + 0.5) * np.float64(s) for k in ks]
        # exact ties, and their float32 neighbours on both sides
        vals = [np.float32(v) for v in vals]
        vals = [np.nextafter(v, np.float32(np.inf)) if i % 3 == 1 else
                np.nextafter(v, np.float32(-np.inf)) if i % 3 == 2 else v for i, v in enumerate(vals)]
        rows.append([np.float32(m)] + vals)
    return np.array(rows, dtype=np.float32)


@pytest.mark.parametrize("dtype_name", ["float32", "bfloat16", "float16", "float64"])
def test_batched_rows_bit_exact(device, native, dtype_name):
    import torch

    dtype = getattr(torch, dtype_name)
    rng = np.random.default_rng(17)
    parts = [
        rng.standard_normal((4000, 128)) * rng.uniform(1e-3, 1e3, size=(4000, 1)),
        rng.standard_normal((200, 128)) * 1e-36,       # scales below 2^-100: double path
        rng.standard_normal((200, 128)) * 1e37,
        np.zeros((10, 128)),
        _tie_rows(rng, 500, 128).astype(np.float64),
    ]
    if dtype_name == "float16":
        parts[1] = parts[1] * 1e32  # keep inside fp16's range
        parts[2] = parts[2] * 1e-33
    x = np.concatenate(parts).astype(np.float64)
    src = torch.from_numpy(x).to(dtype)
    exact = src.double().cpu().numpy()  # the values the kernel actually sees
    codes, scales, status = native.quantize_batch(src.to(device))
    ref_codes, ref_scales, ref_status = quantize_rows(exact)
    status = status.cpu().numpy()
    assert np.array_equal(status, ref_status)
    ok = ref_status == 0
    assert np.array_equal(codes.cpu().numpy()[ok], ref_codes[ok])
    assert np.array_equal(bits_f32(scales.cpu().numpy()[ok]), bits_f32(ref_scales[ok]))


def test_batched_rows_report_nonfinite(device, native):
    import torch

    x = torch.ones((4, 16), dtype=torch.float32)
    x[1, 3] = float("nan")
    x[2, 0] = float("inf")
    _, _, status = native.quantize_batch(x.to(device))
    assert status.cpu().tolist() == [0, 3, 3, 0]


def test_odd_lengths(device, native):
    import torch

    rng = np.random.default_rng(3)
    for count in (1, 3, 17, 33, 100, 1000):
        x = rng.standard_normal((7, count))
        codes, scales, status = native.quantize_batch(torch.from_numpy(x).to(device))
        ref_codes, ref_scales, _ = quantize_rows(x)
        assert (status.cpu().numpy() == 0).all()
        assert np.array_equal(codes.cpu().numpy(), ref_codes)
        assert np.array_equal(bits_f32(scales.cpu().numpy()), bits_f32(ref_scales))
