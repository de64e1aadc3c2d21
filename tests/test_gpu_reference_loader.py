"""The reference's own native-library consumers, unchanged (from the copy of
its package in oracle/_ref/), running on libspecdecode_cuda.so's sd_* entry
points, which compute on the GPU:

* NativeKVQuantizer.load(<this library>) quantizes and dequantizes the 80
  known-answer vectors exactly as recorded from the reference;
* NativeSamplingBackend.load(<this library>) gives, on every seeded case of
  tests/sampling_cases.py, the sampled indices and first rejections the
  reference's own library gives, acceptance probabilities within 2 ulp and
  normalised / residual rows within 1e-15 of them, and the reference's
  statuses on its error cases;
* the reference's SpeculativeDecoder with that backend reproduces the 10
  recorded decodes (tokens, events, statistics, generator state).
"""

from __future__ import annotations

import hashlib
import json
import random
from pathlib import Path

import numpy as np
import pytest

import sampling_cases as sc

pytestmark = pytest.mark.gpu

GOLDEN_DIR = Path(__file__).parent / "golden"
SAMPLING = json.loads((GOLDEN_DIR / "sampling.json").read_text())


@pytest.fixture(scope="module")
def ref():
    from oracle.reference_runs import ReferenceUnavailable, reference_package

    try:
        reference_package()
    except ReferenceUnavailable as error:
        pytest.skip(str(error))
    from specdecode import native as ref_native

    return ref_native


@pytest.fixture(scope="module")
def ours_path():
    from specdecode_b200 import _lib

    return _lib.load_library().path


@pytest.fixture(scope="module")
def theirs_path(ref):
    return str(Path(ref.__file__).resolve().parents[1] / "libspecdecode_native.so")


def test_reference_quantizer_on_this_library(device, ref, ours_path):
    kat = json.loads((GOLDEN_DIR / "kat_quant.json").read_text())
    quantizer = ref.NativeKVQuantizer.load(ours_path)
    for name, case in kat["vectors"].items():
        q = quantizer.quantize(case["input"])
        assert list(q.values) == case["codes"], name
        assert q.scale == case["scale"], name
        assert list(quantizer.dequantize(q)) == case["dequantized"], name
    with pytest.raises(ref.NativeBackendError) as info:
        quantizer.quantize((1.0, float("nan")))
    assert info.value.status == 3


def _ulps(got, want, n=2):
    got, want = np.asarray(got, dtype=np.float64), np.asarray(want, dtype=np.float64)
    return bool(np.all(np.abs(got - want) <= n * np.spacing(np.maximum(np.abs(got), np.abs(want)))))


def test_reference_sampling_backend_on_this_library(device, ref, ours_path, theirs_path):
    ours = ref.NativeSamplingBackend.load(ours_path)
    theirs = ref.NativeSamplingBackend.load(theirs_path)
    for case in sc.cases():
        k = len(case.proposed)
        target = [[float(x) for x in row] for row in case.target]  # the reference's API takes sequences
        draft = [[float(x) for x in row] for row in case.draft]
        for r in range(k + 1):
            got, want = ours.normalize(target[r]), theirs.normalize(target[r])
            assert np.abs(np.subtract(got, want)).max() <= 1e-15, case.name
        for u in case.uniforms:
            assert ours.categorical(target[0], u) == theirs.categorical(target[0], u), case.name
        for r in range(k):
            got = ours.residual_weights(target[r], draft[r])
            want = theirs.residual_weights(target[r], draft[r])
            assert np.abs(np.subtract(got, want)).max() <= 1e-15, case.name
        tokens = [int(t) for t in case.proposed]
        probs_ours = ours.acceptance_probabilities(target[:k], draft, tokens)
        probs_theirs = theirs.acceptance_probabilities(target[:k], draft, tokens)
        assert _ulps(probs_ours, probs_theirs), case.name
        uniforms = [float(u) for u in case.uniforms[:k]]
        assert ours.first_rejection(probs_theirs, uniforms) == theirs.first_rejection(probs_theirs, uniforms), case.name
    # error statuses of single-fault inputs
    for weights, uniform, status in (([0.5, float("nan")], 0.3, 3), ([0.5, -0.1], 0.3, 4), ([0.0, 0.0], 0.3, 5),
                                      ([0.5, 0.5], 1.0, 7)):
        for backend in (ours, theirs):
            with pytest.raises(ref.NativeBackendError) as info:
                backend.categorical(weights, uniform)
            assert info.value.status == status
    for backend in (ours, theirs):
        with pytest.raises(ref.NativeBackendError) as info:
            backend.acceptance_probabilities([[0.5, 0.5]], [[0.5, 0.5]], [2])
        assert info.value.status == 6


@pytest.mark.parametrize("record", SAMPLING["decodes"], ids=lambda r: r["name"])
def test_reference_decoder_with_its_native_backend_on_this_library(device, ref, ours_path, record):
    from specdecode.config import DecodeConfig
    from specdecode.decoder import SpeculativeDecoder
    from specdecode.models import TableModel

    run = next(r for r in sc.decode_runs() if r["name"] == record["name"])
    (dt, dd), (tt, td) = sc.tables_for(run)
    config = DecodeConfig(max_new_tokens=run["max_new_tokens"], eos_token_id=run["eos_token_id"],
                          initial_draft_tokens=run.get("initial_draft_tokens", 4),
                          dynamic_draft=run.get("dynamic_draft", True))
    rng = random.Random(run["seed"])
    events = []
    decoder = SpeculativeDecoder(TableModel(dt, dd), TableModel(tt, td), config, rng=rng,
                                 sampling_backend=ref.NativeSamplingBackend.load(ours_path))
    result = decoder.generate(run["prompt"], on_token=events.append)
    assert list(result.generated_tokens) == record["generated"]
    assert [e.source for e in events] == record["sources"]
    s = result.stats
    assert dict(drafted_tokens=s.drafted_tokens, accepted_tokens=s.accepted_tokens,
                rejected_tokens=s.rejected_tokens, target_tokens=s.target_tokens,
                verification_rounds=s.verification_rounds, fallback_steps=s.fallback_steps) == record["stats"]
    assert hashlib.sha256(repr(rng.getstate()).encode()).hexdigest() == record["rng_sha"]
