"""The sampling oracle (oracle/sampling.py) pinned to the reference.

CPU only.  The restatement must reproduce, bit for bit, what the
reference's native sampling library and its decoder produced for the seeded
cases of tests/sampling_cases.py (tests/golden/sampling.json, written by
tests/golden/make_golden_sampling.py), and agree with the library built from
the reference's sources (oracle/_ref/) on further random rows and on its
error statuses.
"""

from __future__ import annotations

import hashlib
import json
import random
from pathlib import Path

import numpy as np
import pytest

import sampling_cases as sc
from oracle import sampling as orc

GOLDEN = json.loads((Path(__file__).parent / "golden" / "sampling.json").read_text())
CASES = {c.name: c for c in sc.cases()}


def sha(values) -> str:
    return hashlib.sha256(np.asarray(values, dtype=np.float64).tobytes()).hexdigest()


def rows(a):
    return [tuple(float(x) for x in r) for r in a]


@pytest.mark.parametrize("record", GOLDEN["cases"], ids=lambda r: r["name"])
def test_oracle_reproduces_the_reference_functions(record):
    case = CASES[record["name"]]
    n = len(case.proposed)
    target, draft = rows(case.target), rows(case.draft)
    acc = orc.acceptance_probabilities(target[:n], draft, case.proposed)
    assert list(acc) == record["acceptance"]
    assert orc.first_rejection(acc, case.uniforms[:n]) == record["first_rejection"]
    assert [sha(orc.residual_weights(target[i], draft[i])) for i in range(n)] == record["residual_sha"]
    assert [sha(orc.normalize(r)) for r in target] == record["normalized_sha"]
    assert [[orc.sample_categorical(r, u) for u in case.uniforms] for r in target] == record["categorical"]


@pytest.mark.parametrize("record", GOLDEN["cases"], ids=lambda r: r["name"])
def test_oracle_round_matches_the_reference_decoder(record):
    case = CASES[record["name"]]
    tn = [orc.python_normalize(r) for r in rows(case.target)]
    dn = [orc.python_normalize(r) for r in rows(case.draft)]
    got = orc.verify_round(tn, dn, case.proposed, case.uniforms, case.bonus)
    want = record["round"]
    assert (got.accepted, got.token, got.draws) == (want["accepted"], want["token"], want["draws"])
    assert list(got.probabilities) == want["probabilities"]


def test_oracle_known_answers():
    kat = GOLDEN["kat"]
    w = sc.KAT_CATEGORICAL_WEIGHTS
    assert list(orc.normalize(w)) == kat["normalized"]
    assert [orc.sample_categorical(w, u) for u in sc.KAT_CATEGORICAL_UNIFORMS] == kat["categorical"]
    assert [orc.python_categorical(w, u) for u in sc.KAT_CATEGORICAL_UNIFORMS] == kat["python_categorical"]
    assert list(orc.acceptance_probabilities(sc.KAT_TARGET_ROWS, sc.KAT_DRAFT_ROWS, sc.KAT_TOKENS)) == \
        kat["acceptance"]
    assert list(orc.residual_weights(sc.KAT_TARGET_ROWS[0], sc.KAT_DRAFT_ROWS[0])) == kat["residual_0"]
    assert list(orc.residual_weights(sc.KAT_TARGET_ROWS[2], sc.KAT_TARGET_ROWS[2])) == kat["residual_same"]
    assert orc.first_rejection(sc.KAT_REJECTION_PROBABILITIES, sc.KAT_REJECTION_UNIFORMS) == kat["first_rejection"]


@pytest.mark.parametrize("record", GOLDEN["decodes"], ids=lambda r: r["name"])
def test_oracle_decode_matches_the_reference_decoder(record):
    run = next(r for r in sc.decode_runs() if r["name"] == record["name"])
    (dt, dd), (tt, td) = sc.tables_for(run)
    rng = random.Random(run["seed"])
    out = orc.decode(orc.TableModel(dt, dd), orc.TableModel(tt, td), run["prompt"], rng,
                     max_new_tokens=run["max_new_tokens"], eos_token_id=run["eos_token_id"],
                     initial_draft_tokens=run.get("initial_draft_tokens", 4),
                     dynamic_draft=run.get("dynamic_draft", True))
    assert out.generated == record["generated"]
    assert out.sources == record["sources"]
    assert vars(out.stats) == record["stats"]
    assert hashlib.sha256(repr(rng.getstate()).encode()).hexdigest() == record["rng_sha"]


@pytest.fixture(scope="module")
def reference_library():
    if not orc.REF_LIBRARY.is_file():
        pytest.skip("oracle/_ref is not built (make -C oracle ref)")
    return orc.ReferenceLibrary()


def test_oracle_matches_the_reference_library_on_random_rows(reference_library):
    ref = reference_library
    rng = np.random.default_rng(77)
    for trial in range(40):
        vocab = int(rng.integers(1, 300))
        kind_t, kind_d = rng.choice(["softmax", "sparse", "wide", "exact", "peaked"], 2)
        t = rows(np.stack([sc._row(rng, kind_t, vocab) for _ in range(3)]))
        d = rows(np.stack([sc._row(rng, kind_d, vocab) for _ in range(2)]))
        tokens = [int(x) for x in rng.integers(0, vocab, 2)]
        assert orc.acceptance_probabilities(t[:2], d, tokens) == ref.acceptance_probabilities(t[:2], d, tokens)
        assert orc.residual_weights(t[0], d[0]) == ref.residual_weights(t[0], d[0])
        assert orc.normalize(t[2]) == ref.normalize(t[2])
        for u in rng.random(4):
            assert orc.sample_categorical(t[1], float(u)) == ref.sample_categorical(t[1], float(u))
        p, u = rng.random(5).tolist(), rng.random(5).tolist()
        assert orc.first_rejection(p, u) == ref.first_rejection(p, u)


@pytest.mark.parametrize("call", [
    lambda m: m.sample_categorical((0.5, -0.5), 0.1),
    lambda m: m.sample_categorical((0.5, 0.5), 1.0),
    lambda m: m.sample_categorical((0.0, 0.0), 0.1),
    lambda m: m.sample_categorical((float("nan"), 1.0), 0.1),
    lambda m: m.acceptance_probabilities(((1.0, 0.0),), ((1.0, 0.0),), (2,)),
    lambda m: m.residual_weights((0.0, 0.0), (1.0, 0.0)),
    lambda m: m.first_rejection((1.5,), (0.1,)),
    lambda m: m.first_rejection((0.5,), (-0.1,)),
])
def test_oracle_errors_carry_the_reference_status(reference_library, call):
    with pytest.raises(orc.SamplingError) as want:
        call(reference_library)
    with pytest.raises(orc.SamplingError) as got:
        call(orc)
    assert got.value.status == want.value.status


def _weights(draw_rows):
    from hypothesis import strategies as st

    value = st.one_of(
        st.just(0.0),
        st.floats(min_value=0.0, max_value=1.0, allow_nan=False, allow_infinity=False),
        st.floats(min_value=0.0, max_value=1e300, allow_nan=False, allow_infinity=False),
        st.floats(min_value=0.0, max_value=1e-300, allow_nan=False, allow_infinity=False, allow_subnormal=True),
    )
    return st.lists(value, min_size=draw_rows, max_size=draw_rows)


@pytest.mark.parametrize("vocab", [1, 3, 17])
def test_oracle_matches_the_reference_library_on_generated_rows(reference_library, vocab):
    """Property check over generated rows: zeros, subnormals, 300-decade
    ranges and all-zero rows (a zero-mass status) -- the restatement and the
    reference library agree on every output value and every status."""
    from hypothesis import HealthCheck, given, settings
    from hypothesis import strategies as st

    ref = reference_library

    def both(call):
        try:
            want = ("ok", call(ref))
        except orc.SamplingError as e:
            want = ("status", e.status)
        try:
            got = ("ok", call(orc))
        except orc.SamplingError as e:
            got = ("status", e.status)
        assert got == want

    @settings(max_examples=150, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
    @given(t=_weights(vocab), d=_weights(vocab), token=st.integers(0, vocab - 1),
           u=st.floats(min_value=0.0, max_value=1.0, exclude_max=True, allow_nan=False))
    def check(t, d, token, u):
        both(lambda m: m.normalize(t))
        both(lambda m: m.sample_categorical(t, u))
        both(lambda m: m.residual_weights(t, d))
        both(lambda m: m.acceptance_probabilities([t], [d], [token]))

    check()


@pytest.mark.parametrize("record", GOLDEN["cases"], ids=lambda r: r["name"])
def test_round_decisions_do_not_depend_on_normalising_first(record):
    """The device round takes the rows as stored (softmax output, not
    renormalised the way the decoder's ``_probabilities`` does); on every
    case the reference functions reach the same decisions either way."""
    case = CASES[record["name"]]
    got = orc.verify_round(rows(case.target), rows(case.draft), case.proposed, case.uniforms, case.bonus)
    want = record["round"]
    assert (got.accepted, got.token, got.draws) == (want["accepted"], want["token"], want["draws"])
