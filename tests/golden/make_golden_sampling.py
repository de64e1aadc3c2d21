"""Generate tests/golden/sampling.json by running the reference itself.

Run in a checkout that has the reference at /root/reference (read-only) and
its native library built by ``make -C oracle ref``::

    python tests/golden/make_golden_sampling.py

It imports the reference's Python package from /root/reference/src, loads its
native sampling library from oracle/_ref/, and records for the seeded cases
of tests/sampling_cases.py:

* per case: the native acceptance probabilities, first rejection, a sha256
  of every residual-weight row and every normalised row, categorical samples
  of every target row at every draw of the case, and the outcome of the
  decoder's verification round (src/specdecode/decoder.py:206-257) composed
  from the reference's own functions on the rows normalised as the decoder
  normalises them;
* the reference tests' known-answer vectors (tests/test_native.py:40-82);
* whole decodes of SpeculativeDecoder over table models with the native and
  the Python backend (which must agree): tokens, event sources, statistics
  and a sha256 of the generator state afterwards.

Nothing at test time reads /root/reference; tests only read the fixture.
"""

from __future__ import annotations

import hashlib
import json
import random
import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, "/root/reference/src")
sys.path.insert(0, str(REPO / "tests"))

from specdecode.backends import PythonSamplingBackend  # noqa: E402
from specdecode.config import DecodeConfig  # noqa: E402
from specdecode.decoder import SpeculativeDecoder  # noqa: E402
from specdecode.models import TableModel  # noqa: E402
from specdecode.native import NativeSamplingBackend  # noqa: E402
from specdecode.sampling import normalize_probabilities  # noqa: E402

import sampling_cases as sc  # noqa: E402

NATIVE = NativeSamplingBackend.load(REPO / "oracle" / "_ref" / "libspecdecode_native.so")
PYTHON = PythonSamplingBackend()


def sha(values) -> str:
    return hashlib.sha256(np.asarray(values, dtype=np.float64).tobytes()).hexdigest()


def rows(a: np.ndarray):
    return [tuple(float(x) for x in r) for r in a]


def reference_round(target, draft, proposed, uniforms, bonus):
    n = len(proposed)
    tn = [normalize_probabilities(r) for r in target]
    dn = [normalize_probabilities(r) for r in draft]
    probs = NATIVE.acceptance_probabilities(tn[:n], dn, proposed)
    for i in range(n):
        if uniforms[i] < probs[i]:
            continue
        correction = normalize_probabilities(NATIVE.residual_weights(tn[i], dn[i]))
        return dict(accepted=i, token=NATIVE.categorical(correction, uniforms[i + 1]), draws=i + 2,
                    probabilities=list(probs))
    if not bonus:
        return dict(accepted=n, token=-1, draws=n, probabilities=list(probs))
    return dict(accepted=n, token=NATIVE.categorical(tn[n], uniforms[n]), draws=n + 1, probabilities=list(probs))


def case_record(case: sc.Case) -> dict:
    n = len(case.proposed)
    target, draft = rows(case.target), rows(case.draft)
    acc = NATIVE.acceptance_probabilities(target[:n], draft, case.proposed)
    rej = NATIVE.first_rejection(acc, case.uniforms[:n])
    return dict(
        name=case.name,
        acceptance=list(acc),
        first_rejection=rej.accepted_count,
        residual_sha=[sha(NATIVE.residual_weights(target[i], draft[i])) for i in range(n)],
        normalized_sha=[sha(NATIVE.normalize(r)) for r in target],
        categorical=[[NATIVE.categorical(r, u) for u in case.uniforms] for r in target],
        round=reference_round(target, draft, case.proposed, case.uniforms, case.bonus),
    )


def kat_record() -> dict:
    w = sc.KAT_CATEGORICAL_WEIGHTS
    return dict(
        normalized=list(NATIVE.normalize(w)),
        categorical=[NATIVE.categorical(w, u) for u in sc.KAT_CATEGORICAL_UNIFORMS],
        python_categorical=[PYTHON.categorical(w, u) for u in sc.KAT_CATEGORICAL_UNIFORMS],
        acceptance=list(NATIVE.acceptance_probabilities(sc.KAT_TARGET_ROWS, sc.KAT_DRAFT_ROWS, sc.KAT_TOKENS)),
        residual_0=list(NATIVE.residual_weights(sc.KAT_TARGET_ROWS[0], sc.KAT_DRAFT_ROWS[0])),
        residual_same=list(NATIVE.residual_weights(sc.KAT_TARGET_ROWS[2], sc.KAT_TARGET_ROWS[2])),
        first_rejection=NATIVE.first_rejection(sc.KAT_REJECTION_PROBABILITIES, sc.KAT_REJECTION_UNIFORMS)
        .accepted_count,
    )


def decode_record(run: dict) -> dict:
    (dt, dd), (tt, td) = sc.tables_for(run)
    config = DecodeConfig(max_new_tokens=run["max_new_tokens"], eos_token_id=run["eos_token_id"],
                          initial_draft_tokens=run.get("initial_draft_tokens", 4),
                          dynamic_draft=run.get("dynamic_draft", True))
    results = []
    for backend in (NATIVE, PYTHON):
        rng = random.Random(run["seed"])
        events = []
        result = SpeculativeDecoder(TableModel(dt, dd), TableModel(tt, td), config, rng=rng,
                                    sampling_backend=backend).generate(run["prompt"], on_token=events.append)
        stats = result.stats
        results.append(dict(
            generated=list(result.generated_tokens),
            sources=[e.source for e in events],
            indices=[e.index for e in events],
            stats=dict(drafted_tokens=stats.drafted_tokens, accepted_tokens=stats.accepted_tokens,
                       rejected_tokens=stats.rejected_tokens, target_tokens=stats.target_tokens,
                       verification_rounds=stats.verification_rounds, fallback_steps=stats.fallback_steps),
            rng_sha=hashlib.sha256(repr(rng.getstate()).encode()).hexdigest(),
        ))
    assert results[0] == results[1], run["name"]
    return dict(name=run["name"], **results[0])


def main() -> None:
    out = dict(
        cases=[case_record(c) for c in sc.cases()],
        kat=kat_record(),
        decodes=[decode_record(r) for r in sc.decode_runs()],
    )
    path = REPO / "tests" / "golden" / "sampling.json"
    path.write_text(json.dumps(out, indent=1) + "\n")
    print(path, path.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
