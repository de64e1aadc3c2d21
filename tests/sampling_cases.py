"""Seeded verification-round cases shared by tests/golden/make_golden_sampling.py
and the sampling tests.

A case is one sequence's round: ``target`` rows [n + 1][V] (the proposal
positions plus the bonus position), ``draft`` rows [n][V], the ``proposed``
tokens, the round's ``uniforms`` [n + 1] and whether a full acceptance earns a
bonus.  Rows are float64 weights (not normalised) of several shapes: float32
softmax rows (what a model's logits give), sparse rows with exact zeros,
rows spanning 300 decades, small-integer rows whose sums are exact, and
peaked rows.  The generator is numpy's PCG64, stable across numpy versions.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class Case:
    name: str
    target: np.ndarray  # [n + 1, V] float64
    draft: np.ndarray  # [n, V] float64
    proposed: list[int]
    uniforms: list[float]
    bonus: bool = True


def _row(rng: np.random.Generator, kind: str, vocab: int) -> np.ndarray:
    if kind == "softmax":
        logits = rng.normal(0.0, 3.0, vocab)
        p = np.exp(logits - logits.max())
        return (p / p.sum()).astype(np.float32).astype(np.float64)
    if kind == "sparse":
        w = rng.random(vocab)
        w[rng.random(vocab) < 0.7] = 0.0
        if not w.any():
            w[rng.integers(vocab)] = 1.0
        return w
    if kind == "wide":
        return 10.0 ** rng.uniform(-300.0, 0.0, vocab)
    if kind == "exact":
        w = rng.integers(0, 6, vocab).astype(np.float64)
        if not w.any():
            w[0] = 1.0
        return w
    if kind == "peaked":
        w = np.full(vocab, 1.0e-12)
        w[rng.integers(vocab)] = 1.0
        return w
    raise ValueError(kind)


def _propose(rng: np.random.Generator, draft: np.ndarray) -> list[int]:
    """A token per draft row, drawn from the row (as the draft would)."""
    out = []
    for row in draft:
        p = row / row.sum()
        out.append(int(rng.choice(len(row), p=p)))
    return out


def random_case(name: str, seed: int, vocab: int, n: int, target_kind: str, draft_kind: str, *,
                bonus: bool = True) -> Case:
    rng = np.random.default_rng(seed)
    target = np.stack([_row(rng, target_kind, vocab) for _ in range(n + 1)])
    draft = np.stack([_row(rng, draft_kind, vocab) for _ in range(n)])
    proposed = _propose(rng, draft)
    uniforms = rng.random(n + 1).tolist()
    return Case(name, target, draft, proposed, uniforms, bonus)


def cases() -> list[Case]:
    out = [
        random_case("softmax_v1000", 1, 1000, 5, "softmax", "softmax"),
        random_case("softmax_v4097", 2, 4097, 4, "softmax", "softmax"),
        random_case("softmax_v300_k8", 3, 300, 8, "softmax", "softmax"),
        random_case("sparse_v513", 4, 513, 6, "sparse", "sparse"),
        random_case("wide_v700", 5, 700, 3, "wide", "wide"),
        random_case("exact_v64", 6, 64, 4, "exact", "exact"),
        random_case("peaked_v2000", 7, 2000, 5, "peaked", "softmax"),
        random_case("mixed_v129", 8, 129, 7, "softmax", "sparse"),
        random_case("v1", 9, 1, 2, "softmax", "softmax"),
        random_case("v3", 10, 3, 3, "exact", "exact"),
        random_case("no_bonus_v200", 11, 200, 4, "softmax", "softmax", bonus=False),
    ]
    # identical draft and target: every proposal accepted (probability 1),
    # and the residual of any row is the fallback to the target
    same = random_case("identical_v257", 12, 257, 4, "softmax", "softmax")
    same.draft = same.target[:-1].copy()
    out.append(same)
    # the draft gives the proposed token zero probability: acceptance 1
    zero_q = random_case("draft_zero_v100", 13, 100, 3, "softmax", "sparse")
    zero_q.draft[0, zero_q.proposed[0]] = 0.0
    out.append(zero_q)
    # the target gives the first proposal zero probability: acceptance 0, so
    # the first draw rejects it whatever it is (0 included)
    zero_p = random_case("target_zero_v100", 14, 100, 3, "softmax", "softmax")
    zero_p.target[0, zero_p.proposed[0]] = 0.0
    zero_p.uniforms[0] = 0.0
    out.append(zero_p)
    # a full acceptance that earns no bonus: the round ends after n draws
    same_no_bonus = random_case("identical_no_bonus_v90", 15, 90, 3, "softmax", "softmax", bonus=False)
    same_no_bonus.draft = same_no_bonus.target[:-1].copy()
    out.append(same_no_bonus)
    # drafts close to the target (every weight scaled by exp(N(0, 0.3))):
    # acceptance probabilities spread over (0, 1], rounds end at every index
    for seed in range(30, 38):
        near = random_case(f"near_v500_s{seed}", seed, 500, 6, "softmax", "softmax")
        rng = np.random.default_rng(seed + 1000)
        near.draft = near.target[:-1] * np.exp(rng.normal(0.0, 0.3, near.draft.shape))
        near.proposed = _propose(rng, near.draft)
        out.append(near)
    for seed in range(20, 26):
        out.append(random_case(f"softmax_v50_s{seed}", seed, 50, 3, "softmax", "softmax"))
    return out


# The reference's own test vectors (tests/test_native.py:40-82).
KAT_CATEGORICAL_WEIGHTS = (0.0, 2.0, 3.0, 5.0, 0.0)
KAT_CATEGORICAL_UNIFORMS = (0.0, 0.19, 0.2, 0.499, 0.5, float(np.nextafter(1.0, 0.0)))
KAT_TARGET_ROWS = ((0.2, 0.5, 0.3), (0.2, 0.6, 0.2), (0.0, 0.0, 1.0))
KAT_DRAFT_ROWS = ((0.4, 0.4, 0.2), (0.6, 0.2, 0.2), (0.0, 1.0, 0.0))
KAT_TOKENS = (0, 1, 2)
KAT_REJECTION_PROBABILITIES = (0.0, 0.5, 1.0)
KAT_REJECTION_UNIFORMS = (0.0, 0.1, 0.1)

# Table models for whole-decode comparisons: the reference test's tables
# (tests/test_native.py:92-124) and seeded random tables.
REFERENCE_DRAFT = ({(0,): (0.05, 0.70, 0.20, 0.05), (1,): (0.05, 0.20, 0.65, 0.10)}, (0.05, 0.10, 0.35, 0.50))
REFERENCE_TARGET = ({(0,): (0.05, 0.55, 0.30, 0.10), (1,): (0.05, 0.15, 0.60, 0.20)}, (0.05, 0.10, 0.25, 0.60))


def random_tables(seed: int, vocab: int = 20, contexts: int = 8):
    rng = np.random.default_rng(seed)

    def dist():
        p = rng.gamma(0.5, 1.0, vocab)
        return tuple(float(x) for x in (p / p.sum()))

    draft = ({(int(t),): dist() for t in rng.choice(vocab, contexts, replace=False)}, dist())
    target = ({(int(t),): dist() for t in rng.choice(vocab, contexts, replace=False)}, dist())
    return draft, target


def decode_runs() -> list[dict]:
    """Decoder configurations run by the fixture script and the tests."""
    runs = [dict(name="reference_tables_eos", tables="reference", seed=7, prompt=[0], max_new_tokens=12,
                 eos_token_id=3)]
    for seed in range(3):
        runs.append(dict(name=f"reference_tables_s{seed}", tables="reference", seed=seed, prompt=[0],
                         max_new_tokens=40, eos_token_id=None))
    for seed in range(4):
        runs.append(dict(name=f"random_tables_s{seed}", tables=100 + seed, seed=seed, prompt=[1, 2],
                         max_new_tokens=48, eos_token_id=None))
    runs.append(dict(name="random_tables_eos", tables=200, seed=11, prompt=[3], max_new_tokens=64, eos_token_id=5))
    runs.append(dict(name="static_window", tables=201, seed=12, prompt=[4], max_new_tokens=30, eos_token_id=None,
                     initial_draft_tokens=3, dynamic_draft=False))
    return runs


def tables_for(run: dict):
    if run["tables"] == "reference":
        return REFERENCE_DRAFT, REFERENCE_TARGET
    return random_tables(run["tables"])
