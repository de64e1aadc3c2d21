"""ORACLE -- test infrastructure only.  Only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline leg may use this module, and only as the checker.

CPU restatement of the reference's sampling arithmetic and of one round of
its speculative decoder, the algorithm that the device kernels of
csrc/sampling.cu follow:

* ``normalize`` / ``sample_categorical`` / ``residual_weights`` /
  ``acceptance_probabilities`` / ``first_rejection`` restate the native
  functions of native/src/native.cpp:84-273 with numpy's ``longdouble``,
  which on x86-64 is the same 80-bit extended type the reference compiles
  ``long double`` to, so they reproduce the reference library bit for bit
  (pinned by tests/test_sampling_oracle.py against the library built from
  the reference's sources in oracle/_ref/ and against the fixtures of
  tests/golden/sampling.json);
* ``python_normalize`` / ``python_categorical`` restate the Python backend
  (src/specdecode/sampling.py:14-62), which the decoder applies between the
  native calls;
* ``verify_round`` composes them in the order of one verification round of
  src/specdecode/decoder.py:206-257 with the draws given as a list;
* ``decode`` restates SpeculativeDecoder.generate (decoder.py:148-257) for
  table models.

Scalar Python loops over numpy scalars: meant for vocabularies up to a few
thousand.
"""

from __future__ import annotations

import ctypes
import math
import random
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable, Mapping, Sequence

import numpy as np

LD = np.longdouble

STATUS_OK = 0
STATUS_NULL_ARGUMENT = 1
STATUS_INVALID_SIZE = 2
STATUS_NONFINITE_VALUE = 3
STATUS_NEGATIVE_PROBABILITY = 4
STATUS_ZERO_MASS = 5
STATUS_TOKEN_OUT_OF_RANGE = 6
STATUS_INVALID_UNIFORM = 7


class SamplingError(ValueError):
    """A reference status other than OK, as the reference library returns it."""

    def __init__(self, status: int) -> None:
        super().__init__(f"reference status {status}")
        self.status = status


def _kahan_sum(values: Sequence[float]) -> np.longdouble:
    """native.cpp:20-42: validated Kahan sum in extended precision."""
    if len(values) == 0:
        raise SamplingError(STATUS_INVALID_SIZE)
    total = LD(0.0)
    correction = LD(0.0)
    for value in values:
        x = float(value)
        if not math.isfinite(x):
            raise SamplingError(STATUS_NONFINITE_VALUE)
        if x < 0.0:
            raise SamplingError(STATUS_NEGATIVE_PROBABILITY)
        candidate = LD(x) - correction
        updated = total + candidate
        correction = (updated - total) - candidate
        total = updated
    if not total > 0:
        raise SamplingError(STATUS_ZERO_MASS)
    return total


def _invalid_uniform(u: float) -> bool:
    """native.cpp:44-46."""
    return not math.isfinite(u) or u < 0.0 or u >= 1.0


def normalize(weights: Sequence[float]) -> tuple[float, ...]:
    """native.cpp:84-102."""
    total = _kahan_sum(weights)
    return tuple(float(LD(float(w)) / total) for w in weights)


def sample_categorical(weights: Sequence[float], uniform: float) -> int:
    """native.cpp:104-136: the first index whose extended-precision running sum
    exceeds uniform * sum; the last index if none does."""
    if _invalid_uniform(uniform):
        raise SamplingError(STATUS_INVALID_UNIFORM)
    total = _kahan_sum(weights)
    threshold = LD(uniform) * total
    cumulative = LD(0.0)
    for index, w in enumerate(weights):
        cumulative += LD(float(w))
        if threshold < cumulative:
            return index
    return len(weights) - 1


def residual_weights(target: Sequence[float], draft: Sequence[float]) -> tuple[float, ...]:
    """native.cpp:138-177: max(0, t/S_t - d/S_d) per weight, or the normalised
    target when the residual sums to at most 1e-15."""
    st = _kahan_sum(target)
    sd = _kahan_sum(draft)
    out = []
    residual_sum = LD(0.0)
    for t, d in zip(target, draft):
        p = LD(float(t)) / st
        q = LD(float(d)) / sd
        r = float(max(LD(0.0), p - q))
        out.append(r)
        residual_sum += LD(r)
    if residual_sum <= LD(1.0e-15):
        return tuple(float(LD(float(t)) / st) for t in target)
    return tuple(out)


def acceptance_probabilities(target_rows: Sequence[Sequence[float]], draft_rows: Sequence[Sequence[float]],
                             tokens: Sequence[int]) -> tuple[float, ...]:
    """native.cpp:179-232: min(1, (t/S_t) / (d/S_d)) at each proposed token, 1
    where the draft gives it zero.  Every row is validated first."""
    if len(tokens) == 0 or len(target_rows[0]) == 0:
        raise SamplingError(STATUS_INVALID_SIZE)
    vocab = len(target_rows[0])
    sums = []
    for t_row, d_row, token in zip(target_rows, draft_rows, tokens):
        if token >= vocab:
            raise SamplingError(STATUS_TOKEN_OUT_OF_RANGE)
        sums.append((_kahan_sum(t_row), _kahan_sum(d_row)))
    out = []
    for (st, sd), t_row, d_row, token in zip(sums, target_rows, draft_rows, tokens):
        p = LD(float(t_row[token])) / st
        q = LD(float(d_row[token])) / sd
        out.append(1.0 if q == 0 else float(min(LD(1.0), p / q)))
    return tuple(out)


def first_rejection(probabilities: Sequence[float], uniforms: Sequence[float]) -> int:
    """native.cpp:234-273: the first index with !(u < p), or the count."""
    for p, u in zip(probabilities, uniforms):
        if not math.isfinite(p):
            raise SamplingError(STATUS_NONFINITE_VALUE)
        if p < 0.0 or p > 1.0:
            raise SamplingError(STATUS_NEGATIVE_PROBABILITY)
        if _invalid_uniform(u):
            raise SamplingError(STATUS_INVALID_UNIFORM)
    for index, (p, u) in enumerate(zip(probabilities, uniforms)):
        if not u < p:
            return index
    return len(probabilities)


def python_normalize(probabilities: Sequence[float]) -> tuple[float, ...]:
    """src/specdecode/sampling.py:14-36: validate, fsum, divide."""
    values = [float(v) for v in probabilities]
    if not values or any(not math.isfinite(v) or v < 0.0 for v in values):
        raise ValueError("invalid probability vector")
    total = math.fsum(values)
    if total <= 0.0:
        raise ValueError("probability vector must have positive mass")
    return tuple(v / total for v in values)


def python_categorical(probabilities: Sequence[float], uniform: float) -> int:
    """src/specdecode/backends.py:58-60 with sampling.py:39-56."""
    normalized = python_normalize(probabilities)
    cumulative = 0.0
    for index, p in enumerate(normalized):
        cumulative += p
        if uniform < cumulative:
            return index
    return len(normalized) - 1


@dataclass
class Round:
    """The outcome of one verification round."""

    accepted: int
    token: int  # correction or bonus; -1 after a full acceptance without a bonus
    probabilities: tuple[float, ...]
    draws: int  # uniforms consumed


def verify_round(target_rows: Sequence[Sequence[float]], draft_rows: Sequence[Sequence[float]],
                 proposed: Sequence[int], uniforms: Sequence[float], bonus_allowed: bool = True) -> Round:
    """decoder.py:206-257 for rows already normalised as the decoder's
    ``_probabilities`` leaves them: acceptance probabilities of every
    proposal in one call, one draw per proposal reached, then the correction
    (residual weights, Python-normalised, sampled) or the bonus sample.
    ``uniforms`` are the round's draws in order."""
    n = len(proposed)
    probs = acceptance_probabilities(target_rows[:n], draft_rows, proposed)
    for i in range(n):
        if uniforms[i] < probs[i]:
            continue
        weights = python_normalize(residual_weights(target_rows[i], draft_rows[i]))
        return Round(i, sample_categorical(weights, uniforms[i + 1]), probs, i + 2)
    if not bonus_allowed:
        return Round(n, -1, probs, n)
    return Round(n, sample_categorical(target_rows[n], uniforms[n]), probs, n + 1)


# ---------------------------------------------------------------------------
# The decoder loop for table models (decoder.py:148-257, models.py:99-129).
# ---------------------------------------------------------------------------


class TableModel:
    """Exact context match first, then the final token, then the default
    (src/specdecode/models.py:99-129)."""

    def __init__(self, table: Mapping[tuple[int, ...], Sequence[float]], default: Sequence[float]) -> None:
        self.table = {tuple(k): tuple(v) for k, v in table.items()}
        self.default = tuple(default)
        self.vocab_size = len(self.default)

    def next_token_probs(self, context: Sequence[int]) -> tuple[float, ...]:
        context = tuple(context)
        if context in self.table:
            return self.table[context]
        if context and (context[-1],) in self.table:
            return self.table[(context[-1],)]
        return self.default


@dataclass
class Stats:
    drafted_tokens: int = 0
    accepted_tokens: int = 0
    rejected_tokens: int = 0
    target_tokens: int = 0
    verification_rounds: int = 0
    fallback_steps: int = 0


@dataclass
class Decoded:
    generated: list[int] = field(default_factory=list)
    sources: list[str] = field(default_factory=list)
    stats: Stats = field(default_factory=Stats)


def decode(draft: TableModel, target: TableModel, prompt: Sequence[int], rng: random.Random, *,
           max_new_tokens: int, initial_draft_tokens: int = 4, min_draft_tokens: int = 1,
           max_draft_tokens: int = 8, dynamic_draft: bool = True, eos_token_id: int | None = None,
           categorical: Callable[[Sequence[float], float], int] = sample_categorical) -> Decoded:
    """SpeculativeDecoder.generate with the native sampling functions."""
    out = Decoded()
    window = initial_draft_tokens

    def emit(token: int, source: str) -> None:
        out.generated.append(token)
        out.sources.append(source)

    while len(out.generated) < max_new_tokens:
        prefix = list(prompt) + out.generated
        limit = min(window, max_new_tokens - len(out.generated))
        proposed: list[int] = []
        draft_rows: list[tuple[float, ...]] = []
        for _ in range(limit):
            q = python_normalize(draft.next_token_probs(prefix + proposed))
            token = categorical(q, rng.random())
            draft_rows.append(q)
            proposed.append(token)
            out.stats.drafted_tokens += 1
            if token == eos_token_id:
                break
        # (every table model proposes, so the target-only fallback never runs)
        target_rows = [python_normalize(target.next_token_probs(prefix + proposed[:i]))
                       for i in range(len(proposed) + 1)]
        out.stats.verification_rounds += 1
        probs = acceptance_probabilities(target_rows[:len(proposed)], draft_rows, proposed)
        accepted = 0
        rejected = False
        for i, token in enumerate(proposed):
            if rng.random() < probs[i]:
                emit(token, "accepted_draft")
                out.stats.accepted_tokens += 1
                accepted += 1
                if token == eos_token_id or len(out.generated) == max_new_tokens:
                    break
                continue
            weights = python_normalize(residual_weights(target_rows[i], draft_rows[i]))
            emit(sample_categorical(weights, rng.random()), "target_correction")
            out.stats.rejected_tokens += 1
            out.stats.target_tokens += 1
            rejected = True
            break
        if dynamic_draft:
            if accepted == len(proposed):
                window = min(max_draft_tokens, window + 1)
            elif accepted * 2 < len(proposed):
                window = max(min_draft_tokens, window // 2)
            else:
                window = max(min_draft_tokens, window - 1)
        if out.generated and out.generated[-1] == eos_token_id:
            break
        if len(out.generated) == max_new_tokens:
            break
        if rejected:
            continue
        bonus = sample_categorical(target_rows[-1], rng.random())
        emit(bonus, "target_bonus")
        out.stats.target_tokens += 1
        if bonus == eos_token_id:
            break
    return out


# ---------------------------------------------------------------------------
# The reference library built from its own sources (oracle/_ref/).
# ---------------------------------------------------------------------------

REF_LIBRARY = Path(__file__).resolve().parent / "_ref" / "libspecdecode_native.so"


class ReferenceLibrary:
    """ctypes calls into the reference's native library (native.h:43-87)."""

    def __init__(self, path: str | Path = REF_LIBRARY) -> None:
        self.handle = ctypes.CDLL(str(path))
        d, sz = ctypes.POINTER(ctypes.c_double), ctypes.c_size_t
        h = self.handle
        h.sd_normalize_f64.argtypes = [d, sz, d]
        h.sd_sample_categorical_f64.argtypes = [d, sz, ctypes.c_double, ctypes.POINTER(ctypes.c_uint64)]
        h.sd_residual_weights_f64.argtypes = [d, d, sz, d]
        h.sd_acceptance_probabilities_f64.argtypes = [d, d, ctypes.POINTER(ctypes.c_uint64), sz, sz, d]
        h.sd_first_rejection_f64.argtypes = [d, d, sz, ctypes.POINTER(sz), ctypes.POINTER(sz)]
        for name in ("sd_normalize_f64", "sd_sample_categorical_f64", "sd_residual_weights_f64",
                     "sd_acceptance_probabilities_f64", "sd_first_rejection_f64"):
            getattr(h, name).restype = ctypes.c_int

    @staticmethod
    def _doubles(values: Sequence[float]):
        return (ctypes.c_double * max(1, len(values)))(*[float(v) for v in values])

    def _check(self, status: int) -> None:
        if status != STATUS_OK:
            raise SamplingError(status)

    def normalize(self, weights: Sequence[float]) -> tuple[float, ...]:
        out = (ctypes.c_double * len(weights))()
        self._check(self.handle.sd_normalize_f64(self._doubles(weights), len(weights), out))
        return tuple(out)

    def sample_categorical(self, weights: Sequence[float], uniform: float) -> int:
        out = ctypes.c_uint64()
        self._check(self.handle.sd_sample_categorical_f64(self._doubles(weights), len(weights), uniform,
                                                          ctypes.byref(out)))
        return int(out.value)

    def residual_weights(self, target: Sequence[float], draft: Sequence[float]) -> tuple[float, ...]:
        out = (ctypes.c_double * len(target))()
        self._check(self.handle.sd_residual_weights_f64(self._doubles(target), self._doubles(draft), len(target),
                                                        out))
        return tuple(out)

    def acceptance_probabilities(self, target_rows, draft_rows, tokens) -> tuple[float, ...]:
        vocab = len(target_rows[0])
        flat_t = self._doubles([v for row in target_rows for v in row])
        flat_d = self._doubles([v for row in draft_rows for v in row])
        toks = (ctypes.c_uint64 * len(tokens))(*tokens)
        out = (ctypes.c_double * len(tokens))()
        self._check(self.handle.sd_acceptance_probabilities_f64(flat_t, flat_d, toks, len(tokens), vocab, out))
        return tuple(out)

    def first_rejection(self, probabilities: Sequence[float], uniforms: Sequence[float]) -> int:
        accepted, index = ctypes.c_size_t(), ctypes.c_size_t()
        self._check(self.handle.sd_first_rejection_f64(self._doubles(probabilities), self._doubles(uniforms),
                                                       len(probabilities), ctypes.byref(accepted),
                                                       ctypes.byref(index)))
        return int(index.value)
