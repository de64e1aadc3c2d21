"""The reference's single-sequence speculative decoder with its verification
on the device.

``SpeculativeDecoder`` keeps the reference's constructor, ``generate``
signature, results, token events, statistics and seeded draw order
(src/specdecode/decoder.py:20-257, config.py:7-30, events.py): the draft
proposes one token per draw of the caller's ``random.Random``, the target
scores the proposals, and each proposal is accepted with probability
min(1, p/q) until the first rejection, which is replaced by a sample of the
normalised residual; a fully accepted window earns a bonus token.

What runs where:

* draft proposals and the target-only fallback sample through
  ``sampling_backend.categorical`` (default: ``DeviceSamplingBackend``, the
  device kernel of sd_sample_categorical_f64);
* the verification round -- acceptance probabilities, first rejection,
  residual construction and the correction or bonus sample -- is one
  ``sdc_speculative_verify`` call.  The reference draws its round's uniforms
  one at a time, as the round consumes them; here the round's maximum (one
  per proposal plus one) is drawn ahead, the kernel reports how far the
  round got, and the generator is rewound and advanced by exactly the draws
  the reference would have taken, so the generator state after every round
  equals the reference's.
"""

from __future__ import annotations

import math
import random
from collections.abc import Callable, Sequence
from dataclasses import dataclass
from numbers import Integral
from typing import Any, Literal, Protocol

from .sampling import DeviceSamplingBackend, raise_for_status, verify_batch

TokenSource = Literal["accepted_draft", "target_correction", "target_bonus", "target_fallback", "target_only"]


class DistributionError(ValueError):
    """src/specdecode/sampling.py:10-11."""


class ProbabilityModel(Protocol):
    vocab_size: int

    def next_token_probs(self, token_ids: Sequence[int]) -> Sequence[float]: ...


@dataclass(frozen=True)
class DecodeConfig:
    """src/specdecode/config.py:7-30."""

    max_new_tokens: int = 32
    initial_draft_tokens: int = 4
    min_draft_tokens: int = 1
    max_draft_tokens: int = 8
    dynamic_draft: bool = True
    eos_token_id: int | None = None

    def __post_init__(self) -> None:
        if self.max_new_tokens < 0:
            raise ValueError("max_new_tokens must be non-negative")
        if self.min_draft_tokens < 1:
            raise ValueError("min_draft_tokens must be at least 1")
        if self.max_draft_tokens < self.min_draft_tokens:
            raise ValueError("max_draft_tokens must be >= min_draft_tokens")
        if not self.min_draft_tokens <= self.initial_draft_tokens <= self.max_draft_tokens:
            raise ValueError("initial_draft_tokens must be inside the configured range")


@dataclass(frozen=True)
class TokenEvent:
    """src/specdecode/events.py."""

    token_id: int
    index: int
    source: TokenSource


@dataclass
class DecodeStats:
    """src/specdecode/decoder.py:20-33."""

    drafted_tokens: int = 0
    accepted_tokens: int = 0
    rejected_tokens: int = 0
    target_tokens: int = 0
    verification_rounds: int = 0
    fallback_steps: int = 0

    @property
    def acceptance_rate(self) -> float:
        return self.accepted_tokens / self.drafted_tokens if self.drafted_tokens else 0.0


@dataclass(frozen=True)
class DecodeResult:
    """src/specdecode/decoder.py:36-44."""

    prompt_tokens: tuple[int, ...]
    generated_tokens: tuple[int, ...]
    stats: DecodeStats

    @property
    def all_tokens(self) -> tuple[int, ...]:
        return self.prompt_tokens + self.generated_tokens


def normalize_probabilities(probabilities: Sequence[float], *, expected_size: int | None = None) -> tuple[float, ...]:
    """Host-side validation and normalisation of a model's row, as the
    reference decoder applies it to every distribution it receives
    (src/specdecode/sampling.py:14-36)."""
    if expected_size is not None and len(probabilities) != expected_size:
        raise DistributionError(f"expected {expected_size} probabilities, received {len(probabilities)}")
    if not probabilities:
        raise DistributionError("probability vector cannot be empty")
    values = []
    for value in probabilities:
        number = float(value)
        if not math.isfinite(number) or number < 0.0:
            raise DistributionError("probabilities must be finite and non-negative")
        values.append(number)
    total = math.fsum(values)
    if total <= 0.0:
        raise DistributionError("probability vector must have positive mass")
    return tuple(v / total for v in values)


class _Window:
    """src/specdecode/decoder.py:47-60."""

    def __init__(self, config: DecodeConfig) -> None:
        self._config = config
        self.size = config.initial_draft_tokens

    def observe(self, accepted: int, proposed: int) -> None:
        if not self._config.dynamic_draft or proposed == 0:
            return
        if accepted == proposed:
            self.size = min(self._config.max_draft_tokens, self.size + 1)
        elif accepted * 2 < proposed:
            self.size = max(self._config.min_draft_tokens, self.size // 2)
        else:
            self.size = max(self._config.min_draft_tokens, self.size - 1)


class SpeculativeDecoder:
    """src/specdecode/decoder.py:69-257 with the round verified on the device."""

    def __init__(self, draft_model: ProbabilityModel, target_model: ProbabilityModel,
                 config: DecodeConfig | None = None, *, rng: random.Random | None = None,
                 sampling_backend: Any = None, device: Any = None) -> None:
        if draft_model.vocab_size != target_model.vocab_size:
            raise ValueError("draft and target models must share a vocabulary")
        if draft_model.vocab_size < 1:
            raise ValueError("model vocabulary must be positive")
        self.draft_model = draft_model
        self.target_model = target_model
        self.config = config or DecodeConfig()
        if self.config.eos_token_id is not None and not 0 <= self.config.eos_token_id < target_model.vocab_size:
            raise ValueError("eos_token_id must be inside the shared vocabulary")
        self.rng = rng or random.Random()
        self.sampling_backend = sampling_backend if sampling_backend is not None else DeviceSamplingBackend(device)
        self.device = getattr(self.sampling_backend, "device", None) or device or "cuda"

    def _probabilities(self, model: ProbabilityModel, context: list[int]) -> tuple[float, ...]:
        return normalize_probabilities(model.next_token_probs(context), expected_size=model.vocab_size)

    def _sample(self, probabilities: Sequence[float]) -> int:
        return self.sampling_backend.categorical(probabilities, self.rng.random())

    def _validate_prompt(self, prompt_tokens: Sequence[int]) -> tuple[int, ...]:
        prompt = []
        for token in prompt_tokens:
            if isinstance(token, bool) or not isinstance(token, Integral):
                raise TypeError("prompt token IDs must be integers")
            token_id = int(token)
            if not 0 <= token_id < self.target_model.vocab_size:
                raise ValueError("prompt token ID is outside the shared vocabulary")
            prompt.append(token_id)
        return tuple(prompt)

    def _verify(self, target_rows, draft_rows, proposed: list[int], bonus_allowed: bool):
        """One device verification round; returns (accepted, token), with the
        generator left where the reference's would be."""
        import torch

        n = len(proposed)
        state = self.rng.getstate()
        draws = [self.rng.random() for _ in range(n + 1)]
        dev = self.device
        target = torch.tensor([list(target_rows)], dtype=torch.float64, device=dev)
        draft = torch.tensor([list(draft_rows)], dtype=torch.float64, device=dev)
        tokens = torch.tensor([proposed], dtype=torch.int64, device=dev)
        uniforms = torch.tensor([draws], dtype=torch.float64, device=dev)
        bonus = torch.tensor([1 if bonus_allowed else 0], dtype=torch.uint8, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        accepted, token, _ = verify_batch(target, draft, tokens, uniforms, bonus_allowed=bonus, status=status)
        raise_for_status(status, "speculative verification")
        j, tok = int(accepted.item()), int(token.item())
        consumed = j + 2 if j < n else (n + 1 if bonus_allowed else n)
        self.rng.setstate(state)
        for _ in range(consumed):
            self.rng.random()
        return j, tok

    def generate(self, prompt_tokens: Sequence[int], *,
                 on_token: Callable[[TokenEvent], None] | None = None) -> DecodeResult:
        config = self.config
        prompt = self._validate_prompt(prompt_tokens)
        for model in {id(self.draft_model): self.draft_model, id(self.target_model): self.target_model}.values():
            reset = getattr(model, "reset_cache", None)
            if callable(reset):
                reset()
        generated: list[int] = []
        stats = DecodeStats()
        window = _Window(config)

        def emit(token: int, source: TokenSource) -> None:
            generated.append(token)
            if on_token is not None:
                on_token(TokenEvent(token_id=token, index=len(generated) - 1, source=source))

        if config.max_new_tokens == 0:
            return DecodeResult(prompt, (), stats)

        while len(generated) < config.max_new_tokens:
            prefix = list(prompt) + generated
            remaining = config.max_new_tokens - len(generated)
            limit = min(window.size, remaining)
            proposed: list[int] = []
            draft_rows: list[tuple[float, ...]] = []
            for _ in range(limit):
                try:
                    q = self._probabilities(self.draft_model, prefix + proposed)
                except (DistributionError, RuntimeError, ValueError):
                    break
                token = self._sample(q)
                draft_rows.append(q)
                proposed.append(token)
                stats.drafted_tokens += 1
                if token == config.eos_token_id:
                    break

            if not proposed:
                token = self._sample(self._probabilities(self.target_model, prefix))
                emit(token, "target_fallback")
                stats.target_tokens += 1
                stats.fallback_steps += 1
                if token == config.eos_token_id:
                    break
                continue

            target_rows = [self._probabilities(self.target_model, prefix + proposed[:i])
                           for i in range(len(proposed) + 1)]
            stats.verification_rounds += 1
            bonus_allowed = proposed[-1] != config.eos_token_id and len(proposed) < remaining
            accepted, token = self._verify(target_rows, draft_rows, proposed, bonus_allowed)
            for t in proposed[:accepted]:
                emit(t, "accepted_draft")
            stats.accepted_tokens += accepted
            window.observe(accepted, len(proposed))
            if accepted < len(proposed):
                emit(token, "target_correction")
                stats.rejected_tokens += 1
                stats.target_tokens += 1
                if token == config.eos_token_id:
                    break
                continue
            if not bonus_allowed:
                break
            emit(token, "target_bonus")
            stats.target_tokens += 1
            if token == config.eos_token_id:
                break

        return DecodeResult(prompt, tuple(generated), stats)
