"""Host-side logic of the batched speculative decoder on CPU: the
acceptance / resampling rule of the reference decoder
(src/specdecode/decoder.py:202-257), as the oracle restates it and the
device verification follows it (tests/test_gpu_sampling.py holds the device
to the oracle's decisions), greedy verification, and the adaptive window
(src/specdecode/decoder.py:47-60)."""

from __future__ import annotations

import random

import numpy as np
import torch

from oracle import sampling as orc
from specdecode_b200.speculative import DraftWindow, accept_greedy


def _row(rng, V):
    p = rng.gamma(0.7, 1.0, V)
    return tuple(float(x) for x in p / p.sum())


def test_identical_distributions_accept_everything():
    rng = np.random.default_rng(0)
    draws = random.Random(0)
    for _ in range(50):
        target = [_row(rng, 11) for _ in range(5)]
        proposed = [orc.sample_categorical(target[i], draws.random()) for i in range(4)]
        got = orc.verify_round(target, target[:4], proposed, [draws.random() for _ in range(5)])
        assert got.accepted == 4 and got.draws == 5 and 0 <= got.token < 11


def test_committed_tokens_follow_the_target():
    """Speculative sampling is exact: the first committed token (an accepted
    first proposal or the resampled replacement) is distributed as the
    target's first distribution, although the draft's is far from it."""
    rng = np.random.default_rng(1)
    V, k, n = 5, 2, 12_000
    target = [_row(rng, V) for _ in range(k + 1)]
    draft = [_row(rng, V) for _ in range(k)]
    assert 0.5 * sum(abs(a - b) for a, b in zip(target[0], draft[0])) > 0.1
    draws = random.Random(2)
    counts = [0] * V
    for _ in range(n):
        proposed = [orc.sample_categorical(draft[i], draws.random()) for i in range(k)]
        got = orc.verify_round(target, draft, proposed, [draws.random() for _ in range(k + 1)])
        counts[proposed[0] if got.accepted > 0 else got.token] += 1
    freq = np.array(counts) / n
    assert float(np.abs(freq - np.array(target[0])).max()) < 0.02


def test_greedy_verification():
    logits = torch.tensor([[[0.0, 5.0, 1.0], [3.0, 0.0, 0.0], [0.0, 0.0, 9.0]]])  # argmax 1, 0, 2
    acc, tok = accept_greedy(torch.tensor([[1, 2]]), logits)
    assert acc.tolist() == [1] and tok.tolist() == [[0]]
    acc, tok = accept_greedy(torch.tensor([[1, 0]]), logits)
    assert acc.tolist() == [2] and tok.tolist() == [[2]]
    acc, tok = accept_greedy(torch.tensor([[0, 0]]), logits)
    assert acc.tolist() == [0] and tok.tolist() == [[1]]


def test_draft_window_follows_the_reference_rule():
    w = DraftWindow(5, 4, 8)
    w.observe(5, 5)
    assert w.size == 6
    w.observe(2, 6)  # under half accepted: halve, floored at the minimum
    assert w.size == 4
    w.observe(3, 4)  # some rejected: shrink by one, floored
    assert w.size == 4
    for _ in range(10):
        w.observe(w.size, w.size)
    assert w.size == 8
    fixed = DraftWindow(5, dynamic=False)
    fixed.observe(0, 5)
    assert fixed.size == 5
