"""Host-side logic of the batched speculative decoder, on CPU tensors: the
acceptance / resampling rule of the reference decoder
(src/specdecode/decoder.py:202-257) and its adaptive window
(src/specdecode/decoder.py:47-60)."""

from __future__ import annotations

import torch

from specdecode_b200.speculative import DraftWindow, accept_greedy, accept_sampled


def _dists(gen, n, k, V, sharp):
    return torch.softmax(torch.randn((n, k, V), generator=gen) * sharp, dim=-1)


def test_identical_distributions_accept_everything():
    gen = torch.Generator().manual_seed(0)
    p = _dists(gen, 64, 4, 11, 2.0)
    q = torch.cat([p, _dists(gen, 64, 1, 11, 2.0)], dim=1)
    drafts = torch.multinomial(p.reshape(-1, 11), 1, generator=gen).reshape(64, 4)
    accepted, tok = accept_sampled(drafts, p, q, gen)
    assert torch.equal(accepted, torch.full((64,), 4))
    assert tok.shape == (64, 1)


def test_committed_tokens_follow_the_target():
    """Speculative sampling is exact: the first committed token (an accepted
    first proposal or the resampled replacement) is distributed as the
    target's first distribution, and the token committed after an accepted
    first proposal as the target's second."""
    gen = torch.Generator().manual_seed(1)
    V, k, n = 7, 3, 200_000
    p1 = torch.softmax(torch.randn(V, generator=gen) * 2, dim=-1)
    q1 = torch.softmax(torch.randn(V, generator=gen) * 2, dim=-1)
    p = torch.cat([p1[None], _dists(gen, 1, k - 1, V, 2.0)[0]])[None].expand(n, k, V)
    q = torch.cat([q1[None], _dists(gen, 1, k, V, 2.0)[0]])[None].expand(n, k + 1, V)
    drafts = torch.stack([torch.multinomial(p[0, i], n, replacement=True, generator=gen) for i in range(k)], dim=1)
    accepted, tok = accept_sampled(drafts, p.contiguous(), q.contiguous(), gen)
    first = torch.where(accepted > 0, drafts[:, 0], tok[:, 0])
    freq = torch.bincount(first, minlength=V).double() / n
    assert float((freq - q1.double()).abs().max()) < 0.006
    assert float(0.5 * (p1 - q1).abs().sum()) > 0.1  # the draft's own distribution is far off


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
