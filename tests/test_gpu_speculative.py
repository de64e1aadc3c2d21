"""Batched speculative decoding over the paged INT8 caches: the acceptance /
resampling rule of the reference decoder (src/specdecode/decoder.py:148-257)
run for a batch with both models attending through the device kernels.

* identical draft and target models accept (almost) every proposal, with
  sampling and with greedy verification;
* speculative sampling is exact: over many sequences sharing one prompt, the
  first generated token follows the target model's next-token distribution
  over the same INT8 cache (total-variation distance within sampling noise),
  although the draft's distribution is far from it;
* the caches hold exactly the committed tokens but the last after every
  round, and ``generate`` leaves no sequence behind;
* decoding passes replayed from CUDA graphs behave as the eager ones.
"""

from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


def _llama(device, *, layers, hidden, heads, kv_heads, head_dim, vocab, init, seed):
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(seed)
    config = LlamaConfig(hidden_size=hidden, intermediate_size=2 * hidden, num_hidden_layers=layers,
                         num_attention_heads=heads, num_key_value_heads=kv_heads, head_dim=head_dim,
                         vocab_size=vocab, max_position_embeddings=512, initializer_range=init)
    return LlamaForCausalLM(config).to(device=device, dtype=torch.bfloat16).eval()


def _cache_for(device, model, sequences, tokens):
    from gpu_helpers import make_cache

    c = model.config
    blocks = sequences * (-(-tokens // 16) + 1)
    return make_cache(device, c.num_hidden_layers, c.num_key_value_heads, c.head_dim, 16, blocks,
                      max_sequences=sequences)


def _decoder(device, draft, target, sequences, tokens, **kwargs):
    from specdecode_b200.speculative import BatchedSpeculativeDecoder

    return BatchedSpeculativeDecoder(draft, target, _cache_for(device, draft, sequences, tokens),
                                     _cache_for(device, target, sequences, tokens), **kwargs)


@pytest.mark.parametrize("temperature,graphs", [(1.0, False), (0.0, False), (1.0, True)])
def test_identical_models_accept_the_window(device, temperature, graphs):
    import torch

    from specdecode_b200.speculative import DraftWindow

    model = _llama(device, layers=2, hidden=512, heads=4, kv_heads=1, head_dim=128, vocab=1000, init=0.05, seed=1)
    B, P, new = 8, 21, 24
    dec = _decoder(device, model, model, B, P + new * 7 + 16, window=DraftWindow(5, dynamic=False),
                   temperature=temperature, seed=3, cuda_graphs=graphs)
    prompts = torch.randint(0, 1000, (B, P), generator=torch.Generator().manual_seed(5))
    with torch.no_grad():
        result = dec.generate(prompts, new)
    assert [len(g) for g in result.generated_tokens] == [new] * B
    assert result.stats.acceptance_rate >= 0.95, result.stats
    for cache in (dec.draft.cache, dec.target.cache):
        assert cache.stats().allocated_blocks == 0


def test_first_token_follows_the_target_distribution(device):
    import torch

    V = 16
    draft = _llama(device, layers=1, hidden=128, heads=2, kv_heads=1, head_dim=64, vocab=V, init=0.6, seed=11)
    target = _llama(device, layers=2, hidden=256, heads=2, kv_heads=1, head_dim=128, vocab=V, init=0.6, seed=12)
    from specdecode_b200.hf_attention import PagedAttentionSession
    from specdecode_b200.speculative import DraftWindow

    B, P = 8192, 6
    prompt = torch.randint(0, V, (1, P), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        have_draft = torch.softmax(draft(prompt.to(device)).logits[0, -1].float(), dim=-1)
        dec = _decoder(device, draft, target, B, P + 16, window=DraftWindow(4, dynamic=False), temperature=1.0,
                       seed=9)
        # the target's next-token distribution over the same INT8 cache
        ref_cache = _cache_for(device, target, 1, P + 16)
        ref_cache.create_sequence("ref")
        ref = PagedAttentionSession(ref_cache)
        with ref.step(["ref"], P):
            logits = target(input_ids=prompt.to(device), position_ids=torch.arange(P, device=device)[None],
                            use_cache=False).logits
        want = torch.softmax(logits[0, -1].float(), dim=-1)
        result = dec.generate(prompt.expand(B, P), 1)
    first = torch.tensor([g[0] for g in result.generated_tokens])
    got = torch.bincount(first, minlength=V).float() / B
    tv = 0.5 * float((got - want.cpu()).abs().sum())
    tv_draft = 0.5 * float((have_draft.cpu() - want.cpu()).abs().sum())
    print("TV(empirical, target)", tv, "TV(draft, target)", tv_draft, "acceptance", result.stats.acceptance_rate)
    assert tv_draft > 0.15  # the draft alone would fail the check below
    assert tv < 0.05, (tv, got, want)


@pytest.mark.parametrize("graphs", [False, True])
def test_caches_hold_the_committed_tokens(device, graphs):
    import torch

    from specdecode_b200.speculative import BatchedSpeculativeDecoder, DraftWindow

    draft = _llama(device, layers=1, hidden=256, heads=4, kv_heads=2, head_dim=64, vocab=300, init=0.3, seed=4)
    target = _llama(device, layers=2, hidden=512, heads=4, kv_heads=1, head_dim=128, vocab=300, init=0.3, seed=5)
    B, P = 6, 9
    dec = _decoder(device, draft, target, B, P + 40 * 9 + 16, window=DraftWindow(6, min_size=4, max_size=8), seed=1,
                   cuda_graphs=graphs)
    prompts = torch.randint(0, 300, (B, P), generator=torch.Generator().manual_seed(8))
    seen = []
    original = BatchedSpeculativeDecoder._round

    def checked_round(self, ids, last, gen, stats, generated):
        out = original(self, ids, last, gen, stats, generated)
        for i, s in enumerate(ids):
            committed = P + len(generated[i])
            assert self.draft.cache.sequence_length(s) == committed - 1
            assert self.target.cache.sequence_length(s) == committed - 1
        seen.append(self.window.size)
        return out

    BatchedSpeculativeDecoder._round = checked_round
    try:
        with torch.no_grad():
            result = dec.generate(prompts, 40)
    finally:
        BatchedSpeculativeDecoder._round = original
    assert [len(g) for g in result.generated_tokens] == [40] * B
    assert all(4 <= w <= 8 for w in seen)
    s = result.stats
    assert s.accepted_tokens + s.rejected_tokens <= s.drafted_tokens
    assert s.target_tokens == B * s.verification_rounds


def test_graphed_passes_match_eager_passes(device):
    """Replaying the captured decoding passes gives the token streams that
    running them eagerly gives (greedy verification, so the streams are a
    deterministic function of the logits)."""
    import torch

    from specdecode_b200.speculative import DraftWindow

    draft = _llama(device, layers=1, hidden=256, heads=4, kv_heads=2, head_dim=64, vocab=300, init=0.3, seed=4)
    target = _llama(device, layers=2, hidden=512, heads=4, kv_heads=1, head_dim=128, vocab=300, init=0.3, seed=5)
    B, P, new = 4, 13, 20
    prompts = torch.randint(0, 300, (B, P), generator=torch.Generator().manual_seed(21))
    streams = []
    for graphs in (False, True):
        dec = _decoder(device, draft, target, B, P + new * 9 + 16, window=DraftWindow(5, dynamic=False),
                       temperature=0.0, seed=1, cuda_graphs=graphs)
        with torch.no_grad():
            dec.generate(prompts, 6)  # with graphs: eager first passes, then capture
            streams.append(dec.generate(prompts, new).generated_tokens)
    same = sum(a == b for a, b in zip(*streams))
    assert same >= B - 1, streams
