"""Batched speculative decoding over the paged INT8 caches.

The reference decoder (src/specdecode/decoder.py:69-257, ``SpeculativeDecoder``)
runs one sequence at a time: the draft proposes up to a window of tokens,
the target scores them, each proposal is accepted with probability
``min(1, p_target / p_draft)`` (src/specdecode/backends.py, native
``sd_acceptance_probabilities_f64``), the first rejected position is
resampled from the normalised residual ``max(0, p_target - p_draft)`` and a
fully accepted window earns one bonus token from the target.  Its models
rebuild a legacy cache from the paged mirror on every forward
(src/specdecode/huggingface.py:382-393).

``BatchedSpeculativeDecoder`` runs the same rule for a whole batch with both
models reading and writing their own device page pools through the
attention hook (``hf_attention``): kernel (a) appends each layer's new keys
and values, kernel (c) attends over the pool, kernel (b) rolls back the
rejected tail, and sampling stays on the device: the draft's tokens come
from the categorical-sampling kernel and the round's acceptance, first
rejection and correction or bonus sample from ``sdc_speculative_verify``
(``sampling.verify_batch``), with one device-to-host read of the round's
accepted counts and tokens per round.

Draw order.  Each sequence's round takes its uniforms from one row of 2k + 1
float64 draws of the decoder's device generator, in the reference's order
(docs/native.md:58-73 of the reference): draws 0 .. k-1 sample the k draft
tokens, draw k + i decides proposal i, and the draw after the last one used
samples the correction or the bonus.  The generator is torch's, not the
reference's ``random.Random``, so token streams are not the reference's; the
per-sequence decisions given the same draws are (tests/test_gpu_sampling.py).

Cache convention: every committed token but the last is in both caches.  A
round feeds the draft ``last, d_1 .. d_k`` one token at a time (sampling
``d_i`` from the draft's distribution after ``d_{i-1}``), feeds the target
the same ``k + 1`` tokens in one verify pass, and, with ``j`` proposals
accepted, truncates both caches to the old length plus ``j + 1``.

All sequences of a batch share the round's window; the window adapts
between rounds with the reference's rule (src/specdecode/decoder.py:47-60)
applied to the batch's mean acceptance.  Temperature 0 selects greedy
verification (accept while the draft token is the target's argmax).  No
end-of-sequence handling: every sequence generates ``max_new_tokens``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Hashable, Sequence

from .hf_attention import PagedAttentionSession
from .kv_cache import PagedKVCache
from .sampling import raise_for_status, sample_rows, verify_batch


@dataclass
class DecodeStats:
    """Counters with the meaning of the reference's ``DecodeStats``
    (src/specdecode/decoder.py:21-34), summed over the batch."""

    drafted_tokens: int = 0
    accepted_tokens: int = 0
    rejected_tokens: int = 0
    target_tokens: int = 0
    verification_rounds: int = 0

    @property
    def acceptance_rate(self) -> float:
        return self.accepted_tokens / self.drafted_tokens if self.drafted_tokens else 0.0


@dataclass
class BatchDecodeResult:
    prompt_tokens: list[list[int]]
    generated_tokens: list[list[int]]
    stats: DecodeStats = field(default_factory=DecodeStats)


@dataclass
class DraftWindow:
    """The reference's adaptive draft length (src/specdecode/decoder.py:47-60)."""

    size: int = 5
    min_size: int = 4
    max_size: int = 8
    dynamic: bool = True

    def observe(self, accepted: float, proposed: int) -> None:
        if not self.dynamic or proposed == 0:
            return
        if accepted >= proposed:
            self.size = min(self.max_size, self.size + 1)
        elif accepted * 2 < proposed:
            self.size = max(self.min_size, self.size // 2)
        else:
            self.size = max(self.min_size, self.size - 1)


def _distribution(logits, temperature: float):
    import torch

    return torch.softmax(logits.float() / temperature, dim=-1)


def accept_greedy(drafts, target_logits):
    """Greedy verification: proposals are accepted while they equal the
    target's argmax; the final token is the target's argmax after them."""
    import torch

    k = drafts.shape[1]
    best = target_logits.argmax(dim=-1)
    accepted = torch.cumprod((drafts == best[:, :k]).int(), dim=1).sum(dim=1)
    return accepted, best.gather(1, accepted[:, None])


class BatchedSpeculativeDecoder:
    """Speculative decoding of a batch with a draft and a target transformers
    causal LM, each attending over its own ``PagedKVCache``.

    ``draft_cache`` / ``target_cache`` must have the models' layer count, KV
    heads and head_dim and room for every sequence's prompt plus generated
    tokens plus one window.  Sequences are registered in the caches by the
    decoder (ids ``(tag, i)``) and removed when ``generate`` returns.
    """

    def __init__(self, draft_model, target_model, draft_cache: PagedKVCache, target_cache: PagedKVCache, *,
                 window: DraftWindow | None = None, temperature: float = 1.0, seed: int = 0,
                 cuda_graphs: bool = False) -> None:
        if draft_model.config.vocab_size != target_model.config.vocab_size:
            raise ValueError("draft and target models must share a vocabulary")
        if temperature < 0 or not math.isfinite(temperature):
            raise ValueError("temperature must be finite and non-negative")
        self.draft_model = draft_model
        self.target_model = target_model
        self.draft = PagedAttentionSession(draft_cache)
        self.target = PagedAttentionSession(target_cache)
        # the device fault words are read once per round, after the round's
        # device-to-host read has synchronised anyway
        self.draft.check_each_step = False
        self.target.check_each_step = False
        self.window = window or DraftWindow()
        self.temperature = float(temperature)
        self.seed = int(seed)
        self._tag = 0
        # CUDA graphs of the decoding passes (draft single-token steps and
        # target verify windows), one per (model, tokens per sequence),
        # captured the second time a shape runs and replayed after that
        self.cuda_graphs = bool(cuda_graphs)
        self._graphs: dict = {}
        self._seen: set = set()
        self._bound = 0
        self._batch = 0
        self._sampling_status = None
        for model in (draft_model, target_model):
            model.set_attn_implementation(PagedAttentionSession.NAME)

    # -- model passes ---------------------------------------------------------
    def _forward(self, session: PagedAttentionSession, model, ids: Sequence[Hashable], tokens, keep: int):
        """Feeds ``tokens [B, n]`` to ``model`` after each sequence's cached
        tokens; returns the logits of the last ``keep`` positions."""
        import torch

        cache = session.cache
        B, n = tokens.shape
        lengths = torch.tensor([cache.sequence_length(s) for s in ids], device=tokens.device)
        positions = lengths[:, None] + torch.arange(n, device=tokens.device)[None, :]
        with session.step(ids, n):
            out = model(input_ids=tokens, position_ids=positions, use_cache=False, logits_to_keep=keep)
        return out.logits

    def _graphed_forward(self, session: PagedAttentionSession, model, ids: Sequence[Hashable], tokens, keep: int):
        """``_forward`` through a CUDA graph: the host plans the step
        (``fixed_step`` reserves the slots and copies them, the token ids and
        positions into the graph's own buffers) and replays the recorded
        passes; the first pass of a shape runs eagerly, the second is
        captured."""
        import torch

        cache = session.cache
        B, n = tokens.shape
        key = (id(session), n, keep)
        g = self._graphs.get(key)
        if g is None:
            g = {"tokens": torch.zeros((B, n), dtype=torch.long, device=tokens.device),
                 "positions": torch.zeros((B, n), dtype=torch.long, device=tokens.device),
                 "slots": torch.zeros(B * n, dtype=torch.int64, device=tokens.device),
                 "graph": None, "logits": None}
            self._graphs[key] = g
        # a captured graph reads the table / length rows at fixed addresses
        rows_at = cache.block_tables[cache.table_row(ids[0])].data_ptr()
        if g.get("rows_at") != rows_at:
            g["graph"], g["rows_at"] = None, rows_at
            self._seen.discard(key)
        g["tokens"].copy_(tokens)
        with session.fixed_step(ids, n, g["slots"], self._bound):
            # positions from the device lengths, which now include the n new
            # tokens (no host-to-device copy, so no synchronisation)
            lens = session.step_context_lens
            g["positions"].copy_(lens[:, None].long() - n + torch.arange(n, device=tokens.device)[None, :])
            if g["graph"] is not None:
                g["graph"].replay()
            elif key not in self._seen:
                self._seen.add(key)
                g["logits"] = model(input_ids=g["tokens"], position_ids=g["positions"], use_cache=False,
                                    logits_to_keep=keep).logits
            else:
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    g["logits"] = model(input_ids=g["tokens"], position_ids=g["positions"], use_cache=False,
                                        logits_to_keep=keep).logits
                g["graph"] = graph
                graph.replay()
        return g["logits"]

    def _prepare_graphs(self, B: int, bound: int) -> None:
        """Fixed workspaces for the graphed passes (sized for every window the
        decoder can use) and a fresh set of graphs when the batch or the
        context bound changes."""
        if B == self._batch and bound <= self._bound:
            return
        self._graphs.clear()
        self._seen.clear()
        self._batch, self._bound = B, bound
        for session, model in ((self.draft, self.draft_model), (self.target, self.target_model)):
            c = model.config
            need = max(session.attention.workspace_bytes(B, c.num_attention_heads, w, bound)
                       for w in range(1, self.window.max_size + 2))
            session.release_fixed_workspace()
            session.reserve_fixed_workspace(need)

    def _prefill(self, session: PagedAttentionSession, model, ids, tokens, chunk: int) -> None:
        for i in range(0, tokens.shape[1], chunk):
            self._forward(session, model, ids, tokens[:, i:i + chunk], 1)

    # -- decoding -------------------------------------------------------------
    def generate(self, prompt_tokens, max_new_tokens: int, *, prefill_chunk: int = 512,
                 prefill_done=None) -> BatchDecodeResult:
        """``prompt_tokens``: int64 ``[B, P]`` (device or host), P >= 1.
        ``prefill_done``: an optional CUDA event recorded once both caches
        hold the prompts (before the first round)."""
        import torch

        device = self.target.cache.device
        prompts = torch.as_tensor(prompt_tokens, dtype=torch.long).to(device)
        if prompts.dim() != 2 or prompts.shape[1] < 1:
            raise ValueError("prompt_tokens must be [batch, prompt_length] with prompt_length >= 1")
        B = int(prompts.shape[0])
        self._tag += 1
        ids = [(self._tag, i) for i in range(B)]
        gen = torch.Generator(device=device).manual_seed(self.seed)
        stats = DecodeStats()
        generated = [[] for _ in range(B)]
        for cache in (self.draft.cache, self.target.cache):
            for s in ids:
                cache.create_sequence(s)
        try:
            if prompts.shape[1] > 1:
                ctx = prompts[:, :-1]
                self._prefill(self.draft, self.draft_model, ids, ctx, prefill_chunk)
                self._prefill(self.target, self.target_model, ids, ctx, prefill_chunk)
                self.draft.cache.check_status()
                self.target.cache.check_status()
            last = prompts[:, -1:]
            if self.cuda_graphs:
                # a round adds 1 to max_size + 1 tokens to every sequence and
                # rounds continue until the slowest has max_new_tokens, so no
                # context grows beyond this bound during the call
                step = self.window.max_size + 1
                self._prepare_graphs(B, int(prompts.shape[1]) + int(max_new_tokens) * step + step + 1)
            if prefill_done is not None:
                prefill_done.record()
            while min(len(g) for g in generated) < max_new_tokens:
                last = self._round(ids, last, gen, stats, generated)
        finally:
            for cache in (self.draft.cache, self.target.cache):
                for s in ids:
                    cache.remove_sequence(s)
        return BatchDecodeResult(prompts.cpu().tolist(), [g[:max_new_tokens] for g in generated], stats)

    def _round(self, ids, last, gen, stats: DecodeStats, generated) -> "torch.Tensor":
        import torch

        k = self.window.size
        B = last.shape[0]
        greedy = self.temperature == 0.0
        dlen = [self.draft.cache.sequence_length(s) for s in ids]
        tlen = [self.target.cache.sequence_length(s) for s in ids]
        # draft: k proposals, one token per pass; d_k is fed too so that a
        # fully accepted window leaves the draft cache complete
        feed = last
        proposals, draft_probs = [], []
        forward = self._graphed_forward if self.cuda_graphs else self._forward
        if not greedy:
            # the round's draws: k draft samples, then k + 1 for verification
            draws = torch.rand((B, 2 * k + 1), generator=gen, device=last.device, dtype=torch.float64)
            if self._sampling_status is None or self._sampling_status.device != last.device:
                self._sampling_status = torch.zeros(1, dtype=torch.int32, device=last.device)
        for i in range(k + 1):
            logits = forward(self.draft, self.draft_model, ids, feed, 1)[:, -1]
            if i == k:
                break
            if greedy:
                tok = logits.argmax(dim=-1, keepdim=True)
            else:
                p = _distribution(logits, self.temperature)
                tok = sample_rows(p, draws[:, i], status=self._sampling_status)[:, None]
                draft_probs.append(p)
            proposals.append(tok)
            feed = tok
        drafts = torch.cat(proposals, dim=1)  # [B, k]
        # target: one verify pass over last, d_1 .. d_k
        verify = torch.cat([last, drafts], dim=1)
        tlogits = forward(self.target, self.target_model, ids, verify, k + 1)  # [B, k + 1, V]
        if greedy:
            accepted, new_tok = accept_greedy(drafts, tlogits)
        else:
            accepted, token, _ = verify_batch(_distribution(tlogits, self.temperature),
                                              torch.stack(draft_probs, dim=1), drafts, draws[:, k:],
                                              status=self._sampling_status)
            new_tok = token[:, None]
        host = torch.cat([accepted[:, None], drafts, new_tok], dim=1).cpu().tolist()
        self.draft.cache.check_status()
        self.target.cache.check_status()
        if not greedy:
            raise_for_status(self._sampling_status, "speculative sampling")
        keep_d, keep_t = [], []
        for b, row in enumerate(host):
            j = int(row[0])
            generated[b].extend(row[1:1 + j])
            generated[b].append(int(row[1 + k]))
            keep_d.append(dlen[b] + 1 + j)
            keep_t.append(tlen[b] + 1 + j)
            stats.accepted_tokens += j
            stats.rejected_tokens += int(j < k)
        self.draft.cache.truncate_batch(ids, keep_d)
        self.target.cache.truncate_batch(ids, keep_t)
        stats.drafted_tokens += B * k
        stats.target_tokens += B
        stats.verification_rounds += 1
        self.window.observe(sum(int(r[0]) for r in host) / B, k)
        return new_tok
