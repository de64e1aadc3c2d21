"""Hugging Face attention hook over the paged INT8 cache.

Replaces the reference's CPU reconstruct path for a transformers model
(src/specdecode/huggingface.py:382-393 rebuilds a legacy cache from the
paged mirror with ``materialize_like`` before every forward, and
src/specdecode/hf_paged_cache.py:199-232 mirrors new keys / values through
``.tolist()``): with the hook installed, every attention layer of the model
quantizes its new keys and values straight into the device page pool
(kernel (a), one layer at a time) and attends over the pool with the fused
paged attention kernel (c).  The model runs with ``use_cache=False``; the
page pool is its only cache.

Usage::

    session = PagedAttentionSession(cache)          # a PagedKVCache with the model's geometry
    model.set_attn_implementation(PagedAttentionSession.NAME)
    with session.step(sequence_ids, new_tokens):
        logits = model(input_ids, position_ids=positions, use_cache=False).logits

``step`` reserves the new tokens' slots for every layer first.  Each listed
sequence contributes the same number of new tokens, its queries sit at the
end of its own context (the paged cache carries every sequence's length, so
padding masks are neither needed nor supported), and positions must be
``range(length, length + new_tokens)`` per sequence.  Queries too large for
one kernel call (a prefill: query heads per KV head x new tokens above 64
rows) run as consecutive causal windows, each over the context up to its
last position.
"""

from __future__ import annotations

import contextlib
import math
from typing import Hashable, Sequence

from .cuda_kv_cache import PagedVerifyAttention
from .kv_cache import LayerwiseAppend, PagedKVCache

_ACTIVE: list["PagedAttentionSession"] = []
_MAX_ROWS = 64  # query rows per KV head one kernel call serves


class PagedAttentionError(RuntimeError):
    """The model's attention call does not match the paged cache."""


def _attention_forward(module, query, key, value, attention_mask, dropout: float = 0.0, scaling=None, **kwargs):
    if not _ACTIVE:
        raise PagedAttentionError("paged attention used outside PagedAttentionSession.step()")
    return _ACTIVE[-1].forward(module, query, key, value, scaling, dropout)


def _no_mask(*args, **kwargs):
    return None


def register() -> None:
    """Register the hook's attention and (empty) mask functions with transformers."""
    from transformers import AttentionInterface
    from transformers.masking_utils import AttentionMaskInterface

    AttentionInterface.register(PagedAttentionSession.NAME, _attention_forward)
    AttentionMaskInterface.register(PagedAttentionSession.NAME, _no_mask)


class PagedAttentionSession:
    """Routes a model's attention layers through one ``PagedKVCache``."""

    NAME = "specdecode_paged"

    def __init__(self, cache: PagedKVCache) -> None:
        self.cache = cache
        self.attention = PagedVerifyAttention.for_cache(cache)
        self._pending = None
        self._ids: list[Hashable] = []
        self._new = 0
        self._inputs = None
        # optional device timing of the attention calls: (start, end, algorithmic bytes)
        self.timed = False
        self.timings: list = []
        # with timing on: device cycles to hold the stream before each timed
        # call's start event (torch.cuda._sleep), so that its launches are
        # queued before the event runs and the interval is device time only
        self.timing_hold_cycles = 0
        self._lengths: list[int] = []
        # fixed_step state: attention with its own workspace, so that device
        # addresses recorded in a CUDA graph stay valid
        self._fixed_attention: PagedVerifyAttention | None = None
        self._active_attention = self.attention
        # read the cache's device fault word after every step (a device
        # synchronisation); a caller that checks it itself less often, once
        # it synchronises anyway, turns this off
        self.check_each_step = True
        register()

    @contextlib.contextmanager
    def step(self, sequence_ids: Sequence[Hashable], new_tokens: int):
        """Reserve ``new_tokens`` slots per sequence, then run the model inside
        the block.  Every layer must be written by the forward pass."""
        if self._pending is not None:
            raise PagedAttentionError("a step is already open")
        self._ids = list(sequence_ids)
        self._new = int(new_tokens)
        self._pending = self.cache.reserve(self._ids, self._new)
        self._inputs = self.cache.attention_inputs(self._ids)
        if self.timed:
            self._lengths = [self.cache.sequence_length(s) for s in self._ids]
        _ACTIVE.append(self)
        try:
            yield self
        finally:
            _ACTIVE.remove(self)
            self._pending = None
            self._inputs = None
        if self.check_each_step:
            self.cache.check_status()

    @property
    def step_context_lens(self):
        """Device int32 context lengths of the open step's sequences,
        including the step's new tokens."""
        if self._inputs is None:
            raise PagedAttentionError("no step is open")
        return self._inputs[1]

    def release_fixed_workspace(self) -> None:
        """Drop the ``fixed_step`` workspace (graphs that recorded its address
        must be dropped with it)."""
        self._fixed_attention = None

    def reserve_fixed_workspace(self, nbytes: int) -> None:
        """Size the workspace used inside ``fixed_step`` once, before any CUDA
        graph is captured: a captured graph keeps the address."""
        import torch

        if self._fixed_attention is None:
            self._fixed_attention = PagedVerifyAttention.for_cache(self.cache)
        fa = self._fixed_attention
        if fa._workspace is None or fa._workspace.numel() < nbytes:
            if fa._workspace is not None:
                raise PagedAttentionError("the fixed workspace is already in use and cannot grow")
            fa._workspace = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=self.cache.device)

    @contextlib.contextmanager
    def fixed_step(self, sequence_ids: Sequence[Hashable], new_tokens: int, slots, max_len: int):
        """``step`` with device addresses that do not change from step to
        step, for a forward pass captured once in a CUDA graph and replayed:
        the reserved slots are copied into ``slots`` (int64 ``[B *
        new_tokens]``), attention reads the cache's own block-table and
        length rows (the sequences must occupy consecutive rows) with the
        context bound ``max_len`` (at least every sequence's new length),
        and its workspace is the one ``reserve_fixed_workspace`` sized."""
        if self._pending is not None:
            raise PagedAttentionError("a step is already open")
        if self._fixed_attention is None or self._fixed_attention._workspace is None:
            raise PagedAttentionError("reserve_fixed_workspace must size the workspace first")
        self._ids = list(sequence_ids)
        self._new = int(new_tokens)
        pending = self.cache.reserve(self._ids, self._new)
        slots[:pending.tokens].copy_(pending.slots)
        self._pending = LayerwiseAppend(pending.plan, slots, pending.tokens)
        tables, lens, longest = self.cache.attention_inputs(self._ids)
        if tables.data_ptr() != self.cache.block_tables[self.cache.table_row(self._ids[0])].data_ptr():
            self._pending = None
            raise PagedAttentionError("fixed_step needs the sequences in consecutive cache rows")
        if longest > max_len:
            self._pending = None
            raise PagedAttentionError(f"a sequence is {longest} tokens long, beyond the bound {max_len}")
        self._inputs = (tables, lens, int(max_len))
        self._active_attention = self._fixed_attention
        _ACTIVE.append(self)
        try:
            yield self
        finally:
            _ACTIVE.remove(self)
            self._pending = None
            self._inputs = None
            self._active_attention = self.attention
        if self.check_each_step:
            self.cache.check_status()

    def forward(self, module, query, key, value, scaling, dropout):
        import torch

        if dropout:
            raise PagedAttentionError("paged attention has no dropout")
        B, Hq, q_len, D = (int(d) for d in query.shape)
        Hkv = int(key.shape[1])
        if B != len(self._ids) or q_len != self._new:
            raise PagedAttentionError(
                f"attention over {B} x {q_len} new tokens, but the step reserved {len(self._ids)} x {self._new}")
        if scaling is not None and not math.isclose(float(scaling), 1.0 / math.sqrt(D), rel_tol=1e-6):
            raise PagedAttentionError("paged attention uses the 1/sqrt(head_dim) softmax scale")
        layer = int(module.layer_idx)
        # this layer's new keys / values, sequence-major: [B * q_len, Hkv, D]
        k = key.transpose(1, 2).reshape(B * q_len, Hkv, D)
        v = value.transpose(1, 2).reshape(B * q_len, Hkv, D)
        self.cache.write_layer(self._pending, layer, k, v)
        tables, lens, max_len = self._inputs
        group = Hq // Hkv
        window = max(1, _MAX_ROWS // group)
        if q_len <= window:
            kind = "decode" if q_len == 1 else "verify"
            out = self._attend(query.contiguous(), tables, lens, max_len, layer, 0, kind)
        else:
            parts = []
            for j in range(0, q_len, window):
                w = min(window, q_len - j)
                behind = q_len - (j + w)  # new tokens after this window
                parts.append(self._attend(query[:, :, j:j + w].contiguous(), tables, lens - behind,
                                          max_len - behind, layer, behind, "prefill"))
            out = torch.cat(parts, dim=2)
        return out.transpose(1, 2).contiguous(), None

    def _attend(self, query, tables, lens, max_len, layer, behind, kind):
        if not self.timed or self._active_attention is not self.attention:
            return self._active_attention(query, tables, lens, max_len, layer)
        import torch

        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if self.timing_hold_cycles > 0:
            torch.cuda._sleep(int(self.timing_hold_cycles))
        start.record()
        out = self.attention(query, tables, lens, max_len, layer)
        end.record()
        B, Hq, w, D = (int(d) for d in query.shape)
        cfg = self.cache.config
        per_token = 2 * cfg.num_heads * D + 2 * cfg.num_heads * 4
        nbytes = sum((t - behind) * per_token + -(-(t - behind) // cfg.block_size) * 4 for t in self._lengths)
        nbytes += 2 * B * Hq * w * D * query.element_size()
        self.timings.append((start, end, nbytes, kind))
        return out

    def attention_time(self) -> tuple[float, int]:
        """Milliseconds and algorithmic bytes of the timed attention calls so
        far (synchronises the device)."""
        import torch

        torch.cuda.synchronize()
        return sum(t[0].elapsed_time(t[1]) for t in self.timings), sum(t[2] for t in self.timings)

    def attention_time_by_kind(self) -> dict[str, tuple[int, float, int]]:
        """Per kind of call ("prefill" windows of a prompt, single-token
        "decode" steps, multi-token "verify" windows): the timed calls' count,
        milliseconds and algorithmic bytes (synchronises the device)."""
        import torch

        torch.cuda.synchronize()
        out: dict[str, tuple[int, float, int]] = {}
        for start, end, nbytes, kind in self.timings:
            n, ms, b = out.get(kind, (0, 0.0, 0))
            out[kind] = (n + 1, ms + start.elapsed_time(end), b + nbytes)
        return out
