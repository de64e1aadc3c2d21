"""Hugging Face KV-state mirror backed by the device paged INT8 cache.

The public surface is the reference's ``HuggingFacePagedCacheMirror``
(src/specdecode/hf_paged_cache.py): the class, config and stats names, the
constructor and ``from_model_config`` signatures, ``synchronize`` /
``truncate`` / ``reset`` / ``materialize_legacy_cache`` /
``materialize_like``, and the error types and messages callers match on.

The data path is the device's.  ``synchronize`` stacks the model's new
key / value rows into one ``[tokens, layers, heads, dim]`` tensor and hands
it to the fused quantize-and-append kernel (the reference copies every head
row to the host with ``.tolist()`` and quantizes per vector, :199-228).
``materialize_*`` runs the gather-dequantize kernel straight into the
template's dtype on the device (the reference rebuilds nested Python lists
on the host, :247-313).

Model geometry comes from a table of attribute spellings (Llama-style and
GPT-2-style configs); the first positive integer found wins.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

from .kv_cache import KVCacheConfig, KVCacheStats, KVQuantizer, PagedKVCache


class HuggingFacePagedCacheError(RuntimeError):
    """Raised when model cache tensors cannot be mirrored safely."""


def _is_count(value: Any) -> bool:
    return isinstance(value, int) and not isinstance(value, bool) and value > 0


@dataclass(frozen=True, slots=True)
class HuggingFacePagedCacheConfig:
    """Page geometry of a mirror; ``num_blocks`` None sizes the pool for the
    model's maximum position count."""

    block_size: int = 16
    num_blocks: int | None = None

    def __post_init__(self) -> None:
        if not _is_count(self.block_size):
            raise ValueError("block_size must be a positive integer")
        if self.num_blocks is not None and not _is_count(self.num_blocks):
            raise ValueError("num_blocks must be a positive integer when provided")


@dataclass(frozen=True, slots=True)
class HuggingFacePagedCacheMirrorStats:
    synchronized_tokens: int
    rollback_tokens: int
    resets: int
    materializations: int
    paged_cache: KVCacheStats


# Attribute spellings per geometry field, in lookup order.
_SPELLINGS = {
    "layers": ("num_hidden_layers", "n_layer"),
    "kv_heads": ("num_key_value_heads", "num_attention_heads", "n_head"),
    "attention_heads": ("num_attention_heads", "n_head"),
    "hidden": ("hidden_size", "n_embd"),
    "positions": ("max_position_embeddings", "n_positions"),
}


def _config_count(model_config: Any, field: str) -> int:
    spellings = _SPELLINGS[field]
    found = (getattr(model_config, name, None) for name in spellings)
    value = next((v for v in found if _is_count(v)), None)
    if value is None:
        raise HuggingFacePagedCacheError(f"model config must define a positive {' or '.join(spellings)}")
    return value


def _head_dim(model_config: Any) -> int:
    explicit = getattr(model_config, "head_dim", None)
    if _is_count(explicit):
        return explicit
    hidden = _config_count(model_config, "hidden")
    heads = _config_count(model_config, "attention_heads")
    if hidden % heads:
        raise HuggingFacePagedCacheError("model hidden size must be divisible by its attention-head count")
    return hidden // heads


def _layer_pairs(past_key_values: Any) -> tuple[Any, ...]:
    """The model cache as a tuple of per-layer (key, value, ...) entries:
    legacy tuples and lists as they are, cache objects through
    ``to_legacy_cache()`` or their ``layers``' keys / values."""
    if callable(getattr(past_key_values, "to_legacy_cache", None)):
        past_key_values = past_key_values.to_legacy_cache()
    elif not isinstance(past_key_values, (tuple, list)) and hasattr(past_key_values, "layers"):
        past_key_values = [(layer.keys, layer.values) for layer in past_key_values.layers]
    if not isinstance(past_key_values, (tuple, list)):
        raise HuggingFacePagedCacheError("past_key_values must be a legacy sequence or support to_legacy_cache()")
    if not past_key_values:
        raise HuggingFacePagedCacheError("past_key_values cannot be empty")
    return tuple(past_key_values)


class HuggingFacePagedCacheMirror:
    """Quantize Hugging Face K/V tensors into a device ``PagedKVCache``."""

    _SEQUENCE_ID = "model"
    _COUNTERS = ("synchronized_tokens", "rollback_tokens", "resets", "materializations")

    def __init__(self, cache: PagedKVCache) -> None:
        self.cache = cache
        cache.create_sequence(self._SEQUENCE_ID)
        self._counts = dict.fromkeys(self._COUNTERS, 0)

    @classmethod
    def from_model_config(cls, model_config: Any, config: HuggingFacePagedCacheConfig | None = None, *,
                          quantizer: KVQuantizer | None = None, device=None) -> "HuggingFacePagedCacheMirror":
        pages = config or HuggingFacePagedCacheConfig()
        layers = _config_count(model_config, "layers")
        kv_heads = _config_count(model_config, "kv_heads")
        head_dim = _head_dim(model_config)
        blocks = pages.num_blocks
        if blocks is None:
            blocks = -(-_config_count(model_config, "positions") // pages.block_size)
        geometry = KVCacheConfig(num_layers=layers, num_heads=kv_heads, head_dim=head_dim,
                                 block_size=pages.block_size, num_blocks=blocks)
        return cls(PagedKVCache(geometry, quantizer=quantizer, device=device, max_sequences=1))

    @property
    def token_count(self) -> int:
        return self.cache.sequence_length(self._SEQUENCE_ID)

    @property
    def block_table(self) -> tuple[int, ...]:
        return self.cache.block_table(self._SEQUENCE_ID)

    @property
    def stats(self) -> HuggingFacePagedCacheMirrorStats:
        return HuggingFacePagedCacheMirrorStats(paged_cache=self.cache.stats(), **self._counts)

    def _sequence_length(self, layers: tuple[Any, ...]) -> int:
        """Check every layer's key and value tensors against the cache's
        geometry and return their common sequence length."""
        config = self.cache.config
        if len(layers) != config.num_layers:
            raise HuggingFacePagedCacheError("past_key_values layer count does not match the paged cache")
        lengths = set()
        for entry in layers:
            if not isinstance(entry, (tuple, list)) or len(entry) < 2:
                raise HuggingFacePagedCacheError("each past_key_values layer must contain key and value tensors")
            for tensor in entry[:2]:
                shape = tuple(int(d) for d in tensor.shape)
                problem = None
                if len(shape) != 4:
                    problem = "KV tensors must use [batch, heads, sequence, head_dim] layout"
                elif shape[0] != 1:
                    problem = "the paged cache mirror currently supports batch size one"
                elif (shape[1], shape[3]) != (config.num_heads, config.head_dim):
                    problem = "KV tensor head geometry does not match the paged cache"
                elif lengths and shape[2] not in lengths:
                    problem = "every KV tensor must have the same sequence length"
                if problem is not None:
                    raise HuggingFacePagedCacheError(problem)
                lengths.add(shape[2])
        if not lengths:
            raise HuggingFacePagedCacheError("past_key_values has no KV tensors")
        return lengths.pop()

    def synchronize(self, past_key_values: Any) -> int:
        """Append newly produced model-cache tokens and return their count."""
        import torch

        layers = _layer_pairs(past_key_values)
        total = self._sequence_length(layers)
        start = self.token_count
        if total < start:
            raise HuggingFacePagedCacheError("model cache is shorter than its paged mirror; truncate first")
        if total == start:
            return 0

        def suffix(which: int):  # [tokens, layers, heads, dim] of the new positions
            return torch.stack([entry[which][0, :, start:total, :].transpose(0, 1) for entry in layers], dim=1)

        keys, values = suffix(0), suffix(1)
        if not keys.is_floating_point():
            raise TypeError("KV values must be real numbers")
        self.cache.append_tensor(self._SEQUENCE_ID, keys, values)
        self._counts["synchronized_tokens"] += total - start
        self.cache.validate_invariants()
        return total - start

    def materialize_legacy_cache(self, torch_module: Any, *, template: Any | None = None) -> tuple[tuple[Any, Any], ...]:
        """Dequantize the paged state into legacy ``[1, heads, seq, head_dim]``
        tensors on the device; each inherits the template's device and dtype
        (float32 on the host when no template is given, like the reference)."""
        if not (callable(getattr(torch_module, "tensor", None)) and callable(getattr(torch_module, "empty", None))):
            raise HuggingFacePagedCacheError("torch_module must provide callable tensor() and empty() factories")
        template_layers = None
        if template is not None:
            template_layers = _layer_pairs(template)
            self._sequence_length(template_layers)
        config = self.cache.config
        length = self.token_count

        def placement(layer: int, which: int):
            like = template_layers[layer][which] if template_layers is not None else None
            return (getattr(like, "dtype", None) or torch_module.float32,
                    getattr(like, "device", None) or torch_module.device("cpu"))

        def rebuild(layer: int):
            wanted = [placement(layer, which) for which in (0, 1)]
            if not length:
                return tuple(torch_module.empty((1, config.num_heads, 0, config.head_dim), dtype=dtype, device=device)
                             for dtype, device in wanted)
            # one gather per distinct dtype: [tokens, 1, heads, dim] keys and values
            gathered = {}
            for dtype, _ in wanted:
                if dtype not in gathered:
                    gathered[dtype] = self.cache.gather_sequence(self._SEQUENCE_ID, dtype, layer_begin=layer,
                                                                 layers=1)
            return tuple(gathered[dtype][which][:, 0].transpose(0, 1).unsqueeze(0).contiguous().to(device)
                         for which, (dtype, device) in enumerate(wanted))

        result = tuple(rebuild(layer) for layer in range(config.num_layers))
        self._counts["materializations"] += 1
        return result

    def materialize_like(self, torch_module: Any, template: Any) -> Any:
        """Materialize into the template's container: a list, a tuple, or a
        cache class rebuilt through its ``from_legacy_cache``."""
        legacy = self.materialize_legacy_cache(torch_module, template=template)
        if isinstance(template, (list, tuple)):
            return type(template)(legacy) if isinstance(template, list) else legacy
        factory = getattr(type(template), "from_legacy_cache", None)
        if not callable(factory):
            raise HuggingFacePagedCacheError("cache type cannot be reconstructed from legacy KV tensors")
        try:
            return factory(legacy)
        except Exception as error:
            raise HuggingFacePagedCacheError("cache type rejected reconstructed legacy KV tensors") from error

    def truncate(self, token_count: int) -> int:
        """Mirror a speculative rollback; returns the number of tokens removed."""
        before = self.token_count
        self.cache.truncate(self._SEQUENCE_ID, token_count)
        self._counts["rollback_tokens"] += before - token_count
        self.cache.validate_invariants()
        return before - token_count

    def reset(self) -> None:
        """Drop every mirrored token (the model starts a new sequence)."""
        if self.token_count:
            self.cache.truncate(self._SEQUENCE_ID, 0)
        self._counts["resets"] += 1
        self.cache.validate_invariants()
