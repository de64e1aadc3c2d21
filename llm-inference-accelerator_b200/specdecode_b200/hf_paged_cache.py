"""Hugging Face KV-state mirror backed by the device paged INT8 cache.

Same surface and errors as the reference's ``HuggingFacePagedCacheMirror``
(src/specdecode/hf_paged_cache.py): geometry from a model config,
``synchronize(past_key_values)`` appends newly produced tokens,
``truncate`` mirrors speculative rollback, ``reset``, stats, and
``materialize_legacy_cache`` / ``materialize_like`` rebuild
``[1, heads, seq, head_dim]`` tensors from the INT8 pages.

What changes is the data path.  ``synchronize`` hands the model's K/V
tensors to the fused quantize-and-append kernel directly (the reference
copies them to the host with ``.tolist()`` and quantizes per head vector,
:199-228).  ``materialize_*`` dequantizes on the device with the
gather-dequantize kernel straight into the template's dtype (the
reference rebuilds nested Python lists on the host, :247-313).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

from .kv_cache import KVCacheConfig, KVCacheStats, KVQuantizer, PagedKVCache


class HuggingFacePagedCacheError(RuntimeError):
    """Raised when model cache tensors cannot be mirrored safely."""


@dataclass(frozen=True, slots=True)
class HuggingFacePagedCacheConfig:
    block_size: int = 16
    num_blocks: int | None = None

    def __post_init__(self) -> None:
        if isinstance(self.block_size, bool) or not isinstance(self.block_size, int) or self.block_size < 1:
            raise ValueError("block_size must be a positive integer")
        if self.num_blocks is not None and (
                isinstance(self.num_blocks, bool) or not isinstance(self.num_blocks, int) or self.num_blocks < 1):
            raise ValueError("num_blocks must be a positive integer when provided")


@dataclass(frozen=True, slots=True)
class HuggingFacePagedCacheMirrorStats:
    synchronized_tokens: int
    rollback_tokens: int
    resets: int
    materializations: int
    paged_cache: KVCacheStats


def _positive_config_int(model_config: Any, *names: str) -> int:
    for name in names:
        value = getattr(model_config, name, None)
        if isinstance(value, int) and not isinstance(value, bool) and value > 0:
            return value
    raise HuggingFacePagedCacheError(f"model config must define a positive {' or '.join(names)}")


class HuggingFacePagedCacheMirror:
    """Quantize Hugging Face K/V tensors into a device ``PagedKVCache``."""

    _SEQUENCE_ID = "model"

    def __init__(self, cache: PagedKVCache) -> None:
        self.cache = cache
        self.cache.create_sequence(self._SEQUENCE_ID)
        self._synchronized_tokens = 0
        self._rollback_tokens = 0
        self._resets = 0
        self._materializations = 0

    @classmethod
    def from_model_config(cls, model_config: Any, config: HuggingFacePagedCacheConfig | None = None, *,
                          quantizer: KVQuantizer | None = None, device=None) -> "HuggingFacePagedCacheMirror":
        mirror_config = config or HuggingFacePagedCacheConfig()
        num_layers = _positive_config_int(model_config, "num_hidden_layers", "n_layer")
        num_heads = _positive_config_int(model_config, "num_key_value_heads", "num_attention_heads", "n_head")
        head_dim = getattr(model_config, "head_dim", None)
        if not isinstance(head_dim, int) or isinstance(head_dim, bool) or head_dim < 1:
            hidden = _positive_config_int(model_config, "hidden_size", "n_embd")
            attention_heads = _positive_config_int(model_config, "num_attention_heads", "n_head")
            if hidden % attention_heads:
                raise HuggingFacePagedCacheError("model hidden size must be divisible by its attention-head count")
            head_dim = hidden // attention_heads
        num_blocks = mirror_config.num_blocks
        if num_blocks is None:
            maximum = _positive_config_int(model_config, "max_position_embeddings", "n_positions")
            num_blocks = (maximum + mirror_config.block_size - 1) // mirror_config.block_size
        cache_config = KVCacheConfig(num_layers=num_layers, num_heads=num_heads, head_dim=head_dim,
                                     block_size=mirror_config.block_size, num_blocks=num_blocks)
        return cls(PagedKVCache(cache_config, quantizer=quantizer, device=device, max_sequences=1))

    @property
    def token_count(self) -> int:
        return self.cache.sequence_length(self._SEQUENCE_ID)

    @property
    def block_table(self) -> tuple[int, ...]:
        return self.cache.block_table(self._SEQUENCE_ID)

    @property
    def stats(self) -> HuggingFacePagedCacheMirrorStats:
        return HuggingFacePagedCacheMirrorStats(
            synchronized_tokens=self._synchronized_tokens, rollback_tokens=self._rollback_tokens,
            resets=self._resets, materializations=self._materializations, paged_cache=self.cache.stats())

    @staticmethod
    def _legacy_layers(past_key_values: Any) -> tuple[Any, ...]:
        convert = getattr(past_key_values, "to_legacy_cache", None)
        if callable(convert):
            past_key_values = convert()
        elif not isinstance(past_key_values, (tuple, list)) and hasattr(past_key_values, "layers"):
            past_key_values = [(layer.keys, layer.values) for layer in past_key_values.layers]
        if not isinstance(past_key_values, (tuple, list)):
            raise HuggingFacePagedCacheError(
                "past_key_values must be a legacy sequence or support to_legacy_cache()")
        layers = tuple(past_key_values)
        if not layers:
            raise HuggingFacePagedCacheError("past_key_values cannot be empty")
        return layers

    def _validate_layers(self, layers: tuple[Any, ...]) -> int:
        config = self.cache.config
        if len(layers) != config.num_layers:
            raise HuggingFacePagedCacheError("past_key_values layer count does not match the paged cache")
        sequence_length = None
        for layer in layers:
            if not isinstance(layer, (tuple, list)) or len(layer) < 2:
                raise HuggingFacePagedCacheError("each past_key_values layer must contain key and value tensors")
            for tensor in layer[:2]:
                shape = tuple(int(d) for d in tensor.shape)
                if len(shape) != 4:
                    raise HuggingFacePagedCacheError("KV tensors must use [batch, heads, sequence, head_dim] layout")
                if shape[0] != 1:
                    raise HuggingFacePagedCacheError("the paged cache mirror currently supports batch size one")
                if shape[1] != config.num_heads or shape[3] != config.head_dim:
                    raise HuggingFacePagedCacheError("KV tensor head geometry does not match the paged cache")
                if sequence_length is None:
                    sequence_length = shape[2]
                elif sequence_length != shape[2]:
                    raise HuggingFacePagedCacheError("every KV tensor must have the same sequence length")
        if sequence_length is None:
            raise HuggingFacePagedCacheError("past_key_values has no KV tensors")
        return sequence_length

    def synchronize(self, past_key_values: Any) -> int:
        """Append newly produced model-cache tokens and return their count."""
        import torch

        layers = self._legacy_layers(past_key_values)
        sequence_length = self._validate_layers(layers)
        current = self.token_count
        if sequence_length < current:
            raise HuggingFacePagedCacheError("model cache is shorter than its paged mirror; truncate first")
        if sequence_length == current:
            return 0
        # [tokens, layers, heads, dim] views of the new suffix, one copy each.
        keys = torch.stack([layer[0][0, :, current:sequence_length, :].transpose(0, 1) for layer in layers], dim=1)
        values = torch.stack([layer[1][0, :, current:sequence_length, :].transpose(0, 1) for layer in layers], dim=1)
        if not keys.is_floating_point():
            raise TypeError("KV values must be real numbers")
        self.cache.append_tensor(self._SEQUENCE_ID, keys, values)
        appended = sequence_length - current
        self._synchronized_tokens += appended
        self.cache.validate_invariants()
        return appended

    def materialize_legacy_cache(self, torch_module: Any, *, template: Any | None = None) -> tuple[tuple[Any, Any], ...]:
        """Dequantize the paged state into legacy ``[1, heads, seq, head_dim]``
        tensors on the device; each inherits the template's device and dtype
        (float32 on the host when no template is given, like the reference)."""
        tensor = getattr(torch_module, "tensor", None)
        empty = getattr(torch_module, "empty", None)
        if not callable(tensor) or not callable(empty):
            raise HuggingFacePagedCacheError("torch_module must provide callable tensor() and empty() factories")
        template_layers = None
        if template is not None:
            template_layers = self._legacy_layers(template)
            self._validate_layers(template_layers)
        config = self.cache.config
        length = self.token_count
        layers = []
        for layer_index in range(config.num_layers):
            targets = []
            for kv in (0, 1):
                t = template_layers[layer_index][kv] if template_layers is not None else None
                dtype = getattr(t, "dtype", None) or torch_module.float32
                device = getattr(t, "device", None) or torch_module.device("cpu")
                targets.append((dtype, device))
            if length:
                k, v = self.cache.gather_sequence(self._SEQUENCE_ID, targets[0][0], layer_begin=layer_index, layers=1)
                if targets[1][0] != targets[0][0]:
                    _, v = self.cache.gather_sequence(self._SEQUENCE_ID, targets[1][0], layer_begin=layer_index,
                                                      layers=1)
                key_tensor = k[:, 0].transpose(0, 1).unsqueeze(0).contiguous().to(targets[0][1])
                value_tensor = v[:, 0].transpose(0, 1).unsqueeze(0).contiguous().to(targets[1][1])
            else:
                shape = (1, config.num_heads, 0, config.head_dim)
                key_tensor = empty(shape, dtype=targets[0][0], device=targets[0][1])
                value_tensor = empty(shape, dtype=targets[1][0], device=targets[1][1])
            layers.append((key_tensor, value_tensor))
        self._materializations += 1
        return tuple(layers)

    def materialize_like(self, torch_module: Any, template: Any) -> Any:
        legacy = self.materialize_legacy_cache(torch_module, template=template)
        if isinstance(template, list):
            return list(legacy)
        if isinstance(template, tuple):
            return legacy
        factory = getattr(type(template), "from_legacy_cache", None)
        if not callable(factory):
            raise HuggingFacePagedCacheError("cache type cannot be reconstructed from legacy KV tensors")
        try:
            return factory(legacy)
        except Exception as error:
            raise HuggingFacePagedCacheError("cache type rejected reconstructed legacy KV tensors") from error

    def truncate(self, token_count: int) -> int:
        current = self.token_count
        self.cache.truncate(self._SEQUENCE_ID, token_count)
        removed = current - token_count
        self._rollback_tokens += removed
        self.cache.validate_invariants()
        return removed

    def reset(self) -> None:
        if self.token_count:
            self.cache.truncate(self._SEQUENCE_ID, 0)
        self._resets += 1
        self.cache.validate_invariants()
