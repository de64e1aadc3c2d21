"""Helpers shared by the GPU tests (device pools built from oracle arrays)."""

from __future__ import annotations

import numpy as np


def make_cache(device, num_layers, num_heads, head_dim, block_size, num_blocks, **kwargs):
    from specdecode_b200.kv_cache import KVCacheConfig, PagedKVCache

    config = KVCacheConfig(num_layers, num_heads, head_dim, block_size=block_size, num_blocks=num_blocks)
    return PagedKVCache(config, device=device, **kwargs)


def load_logical(cache, keys, values, key_scales, value_scales) -> None:
    """Write oracle-layout arrays ``[nb, bs, L, H, D]`` into a device pool."""
    import torch

    cache.keys_view.copy_(torch.from_numpy(np.ascontiguousarray(keys)))
    cache.values_view.copy_(torch.from_numpy(np.ascontiguousarray(values)))
    cache.key_scales_view.copy_(torch.from_numpy(np.ascontiguousarray(key_scales)))
    cache.value_scales_view.copy_(torch.from_numpy(np.ascontiguousarray(value_scales)))


def read_logical(cache):
    """Device pool back to oracle-layout numpy arrays."""
    return (cache.keys_view.contiguous().cpu().numpy(), cache.values_view.contiguous().cpu().numpy(),
            cache.key_scales_view.contiguous().cpu().numpy(), cache.value_scales_view.contiguous().cpu().numpy())


def tables_tensor(tables, device, stride=None):
    import torch

    stride = stride or max(len(t) for t in tables)
    out = np.full((len(tables), stride), -1, dtype=np.int32)
    for i, t in enumerate(tables):
        out[i, : len(t)] = t
    return torch.from_numpy(out).to(device)


def gather_oracle(keys, values, ks, vs, table, T, bs, layer):
    t = np.arange(T)
    blocks = np.asarray(table)[t // bs]
    off = t % bs
    return keys[blocks, off, layer], values[blocks, off, layer], ks[blocks, off, layer], vs[blocks, off, layer]


def random_pool(rng, nb, bs, L, H, D, scale_range=(0.005, 0.05)):
    """Codes and scales as if quantized from N(0,1)-like data."""
    keys = rng.integers(-127, 128, size=(nb, bs, L, H, D)).astype(np.int8)
    values = rng.integers(-127, 128, size=(nb, bs, L, H, D)).astype(np.int8)
    ks = rng.uniform(*scale_range, size=(nb, bs, L, H)).astype(np.float32)
    vs = rng.uniform(*scale_range, size=(nb, bs, L, H)).astype(np.float32)
    return keys, values, ks, vs
