"""Device storage binding, the reference-signature attention entry point and
the Hugging Face mirror (tests/test_cuda.py:510-691 and
tests/test_hf_paged_cache.py:136-235 of the reference, on a real device)."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest

from gpu_helpers import make_cache
from oracle.attention import attention_fp64
from oracle.quant import quantize_rows

pytestmark = pytest.mark.gpu

D = 16


@pytest.fixture()
def runtime(device):
    """The reference's own CudaExecutionRuntime (src/specdecode/cuda.py),
    unchanged, from the copy of its package in oracle/_ref/: the storage
    and attention entry points take the caller's runtime as it is."""
    from oracle.reference_runs import ReferenceUnavailable, reference_package

    try:
        reference_package()
    except ReferenceUnavailable as error:
        pytest.skip(str(error))
    from specdecode.cuda import CudaExecutionRuntime, CudaRuntimeConfig

    return CudaExecutionRuntime(CudaRuntimeConfig(device=f"cuda:{device.index}"))


def _entry(seed):
    import torch

    keys = torch.full((1, 1, 1, D), float(seed))
    keys[..., 1::2] = -float(seed)
    values = torch.arange(D, dtype=torch.float32).reshape(1, 1, 1, D) + seed
    return keys, values


def _append(cache, seq, *seeds):
    import torch

    ks, vs = zip(*(_entry(s) for s in seeds))
    cache.append_tensor(seq, torch.cat(ks), torch.cat(vs))


def test_storage_layout_and_incremental_stats(device, runtime):
    from specdecode_b200.cuda_kv_cache import CudaPagedKVCacheStorage

    cache = make_cache(device, 1, 1, D, 2, 3)
    cache.create_sequence("model")
    storage = CudaPagedKVCacheStorage(cache.config, runtime)
    _append(cache, "model", 1, 2, 3)
    view = storage.synchronize(cache, "model").wait()
    assert tuple(view.keys.shape) == (3, 2, 1, 1, D)
    assert tuple(view.key_scales.shape) == (3, 2, 1, 1)
    assert view.block_table.cpu().tolist() == [0, 1]
    assert view.token_count == 3
    flat = view.keys.reshape(6, D)[:3].cpu().numpy()
    for i in range(3):
        assert flat[i].tolist() == list(cache.read_quantized_token("model", i).keys[0][0].values)
    stats = storage.stats
    assert (stats.synchronizations, stats.uploaded_tokens, stats.active_tokens, stats.active_blocks) == (1, 3, 3, 2)
    assert stats.device_storage_bytes == cache.config.capacity_tokens * cache.config.quantized_bytes_per_token


def test_storage_rollback_clears_and_rewrites(device, runtime):
    from specdecode_b200.cuda_kv_cache import CudaPagedKVCacheError, CudaPagedKVCacheStorage

    cache = make_cache(device, 1, 1, D, 2, 3)
    cache.create_sequence("model")
    storage = CudaPagedKVCacheStorage(cache.config, runtime)
    _append(cache, "model", 1, 2, 3, 4)
    storage.synchronize(cache, "model").wait()
    cache.truncate("model", 1)
    view = storage.synchronize(cache, "model").wait()
    assert view.token_count == 1 and view.block_table.cpu().tolist() == [0]
    assert int(view.keys.reshape(6, D)[1:4].abs().sum()) == 0  # cleared slots
    assert float(view.key_scales.reshape(6)[1:4].abs().sum()) == 0.0
    assert storage.stats.cleared_tokens == 3
    _append(cache, "model", 8, 9)
    storage.synchronize(cache, "model").wait()
    assert storage.stats.uploaded_tokens == 6
    cache.create_sequence("other")
    with pytest.raises(CudaPagedKVCacheError):
        storage.synchronize(cache, "other")


def test_submit_paged_attention_matches_oracle(device, runtime):
    """Offset block table [1, 2], window 2, GQA 2 query heads on 1 KV head
    (the reference's tests/test_cuda.py:611-676 with head_dim 16)."""
    import torch

    from specdecode_b200.cuda_kv_cache import CudaPagedAttentionError, CudaPagedKVCacheStorage, submit_paged_attention

    cache = make_cache(device, 1, 1, D, 2, 3)
    cache.create_sequence("occupied")
    _append(cache, "occupied", 99, 100)
    cache.create_sequence("model")
    _append(cache, "model", 1, 2, 3)
    storage = CudaPagedKVCacheStorage(cache.config, runtime)
    synced = storage.synchronize(cache, "model")
    assert synced.result.block_table.cpu().tolist() == [1, 2]
    q = torch.zeros((1, 2, 2, D))
    q[0, :, 0, 0] = 1.0
    q[0, :, 1, 1] = 1.0
    q = q.to(device)
    out = submit_paged_attention(runtime, q, synced.result, 0, wait_for=(synced,)).wait()
    assert tuple(out.shape) == (1, 2, 2, D)
    k = np.stack([np.asarray(cache.read_quantized_token("model", i).keys[0][0].values) for i in range(3)])
    v = np.stack([np.asarray(cache.read_quantized_token("model", i).values[0][0].values) for i in range(3)])
    ks = np.array([cache.read_quantized_token("model", i).keys[0][0].scale for i in range(3)], np.float32)
    vs = np.array([cache.read_quantized_token("model", i).values[0][0].scale for i in range(3)], np.float32)
    exact = attention_fp64(q[0].cpu().numpy(), k[:, None].astype(np.int8), v[:, None].astype(np.int8),
                           ks[:, None], vs[:, None])
    assert np.abs(out[0].cpu().numpy() - exact).max() < 1e-4
    assert runtime.streams["target"] is not None
    with pytest.raises(CudaPagedAttentionError):
        submit_paged_attention(runtime, torch.zeros((1, 1, 4, D), device=device), synced.result, 0)
    with pytest.raises(CudaPagedAttentionError):
        submit_paged_attention(runtime, q, synced.result, 1)


def test_rejects_token_major_layout(device, runtime):
    """A pool stored token-major (offset stride != head_dim) is refused, not misread."""
    import torch

    from specdecode_b200.cuda_kv_cache import CudaPagedAttentionError, CudaPagedKVCacheView, submit_paged_attention

    keys = torch.zeros((2, 2, 1, 2, D), dtype=torch.int8, device=device)
    scales = torch.zeros((2, 2, 1, 2), dtype=torch.float32, device=device)
    view = CudaPagedKVCacheView(keys, keys.clone(), scales, scales.clone(),
                                torch.tensor([0], device=device), 2, 2)
    with pytest.raises(CudaPagedAttentionError):
        submit_paged_attention(runtime, torch.zeros((1, 2, 1, D), device=device), view, 0)


def _hf_cache(length, heads=2, batch=1, layers=2, dtype="bfloat16", device=None):
    import torch

    gen = torch.Generator().manual_seed(length * 13 + heads)
    return tuple(
        (torch.randn((batch, heads, length, D), generator=gen).to(getattr(torch, dtype)).to(device),
         torch.randn((batch, heads, length, D), generator=gen).to(getattr(torch, dtype)).to(device))
        for _ in range(layers))


def test_hf_mirror_lifecycle(device):
    import torch

    from specdecode_b200.hf_paged_cache import (HuggingFacePagedCacheConfig, HuggingFacePagedCacheError,
                                                HuggingFacePagedCacheMirror)

    model_config = SimpleNamespace(num_hidden_layers=2, num_key_value_heads=2, num_attention_heads=4,
                                   hidden_size=4 * D, max_position_embeddings=8)
    mirror = HuggingFacePagedCacheMirror.from_model_config(model_config, HuggingFacePagedCacheConfig(block_size=2),
                                                           device=device)
    c = mirror.cache.config
    assert (c.num_layers, c.num_heads, c.head_dim, c.block_size, c.num_blocks) == (2, 2, D, 2, 4)
    full = _hf_cache(4, device=device)
    first = tuple((k[:, :, :3], v[:, :, :3]) for k, v in full)
    assert mirror.synchronize(first) == 3
    assert mirror.synchronize(full) == 1
    assert mirror.token_count == 4 and mirror.block_table == (0, 1)
    # every mirrored value is the reference quantization of the model's bf16 value
    for layer in range(2):
        k = full[layer][0][0].float().cpu().numpy().transpose(1, 0, 2)  # [T, H, D]
        codes, scales, _ = quantize_rows(k.astype(np.float64))
        for t in range(4):
            token = mirror.cache.read_quantized_token("model", t)
            for h in range(2):
                assert list(token.keys[layer][h].values) == codes[t, h].tolist()
                assert token.keys[layer][h].scale == float(scales[t, h])
    # materialisation keeps the template's dtype/device and the narrowing rule
    legacy = mirror.materialize_legacy_cache(torch, template=full)
    assert legacy[0][0].shape == (1, 2, 4, D) and legacy[0][0].dtype == torch.bfloat16
    assert legacy[0][0].device == full[0][0].device
    k = full[1][1][0].float().cpu().numpy().transpose(1, 0, 2)
    codes, scales, _ = quantize_rows(k.astype(np.float64))
    expected = torch.from_numpy((codes * scales[..., None].astype(np.float64)).astype(np.float32))
    expected = expected.to(torch.bfloat16).permute(1, 0, 2).unsqueeze(0)
    assert torch.equal(legacy[1][1].cpu(), expected)
    as_list = mirror.materialize_like(torch, list(full))
    assert isinstance(as_list, list)
    assert mirror.truncate(1) == 3
    mirror.reset()
    assert mirror.token_count == 0 and mirror.stats.rollback_tokens == 3 and mirror.stats.resets == 1
    empty = mirror.materialize_legacy_cache(torch)
    assert empty[0][0].shape == (1, 2, 0, D)
    with pytest.raises(HuggingFacePagedCacheError):
        mirror.synchronize(_hf_cache(2, heads=1, device=device))
    with pytest.raises(HuggingFacePagedCacheError):
        mirror.synchronize(_hf_cache(2, batch=2, device=device))
    assert mirror.token_count == 0
    mirror.synchronize(_hf_cache(3, device=device))
    with pytest.raises(HuggingFacePagedCacheError):
        mirror.synchronize(_hf_cache(2, device=device))
    assert mirror.token_count == 3
