"""ORACLE — paged verify/decode attention restated on the CPU.

Test infrastructure only.  Two restatements of the reference's unfused paged
attention, src/specdecode/cuda_kv_cache.py:452-497:

* ``attention_fp64`` — exact-arithmetic restatement in float64 numpy:
  codes x float32 scale (exact in double), query head ``h`` reads KV head
  ``h // (Hq / Hkv)`` (repeat_interleave, :479-482), boolean causal mask
  ``q_pos >= k_pos`` with the query at the last ``k`` cached positions
  (:484-490), softmax scale ``1/sqrt(D)`` (SDPA's default, :491-497).
* ``attention_reference_torch`` — the reference's own dtype behaviour on CPU
  torch: gather pages through the block table, dequantize *in the query dtype*
  (``int8.to(q.dtype) * scale.to(q.dtype)``, :475-476), expand GQA heads,
  build the boolean mask and call ``F.scaled_dot_product_attention``.  This is
  "the reference's dequantize-then-SDPA computation" that the attention
  tolerance (max-abs 2e-2, mean-abs 2e-3 in bf16) is stated against.

The SDPA arithmetic itself lives in PyTorch (a dependency the reference pins
only as ``torch>=2.3``, pyproject.toml:17); the fp64 form restates its
published definition, softmax(q k^T * scale + mask) v.
"""

from __future__ import annotations

import math

import numpy as np


def attention_fp64(q, k_codes, v_codes, k_scales, v_scales) -> np.ndarray:
    """One sequence.

    q: ``[Hq, kw, D]`` (any real dtype); k_codes/v_codes: ``[T, Hkv, D]`` int8;
    k_scales/v_scales: ``[T, Hkv]`` float32.  Returns ``[Hq, kw, D]`` float64.
    """
    q = np.asarray(q, dtype=np.float64)
    Hq, kw, D = q.shape
    T, Hkv, _ = k_codes.shape
    if kw > T or Hq % Hkv:
        raise ValueError("query window longer than the cache, or incompatible heads")
    group = Hq // Hkv
    keys = k_codes.astype(np.float64) * k_scales.astype(np.float64)[..., None]
    values = v_codes.astype(np.float64) * v_scales.astype(np.float64)[..., None]
    out = np.empty((Hq, kw, D), dtype=np.float64)
    k_pos = np.arange(T)
    q_pos = np.arange(T - kw, T)
    mask = q_pos[:, None] >= k_pos[None, :]
    scale = 1.0 / math.sqrt(D)
    for h in range(Hq):
        kv = h // group
        scores = (q[h] @ keys[:, kv, :].T) * scale
        scores = np.where(mask, scores, -np.inf)
        scores -= scores.max(axis=1, keepdims=True)
        weights = np.exp(scores)
        weights /= weights.sum(axis=1, keepdims=True)
        out[h] = weights @ values[:, kv, :]
    return out


def attention_fp64_batch(q, gathered) -> list[np.ndarray]:
    """q: ``[B, Hq, kw, D]``; gathered: per-sequence (k, v, ks, vs) tuples."""
    return [attention_fp64(q[b], *gathered[b]) for b in range(len(gathered))]


def attention_reference_torch(query, keys, values, key_scales, value_scales,
                              block_table, token_count: int, layer: int):
    """The reference's unfused op (cuda_kv_cache.py:452-497) on CPU torch.

    query ``[1, Hq, kw, D]`` (bf16 or fp32); keys/values ``[nb, bs, L, H, D]``
    int8; scales ``[nb, bs, L, H]`` float32; block_table int64 ``[nblk]``.
    """
    import torch
    import torch.nn.functional as F

    def pages(tensor):
        return tensor.index_select(0, block_table).flatten(0, 1)[:token_count].select(1, layer)

    k = pages(keys)
    v = pages(values)
    ks = pages(key_scales).unsqueeze(-1)
    vs = pages(value_scales).unsqueeze(-1)
    k = k.to(dtype=query.dtype) * ks.to(dtype=query.dtype)
    v = v.to(dtype=query.dtype) * vs.to(dtype=query.dtype)
    k = k.transpose(0, 1).unsqueeze(0)
    v = v.transpose(0, 1).unsqueeze(0)
    group = query.shape[1] // k.shape[1]
    if group > 1:
        k = k.repeat_interleave(group, dim=1)
        v = v.repeat_interleave(group, dim=1)
    k_pos = torch.arange(token_count, device=query.device)
    q_pos = torch.arange(token_count - query.shape[2], token_count, device=query.device)
    mask = q_pos.unsqueeze(1) >= k_pos.unsqueeze(0)
    return F.scaled_dot_product_attention(query, k, v, attn_mask=mask, dropout_p=0.0)


def attention_reference_torch_flat(q_seq, k_codes, v_codes, k_scales, v_scales):
    """Same dtype behaviour as ``attention_reference_torch`` but on already
    gathered per-sequence tensors (torch): q ``[Hq, kw, D]``, codes
    ``[T, Hkv, D]`` int8, scales ``[T, Hkv]`` float32.  Returns ``[Hq, kw, D]``."""
    import torch
    import torch.nn.functional as F

    dtype = q_seq.dtype
    T = k_codes.shape[0]
    kw = q_seq.shape[1]
    k = k_codes.to(dtype) * k_scales.unsqueeze(-1).to(dtype)
    v = v_codes.to(dtype) * v_scales.unsqueeze(-1).to(dtype)
    k = k.transpose(0, 1).unsqueeze(0)
    v = v.transpose(0, 1).unsqueeze(0)
    group = q_seq.shape[0] // k.shape[1]
    if group > 1:
        k = k.repeat_interleave(group, dim=1)
        v = v.repeat_interleave(group, dim=1)
    device = q_seq.device
    mask = torch.arange(T - kw, T, device=device).unsqueeze(1) >= torch.arange(T, device=device).unsqueeze(0)
    return F.scaled_dot_product_attention(q_seq.unsqueeze(0), k, v, attn_mask=mask)[0]


def dequantize_like_torch(codes: np.ndarray, scales: np.ndarray, dtype: str) -> np.ndarray:
    """Materialisation rule of src/specdecode/hf_paged_cache.py:274-305:
    ``code * scale`` in double (kv_cache.py:151, exact), then
    ``torch.tensor(..., dtype)``, which narrows double -> float32 -> dtype.
    Returns float32 values of the narrowed result (bf16/fp16 widened back)."""
    import torch

    product = codes.astype(np.float64) * scales.astype(np.float64)[..., None]
    narrowed = torch.from_numpy(product.astype(np.float32))
    target = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}[dtype]
    return narrowed.to(target).to(torch.float32).numpy()
