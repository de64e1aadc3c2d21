"""The Hugging Face attention hook: a transformers Llama model whose attention
reads and writes the paged INT8 cache, against the same model with full
precision SDPA attention.

A random-init 2-layer Llama (4 query heads per KV head, head_dim 128) first
prefills a 37-token prompt through the hook (three causal windows of 16
queries), then verifies a 5-token window.  Two references run the whole
42-token sequence in one forward:

* full-precision SDPA.  The paged path quantizes every key / value to INT8,
  so its logits differ by the quantization error: the test bounds that
  difference relative to the logits' spread (0.25 of the standard deviation)
  and asserts that the greedy token agrees at 80 % of positions or more;
* SDPA over keys / values quantized and dequantized with the reference's rule
  (per (token, head) vector: scale = max|x| / 127, codes rounded half away
  from zero, in float64), attention in float32 — the same numbers the paged
  path stores, so only the kernel's arithmetic differs (then amplified by
  the model's bf16 layers; 0.04 of the logits' spread measured on B200):
  bounded at 0.06.
"""

from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


def _model(device):
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    config = LlamaConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=4,
                         num_key_value_heads=1, head_dim=128, vocab_size=1000, max_position_embeddings=256,
                         initializer_range=0.05)
    return LlamaForCausalLM(config).to(device=device, dtype=torch.bfloat16).eval()


def _qdq(x):
    """Quantize / dequantize per last-axis vector with the reference rule."""
    import torch

    d = x.double()
    m = d.abs().amax(dim=-1, keepdim=True)
    s = (m / 127.0).float().double()
    q = torch.where(s > 0, torch.sign(d) * torch.floor(d.abs() / torch.where(s > 0, s, 1.0) + 0.5), 0.0)
    return (q.clamp(-127, 127) * s).to(x.dtype)


def _qdq_sdpa(module, query, key, value, attention_mask, dropout=0.0, scaling=None, **kwargs):
    import torch.nn.functional as F

    from transformers.integrations.sdpa_attention import repeat_kv

    # float32 attention over the dequantized codes, as the kernel computes it
    k = repeat_kv(_qdq(key.float()), module.num_key_value_groups)
    v = repeat_kv(_qdq(value.float()), module.num_key_value_groups)
    out = F.scaled_dot_product_attention(query.float(), k, v, is_causal=True, scale=scaling)
    return out.to(query.dtype).transpose(1, 2).contiguous(), None


def test_paged_hook_matches_full_precision_attention(device):
    import torch

    from gpu_helpers import make_cache
    from specdecode_b200.hf_attention import PagedAttentionSession

    model = _model(device)
    B, prompt, window = 2, 37, 5
    ids = torch.randint(0, 1000, (B, prompt + window), generator=torch.Generator().manual_seed(3)).to(device)
    with torch.no_grad():
        model.set_attn_implementation("sdpa")
        want = model(ids, use_cache=False).logits[:, prompt:].float()
        from transformers import AttentionInterface
        from transformers.masking_utils import AttentionMaskInterface, sdpa_mask

        AttentionInterface.register("qdq_sdpa", _qdq_sdpa)
        AttentionMaskInterface.register("qdq_sdpa", sdpa_mask)
        model.set_attn_implementation("qdq_sdpa")
        want_q = model(ids, use_cache=False).logits[:, prompt:].float()

        cache = make_cache(device, 2, 1, 128, 16, 64)
        seqs = ["a", "b"]
        for s in seqs:
            cache.create_sequence(s)
        session = PagedAttentionSession(cache)
        model.set_attn_implementation(PagedAttentionSession.NAME)
        with session.step(seqs, prompt):
            pos = torch.arange(prompt, device=device).expand(B, prompt)
            model(ids[:, :prompt], position_ids=pos, use_cache=False)
        with session.step(seqs, window):
            pos = torch.arange(prompt, prompt + window, device=device).expand(B, window)
            got = model(ids[:, prompt:], position_ids=pos, use_cache=False).logits.float()
    assert [cache.sequence_length(s) for s in seqs] == [prompt + window] * B
    spread = float(want.std())
    err = float((got - want).abs().max())
    print("max |paged - sdpa| / logit std:", err / spread)
    assert err <= 0.25 * spread, (err, spread)
    agree = float((got.argmax(-1) == want.argmax(-1)).float().mean())
    assert agree >= 0.8, agree
    err_q = float((got - want_q).abs().max())
    print("max |paged - quantized sdpa| / logit std:", err_q / spread)
    assert err_q <= 0.06 * spread, (err_q, spread)
