"""The reference's own CPU runtime path for the decode step, restated with torch
CPU operators — TEST INFRASTRUCTURE / CPU BASELINE ONLY.

On CPU tensors the reference backend (triton_qwen3vl/backends.py:179-289 in the
reference project) always takes ``sdpa_fallback`` (fallback.py:23-64), which
calls Hugging Face's ``sdpa_attention_forward``, i.e.
``F.scaled_dot_product_attention(q, k, v, scale=s, enable_gqa=True)`` followed by
``transpose(1, 2).contiguous()``.  Before it, Qwen3VLTextAttention applies
``apply_rotary_pos_emb`` and appends to the cache (InplaceDecodeCacheLayer,
dujunbaoV1/evaluation_wrapper.py:84-100).  The reference has no length vector,
so a ragged batch runs request by request over each valid prefix.

``bench.py`` times this on the host cores as the CPU baseline ("port": the
reference is Python and cannot travel to the GPU box).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def apply_rotary_pos_emb(q, k, cos, sin):
    cos = cos.unsqueeze(1)
    sin = sin.unsqueeze(1)
    return q * cos + rotate_half(q) * sin, k * cos + rotate_half(k) * sin


def decode_layer(q, k_new, v_new, cos, sin, k_cache, v_cache, positions, scale: float) -> torch.Tensor:
    """One text-attention layer of a decode step for a ragged batch; returns
    [B, 1, Hq, D] (the backend's output layout) and updates the caches in place."""
    q_rot, k_rot = apply_rotary_pos_emb(q, k_new, cos, sin)
    outs = []
    for b, p in enumerate(positions.tolist()):
        k_cache[b, :, p] = k_rot[b, :, 0]
        v_cache[b, :, p] = v_new[b, :, 0]
        n = p + 1
        o = F.scaled_dot_product_attention(q_rot[b : b + 1], k_cache[b : b + 1, :, :n], v_cache[b : b + 1, :, :n],
                                           scale=scale, enable_gqa=True)
        outs.append(o.transpose(1, 2).contiguous())
    return torch.cat(outs, 0)


def decode_long(q, k, v, scale: float) -> torch.Tensor:
    """Config 5 on the CPU: one SDPA call over the whole cache."""
    return F.scaled_dot_product_attention(q, k, v, scale=scale, enable_gqa=True).transpose(1, 2).contiguous()
