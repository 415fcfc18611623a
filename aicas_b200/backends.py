"""Hugging Face attention-interface functions for Qwen3-VL.

Signatures, module attributes read, backend keys and the ``[B, S, H, D]`` output
layout follow triton_qwen3vl/backends.py:90-289 (paths relative to the
reference project).  What differs by design: there is no multi-backend
dispatch and no SDPA fallback.  Every call either runs the sm_100a kernels or
raises ``ValueError`` naming the unsupported input, so a model patched with this
backend never silently runs a different attention implementation.

Routing (the reference's gates, backends.py:207-247):
  * text, q_len == 1, no mask          -> :func:`ops.gqa_decode_attention`
  * text, q_len == kv_len > 1, causal  -> :func:`ops.gqa_flash_attention`
  * vision with ``cu_seq_lens``        -> :func:`ops.varlen_flash_attention`
  * vision without ``cu_seq_lens``     -> the whole sequence as one packed segment
"""
from __future__ import annotations

import torch

from . import ops

# Both keys must contain "flash": HF passes cu_seqlens to the vision attention
# only for flash-style implementations (transformers utils/generic.py:283).
TEXT_BACKEND_KEY = "qwen3vl_triton_flash_text"
VISION_BACKEND_KEY = "qwen3vl_triton_flash_vision"


def _resolve_is_causal(module: torch.nn.Module, is_causal: bool | None) -> bool:
    if is_causal is not None:
        return bool(is_causal)
    return bool(getattr(module, "is_causal", True))


def _resolve_scale(module: torch.nn.Module, scaling: float | None) -> float:
    if scaling is not None:
        return float(scaling)
    return float(getattr(module, "scaling"))


def _reject_common(dropout: float, kwargs: dict) -> None:
    if kwargs.get("output_attentions", False):
        raise ValueError("the aicas_b200 attention backend does not return attention weights (output_attentions)")
    if dropout != 0.0:
        raise ValueError("the aicas_b200 attention backend is inference-only (dropout must be 0)")


def vision_triton_attention(
    module: torch.nn.Module,
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    attention_mask: torch.Tensor | None = None,
    dropout: float = 0.0,
    scaling: float | None = None,
    cu_seq_lens_q: torch.Tensor | None = None,
    cu_seq_lens_k: torch.Tensor | None = None,
    max_length_q: int | torch.Tensor | None = None,
    max_length_k: int | torch.Tensor | None = None,
    is_causal: bool | None = None,
    **kwargs,
) -> tuple[torch.Tensor, None]:
    """Vision-tower attention (reference: backends.py:90-176): non-causal,
    packed by ``cu_seq_lens``; returns ``([1, T, H, D] contiguous, None)``."""
    del attention_mask
    _reject_common(dropout, kwargs)
    if _resolve_is_causal(module, is_causal):
        raise ValueError("vision attention must be non-causal")
    sm_scale = _resolve_scale(module, scaling)
    if cu_seq_lens_q is None or cu_seq_lens_k is None:
        total = query.shape[2]
        cu = torch.tensor([0, total], dtype=torch.int32, device=query.device)
        cu_seq_lens_q = cu if cu_seq_lens_q is None else cu_seq_lens_q
        cu_seq_lens_k = cu if cu_seq_lens_k is None else cu_seq_lens_k
    metadata_cache = getattr(module, "_qwen3vl_vision_varlen_metadata_cache", None)
    if metadata_cache is None:
        metadata_cache = {}
        setattr(module, "_qwen3vl_vision_varlen_metadata_cache", metadata_cache)
    attn_output = ops.varlen_flash_attention(
        query,
        key,
        value,
        cu_seq_lens_q=cu_seq_lens_q,
        cu_seq_lens_k=cu_seq_lens_k,
        sm_scale=sm_scale,
        max_length_q=max_length_q,
        max_length_k=max_length_k,
        metadata_cache=metadata_cache,
    )
    return attn_output.transpose(1, 2).contiguous(), None


def text_triton_attention(
    module: torch.nn.Module,
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    attention_mask: torch.Tensor | None,
    dropout: float = 0.0,
    scaling: float | None = None,
    is_causal: bool | None = None,
    **kwargs,
) -> tuple[torch.Tensor, None]:
    """Text-decoder attention (reference: backends.py:179-289): GQA decode for
    q_len == 1, causal GQA prefill for q_len == kv_len; returns
    ``([B, S, Hq, D] contiguous, None)``."""
    _reject_common(dropout, kwargs)
    is_causal = _resolve_is_causal(module, is_causal)
    sm_scale = _resolve_scale(module, scaling)
    num_key_value_groups = int(getattr(module, "num_key_value_groups", 1))
    if attention_mask is not None:
        raise ValueError(
            "the aicas_b200 text backend takes no explicit attention mask (padded batches are not supported); "
            "lengths of a preallocated cache are passed as kv_lens instead"
        )
    q_len, kv_len = query.shape[2], key.shape[2]
    if q_len == 1:
        kv_lens = kwargs.get("kv_lens")
        attn_output = ops.gqa_decode_attention(
            query,
            key,
            value,
            sm_scale=sm_scale,
            num_key_value_groups=num_key_value_groups,
            kv_lens=kv_lens,
        )
        return attn_output.transpose(1, 2).contiguous(), None
    if q_len != kv_len:
        raise ValueError(f"text prefill needs q_len == kv_len (got {q_len} vs {kv_len})")
    attn_output = ops.gqa_flash_attention(
        query,
        key,
        value,
        causal=is_causal,
        sm_scale=sm_scale,
        num_key_value_groups=num_key_value_groups,
    )
    return attn_output.transpose(1, 2).contiguous(), None
