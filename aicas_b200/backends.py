"""Hugging Face attention-interface functions for Qwen3-VL.

Signatures, module attributes read, backend keys and the ``[B, S, H, D]`` output
layout follow triton_qwen3vl/backends.py:90-289 (paths relative to the
reference project).  What differs by design: there is no multi-backend
dispatch and no SDPA fallback.  Every call either runs the sm_100a kernels or
raises ``ValueError`` naming the unsupported input, so a model patched with this
backend never silently runs a different attention implementation.

Routing (the reference's gates, backends.py:207-247):
  * text, q_len == 1                   -> :func:`ops.gqa_decode_attention`
  * text, q_len == kv_len > 1, causal  -> :func:`ops.gqa_flash_attention`
  * vision with ``cu_seq_lens``        -> :func:`ops.varlen_flash_attention`
  * vision without ``cu_seq_lens``     -> the whole sequence as one packed segment

A padded text batch (HF's 2-D padding mask, which the ``flash_attention_2``
mask function hands to this backend) is turned into per-request key ranges
on the device: the reference routes every masked call to SDPA
(backends.py:249-260, 277-287); here the kernels take the ranges directly.
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


# the key ranges of the last padding mask seen, with the mask itself (held, so
# that its memory cannot be reused by another tensor while it is cached) and
# its version counter: Hugging Face hands the same mask tensor to every layer
# of a forward pass, so the ranges are derived (and checked) once per pass
_LAST_MASK: list = []


def padding_bounds(attention_mask: torch.Tensor, batch: int, kv_len: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-request key range ``[start, end)`` (int32 ``[B]`` each, on the mask's
    device) of a 2-D padding mask ``[B, kv_len]`` (nonzero = a real token).

    Each row must hold one contiguous run of real tokens (left, right or no
    padding); anything else raises ``ValueError``.  The check costs one host
    synchronisation per new mask, and is skipped while a CUDA graph is being
    captured.  A row with no real token gets ``start == end``."""
    if attention_mask.ndim != 2 or tuple(attention_mask.shape) != (batch, kv_len):
        raise ValueError(f"the text backend takes a 2-D padding mask [{batch}, {kv_len}] "
                         f"(got {tuple(attention_mask.shape)}); other masks are not supported")
    if _LAST_MASK and _LAST_MASK[0] is attention_mask and _LAST_MASK[1] == attention_mask._version:
        return _LAST_MASK[2], _LAST_MASK[3]
    real = attention_mask != 0
    count = real.sum(dim=1, dtype=torch.int32)
    idx = torch.arange(kv_len, device=real.device, dtype=torch.int32)
    start = torch.where(real, idx, kv_len).amin(dim=1).to(torch.int32)
    end = (torch.where(real, idx, -1).amax(dim=1) + 1).to(torch.int32)
    start = torch.minimum(start, end.clamp(min=0))
    end = torch.maximum(end, start)
    capturing = real.is_cuda and torch.cuda.is_current_stream_capturing()
    if not capturing and not bool(((end - start) == count).all()):
        raise ValueError("the text backend needs each padding-mask row to be one contiguous run of real tokens "
                         "(left or right padding)")
    _LAST_MASK[:] = [attention_mask, attention_mask._version, start, end]
    return start, end


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
    q_len, kv_len = query.shape[2], key.shape[2]
    starts = ends = None
    if attention_mask is not None:
        starts, ends = padding_bounds(attention_mask, query.shape[0], kv_len)
    if q_len == 1:
        kv_lens = kwargs.get("kv_lens")
        if ends is not None:
            if kv_lens is not None:
                raise ValueError("pass either a padding mask or kv_lens, not both")
            kv_lens = ends
        attn_output = ops.gqa_decode_attention(
            query,
            key,
            value,
            sm_scale=sm_scale,
            num_key_value_groups=num_key_value_groups,
            kv_lens=kv_lens,
            kv_starts=starts,
        )
        return attn_output.transpose(1, 2).contiguous(), None
    if q_len != kv_len:
        raise ValueError(f"text prefill needs q_len == kv_len (got {q_len} vs {kv_len})")
    # right padding needs no key mask: a real query row never reaches the
    # padding after it (causal); the padded rows' outputs are unused by HF
    attn_output = ops.gqa_flash_attention(
        query,
        key,
        value,
        causal=is_causal,
        sm_scale=sm_scale,
        num_key_value_groups=num_key_value_groups,
        kv_starts=starts,
    )
    return attn_output.transpose(1, 2).contiguous(), None
