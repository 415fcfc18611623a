"""The vision attention's QKV split and RoPE fused ahead of the varlen kernel.

``Qwen3VLVisionAttention.forward`` (transformers
models/qwen3_vl/modeling_qwen3_vl.py:196-262) projects the patches with one
packed linear, splits q/k/v, rotates q and k with
``apply_rotary_pos_emb_vision`` -- fp32 copies and about eight elementwise
kernels per tensor -- and hands the three to the attention interface.
:func:`fused_vision_attention_forward` is the same computation with the
projection, its bias, the split and the rotation in one tensor-core kernel
(:func:`aicas_b200.ops.vision_qkv_rope`); projections that kernel does not
take (other head sizes) keep the library GEMM followed by the one-kernel
rotation (:func:`aicas_b200.ops.vision_rope`, bit-identical to HF).
:func:`install_vision_rope_fusion` puts it on every vision attention module of
a model.
"""
from __future__ import annotations

import types

import torch

from . import ops


def fused_vision_attention_forward(self, hidden_states: torch.Tensor, cu_seqlens: torch.Tensor,
                                   rotary_pos_emb: torch.Tensor | None = None,
                                   position_embeddings: tuple[torch.Tensor, torch.Tensor] | None = None,
                                   **kwargs) -> torch.Tensor:
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    from transformers.models.qwen3_vl.modeling_qwen3_vl import eager_attention_forward

    seq_length = hidden_states.shape[0]
    cos, sin = position_embeddings
    if _projection_fusable(self, hidden_states):
        # projection, bias, split and RoPE in one tensor-core kernel
        qkv = ops.vision_qkv_rope(hidden_states, self.qkv.weight, self.qkv.bias, cos, sin, self.num_heads)
        query_states, key_states = qkv[:, 0], qkv[:, 1]
    else:
        qkv = self.qkv(hidden_states).view(seq_length, 3, self.num_heads, -1)
        query_states, key_states = ops.vision_rope(qkv[:, 0], qkv[:, 1], cos, sin)
    query_states = query_states.transpose(0, 1).unsqueeze(0)
    key_states = key_states.transpose(0, 1).unsqueeze(0)
    value_states = qkv[:, 2].transpose(0, 1).unsqueeze(0)
    attention_interface = ALL_ATTENTION_FUNCTIONS.get_interface(self.config._attn_implementation,
                                                                eager_attention_forward)
    max_seqlen = (cu_seqlens[1:] - cu_seqlens[:-1]).max()
    attn_output, _ = attention_interface(self, query_states, key_states, value_states, attention_mask=None,
                                         scaling=self.scaling, dropout=0.0, cu_seq_lens_q=cu_seqlens,
                                         cu_seq_lens_k=cu_seqlens, max_length_q=max_seqlen,
                                         max_length_k=max_seqlen, is_causal=False, **kwargs)
    attn_output = attn_output.reshape(seq_length, -1).contiguous()
    return self.proj(attn_output)


def _projection_fusable(module, hidden_states: torch.Tensor) -> bool:
    """Whether ``aicas_vision_qkv_rope`` takes this module's projection: a plain
    ``nn.Linear`` of the hidden states' 16-bit dtype, head_dim 64, a multiple
    of 4 heads and of 64 input features (Qwen3-VL-2B's vision tower: 16 heads
    of 64 over 1024 features)."""
    lin = module.qkv
    if type(lin) is not torch.nn.Linear or hidden_states.ndim != 2:
        return False
    heads, (n, k) = module.num_heads, lin.weight.shape
    return (hidden_states.dtype in (torch.float16, torch.bfloat16) and lin.weight.dtype == hidden_states.dtype
            and n == 3 * heads * 64 and heads % 4 == 0 and k % 64 == 0)


def install_vision_rope_fusion(model) -> int:
    """Replaces ``forward`` of every ``Qwen3VLVisionAttention`` in ``model``;
    returns how many modules were switched.  Needs an attention implementation
    that takes ``cu_seqlens`` (this backend's vision key, or any flash one)."""
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLVisionAttention

    n = 0
    for module in model.modules():
        if isinstance(module, Qwen3VLVisionAttention):
            module.forward = types.MethodType(fused_vision_attention_forward, module)
            n += 1
    return n


def remove_vision_rope_fusion(model) -> int:
    """Puts the Hugging Face ``forward`` back on every vision attention module."""
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLVisionAttention

    n = 0
    for module in model.modules():
        if isinstance(module, Qwen3VLVisionAttention) and "forward" in module.__dict__:
            del module.forward
            n += 1
    return n
