"""The vision attention's RoPE in one kernel (aicas_vision_rope) against Hugging
Face's apply_rotary_pos_emb_vision and the CPU restatement: bit-identical, for
q/k taken as strided views of the packed qkv projection; and the fused vision
attention forward against Hugging Face's forward on the same backend."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from aicas_b200 import ops
from oracle import rope as orope

pytestmark = pytest.mark.gpu


def _inputs(T, H, D, dtype, device, seed):
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn(T, 3, H, D, generator=g).to(dtype).to(device)
    freqs = torch.randn(T, D // 2, generator=g) * 4
    emb = torch.cat((freqs, freqs), dim=-1).to(device)
    return qkv, emb.cos(), emb.sin()


@pytest.mark.parametrize("T,H,D", [(1, 16, 64), (37, 16, 64), (4099, 16, 64), (300, 8, 128), (64, 2, 16)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_bit_exact_against_hf(cuda_device, native_lib, T, H, D, dtype):
    from transformers.models.qwen3_vl.modeling_qwen3_vl import apply_rotary_pos_emb_vision

    qkv, cos, sin = _inputs(T, H, D, dtype, cuda_device, seed=T + D)
    q, k = qkv[:, 0], qkv[:, 1]  # strided views, as the vision attention splits them
    hq, hk = apply_rotary_pos_emb_vision(q, k, cos, sin)
    oq, ok = ops.vision_rope(q, k, cos, sin)
    assert oq.is_contiguous() and ok.shape == (T, H, D)
    assert torch.equal(oq, hq) and torch.equal(ok, hk)
    name = "bf16" if dtype == torch.bfloat16 else "fp16"
    ref = orope.apply_rope_vision(q.float().cpu().numpy(), cos.cpu().numpy(), sin.cpu().numpy(), name)
    assert np.array_equal(oq.float().cpu().numpy(), ref)


def test_empty_and_rejected(cuda_device, native_lib):
    qkv, cos, sin = _inputs(0, 4, 64, torch.bfloat16, cuda_device, seed=1)
    oq, ok = ops.vision_rope(qkv[:, 0], qkv[:, 1], cos, sin)
    assert oq.shape == (0, 4, 64)
    qkv, cos, sin = _inputs(8, 4, 40, torch.bfloat16, cuda_device, seed=1)
    with pytest.raises(ValueError, match="multiple of 16"):
        ops.vision_rope(qkv[:, 0], qkv[:, 1], cos, sin)
    qkv, cos, sin = _inputs(8, 4, 64, torch.bfloat16, cuda_device, seed=1)
    with pytest.raises(ValueError, match="floating-point"):
        ops.vision_rope(qkv[:, 0], qkv[:, 1], cos[:, :32], sin)
    # 16-bit cos/sin (a bf16 model's rotary buffer): upcast as HF does
    from transformers.models.qwen3_vl.modeling_qwen3_vl import apply_rotary_pos_emb_vision

    cb, sb = cos.to(torch.bfloat16), sin.to(torch.bfloat16)
    hq, hk = apply_rotary_pos_emb_vision(qkv[:, 0], qkv[:, 1], cb, sb)
    oq, ok = ops.vision_rope(qkv[:, 0], qkv[:, 1], cb, sb)
    assert torch.equal(oq, hq) and torch.equal(ok, hk)


def test_fused_vision_attention_forward_matches_hf(cuda_device, native_lib):
    """One Qwen3-VL vision attention module on this backend: the fused forward
    (QKV split + RoPE in one kernel) gives the same bits as Hugging Face's."""
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLVisionConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLVisionAttention

    from aicas_b200 import VISION_BACKEND_KEY, install_qwen3vl_triton_attention  # noqa: F401  (registers the key)
    from aicas_b200.vision import fused_vision_attention_forward

    install_qwen3vl_triton_attention(torch.nn.Module())
    cfg = Qwen3VLVisionConfig(hidden_size=256, num_heads=4, intermediate_size=512, depth=1)
    cfg._attn_implementation = VISION_BACKEND_KEY
    torch.manual_seed(0)
    attn = Qwen3VLVisionAttention(cfg).to(torch.bfloat16).to(cuda_device).eval()
    lens = [64, 100, 36]
    T = sum(lens)
    cu = torch.tensor([0, 64, 164, 200], dtype=torch.int32, device=cuda_device)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(T, 256, generator=g).to(torch.bfloat16).to(cuda_device)
    freqs = torch.randn(T, 32, generator=g) * 4
    emb = torch.cat((freqs, freqs), dim=-1).to(cuda_device)
    pe = (emb.cos(), emb.sin())
    with torch.no_grad():
        ref = attn(x, cu_seqlens=cu, position_embeddings=pe)
        out = fused_vision_attention_forward(attn, x, cu_seqlens=cu, position_embeddings=pe)
    assert torch.equal(out, ref)
