"""The vision attention's packed QKV projection with the RoPE in its epilogue
(aicas_vision_qkv_rope) against Hugging Face's own path on the GPU (nn.Linear
through cuBLAS, then apply_rotary_pos_emb_vision) and against an fp64
reference of the same arithmetic.  Tolerance: the projection's output y is
rounded to the dtype (as nn.Linear's is) and the rotation's result again
(y_d cos - y_p sin, with p the partner column of rotate_half), so against the
unrounded fp64 reference each element is within half an ulp of each of
y_d, y_p and the result: |err| <= 2^-8 (|y_d| + |y_p| + |ref|) + 1e-3
elementwise (twice that sum of half-ulps of bf16), and mean-abs <= 2e-3.
HF's own path rounds at the same two places, so against it the same bound
holds (only the accumulation order differs)."""
from __future__ import annotations

import pytest
import torch

import aicas_b200 as ab
from aicas_b200 import _native as nat
from aicas_b200 import ops
from tests.conftest import bf16_tolerance_check

pytestmark = pytest.mark.gpu


def close(out: torch.Tensor, ref: torch.Tensor, pre: torch.Tensor) -> None:
    """out/ref [T, 3, H, D]; pre: the unrotated projection [T, 3, H, D]."""
    out, ref, pre = out.double().cpu(), ref.double().cpu(), pre.double().cpu()
    assert out.shape == ref.shape and torch.isfinite(out).all()
    partner = torch.cat([pre[..., 32:], pre[..., :32]], dim=-1)
    partner[:, 2] = 0.0  # v is not rotated
    err = (out - ref).abs()
    bound = (pre.abs() + partner.abs() + ref.abs()) * 2.0 ** -8 + 1e-3
    worst = float((err - bound).max())
    assert worst <= 0, f"max-abs {float(err.max()):.3e}, {int((err > bound).sum())} elements past the bound"
    assert float(err.mean()) <= 2e-3, f"mean-abs {float(err.mean()):.3e} > 2e-3"


def _inputs(T, K, H, dtype, device, seed, bias=True):
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(T, K, device=device, generator=g).to(dtype)
    w = (torch.randn(3 * H * 64, K, device=device, generator=g) / K ** 0.5).to(dtype)
    b = (0.1 * torch.randn(3 * H * 64, device=device, generator=g)).to(dtype) if bias else None
    emb = torch.randn(T, 32, device=device, generator=g).repeat(1, 2)
    return x, w, b, emb.cos(), emb.sin()


def _reference(x, w, b, cos, sin, H):
    """fp64: x W^T + b, split, rotate_half RoPE (HF's formula); returns
    (rotated [T, 3, H, D], unrotated [T, 3, H, D])."""
    y = x.double() @ w.double().T + (b.double() if b is not None else 0.0)
    qkv = y.view(x.shape[0], 3, H, 64)
    c, s = cos.double()[:, None], sin.double()[:, None]

    def rot(t):
        return t * c + torch.cat([-t[..., 32:], t[..., :32]], dim=-1) * s

    return torch.stack([rot(qkv[:, 0]), rot(qkv[:, 1]), qkv[:, 2]], dim=1), qkv


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T", [1, 127, 128, 300, 1000])
def test_against_fp64_reference(cuda_device, dtype, T):
    x, w, b, cos, sin = _inputs(T, 1024, 16, dtype, cuda_device, seed=T)
    out = ops.vision_qkv_rope(x, w, b, cos, sin, 16)
    assert out.shape == (T, 3, 16, 64) and out.dtype == dtype
    close(out, *_reference(x, w, b, cos, sin, 16))


def test_other_sizes_and_no_bias(cuda_device):
    for T, K, H, bias in ((77, 128, 4, False), (513, 64, 8, True), (256, 1280, 12, True)):
        x, w, b, cos, sin = _inputs(T, K, H, torch.bfloat16, cuda_device, seed=K + H, bias=bias)
        out = ops.vision_qkv_rope(x, w, b, cos, sin, H)
        close(out, *_reference(x, w, b, cos, sin, H))


def test_matches_the_hf_path_at_config_3_size(cuda_device):
    """T = 48478 patches (config 3), hidden 1024, 16 heads of 64: HF's
    nn.Linear + apply_rotary_pos_emb_vision against this kernel."""
    from transformers.models.qwen3_vl.modeling_qwen3_vl import apply_rotary_pos_emb_vision

    from aicas_b200 import workloads as wl

    _, _, _, cu, _ = wl.cfg3_varlen(seed=0, device=cuda_device)
    T = int(cu[-1])
    x, w, b, cos, sin = _inputs(T, 1024, 16, torch.bfloat16, cuda_device, seed=3)
    qkv = torch.nn.functional.linear(x, w, b).view(T, 3, 16, 64)
    q_hf, k_hf = apply_rotary_pos_emb_vision(qkv[:, 0], qkv[:, 1], cos, sin)
    out = ops.vision_qkv_rope(x, w, b, cos, sin, 16)
    close(out, torch.stack([q_hf, k_hf, qkv[:, 2]], dim=1), qkv)
    torch.cuda.synchronize(cuda_device)
    assert nat.device_error_flags() == 0


def test_fused_vision_attention_forward_uses_it(cuda_device):
    """The patched vision attention module (fuse_vision_rope) runs the fused
    projection and gives HF's result within the bar."""
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLVisionAttention

    from aicas_b200 import integration as it
    from aicas_b200.vision import fused_vision_attention_forward

    cfg = it.qwen3vl_config().vision_config
    cfg._attn_implementation = ab.VISION_BACKEND_KEY
    ab.install_qwen3vl_triton_attention(torch.nn.Module())  # registers the backend keys
    torch.manual_seed(0)
    mod = Qwen3VLVisionAttention(cfg).to(cuda_device).to(torch.bfloat16).eval()
    T = 700
    h = torch.randn(T, 1024, device=cuda_device).to(torch.bfloat16)
    emb = torch.randn(T, 32, device=cuda_device).repeat(1, 2)
    cu = torch.tensor([0, 300, 700], dtype=torch.int32, device=cuda_device)
    with torch.no_grad():
        ref = mod(h, cu, position_embeddings=(emb.cos(), emb.sin()))
        calls = {"n": 0}
        orig = ops.vision_qkv_rope

        def counted(*a, **k):
            calls["n"] += 1
            return orig(*a, **k)

        ops.vision_qkv_rope = counted
        try:
            got = fused_vision_attention_forward(mod, h, cu, position_embeddings=(emb.cos(), emb.sin()))
        finally:
            ops.vision_qkv_rope = orig
    assert calls["n"] == 1
    # the attention output (magnitude <= ~1) of the two paths
    bf16_tolerance_check(got.float().cpu().numpy(), ref.float().cpu().numpy())
