"""Seeded synthetic inputs for the five benchmark configurations.

No dataset drives this path (the reference's VQA set is not available, and
synthetic inputs stand in for it); every tensor is ~N(0, 1) from a
``torch.Generator`` seeded per config, in the shapes of the Qwen3-VL-2B hot path:

1. GQA decode, B=1, Hq=16, Hkv=8, D=128, L=1024, fp32.
2. Batched GQA decode, B=64, 28 layers, per-request lengths ~ U[256, 4096]
   in caches padded to 4096, bf16; each step rotates and appends the new token.
3. ViT varlen attention, 32 images with patch grids h, w ~ U[16, 64], H=16, D=64, bf16.
4. Causal GQA prefill, B=8, S=2048, Hq=16, Hkv=8, D=128, bf16, q/k rotated with
   multimodal RoPE from 3-axis position ids (text, an image span, text).
5. Long-context decode, B=4, L=131072, Hq=16, Hkv=8, D=128, bf16.

Text RoPE constants are those of the Qwen3-VL text config as assumed here:
rope_theta 5e6 and mrope_section [24, 20, 20] (head_dim 128); they are
assumptions, the checkpoint is not available.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

HQ, HKV, HEAD_DIM = 16, 8, 128
VIT_HEADS, VIT_HEAD_DIM = 16, 64
NUM_LAYERS = 28
ROPE_THETA = 5_000_000.0
MROPE_SECTION = (24, 20, 20)
SCALE_TEXT = 1.0 / math.sqrt(HEAD_DIM)
SCALE_VIT = 1.0 / math.sqrt(VIT_HEAD_DIM)


def generator(seed: int, device: str | torch.device = "cpu") -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def randn(shape, g: torch.Generator, dtype=torch.float32, device="cpu") -> torch.Tensor:
    return torch.randn(shape, generator=g, dtype=torch.float32, device=device).to(dtype)


# ---------------------------------------------------------------- text RoPE tables


def mrope_cos_sin(position_ids: torch.Tensor, dtype: torch.dtype, head_dim: int = HEAD_DIM,
                  theta: float = ROPE_THETA, section=MROPE_SECTION):
    """cos/sin [B, S, D] of Qwen3-VL's interleaved multimodal RoPE for
    position_ids [3, B, S] (computed in fp32, then cast to ``dtype``)."""
    dev = position_ids.device
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64, device=dev).float() / head_dim))
    freqs = position_ids.float()[..., None] * inv  # [3, B, S, D/2]
    ft = freqs[0].clone()
    for axis, offset in ((1, 1), (2, 2)):
        length = section[axis] * 3
        ft[..., offset:length:3] = freqs[axis][..., offset:length:3]
    emb = torch.cat([ft, ft], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def text_position_ids(positions: torch.Tensor) -> torch.Tensor:
    """Pure-text tokens carry the same id on all three axes: [B, S] -> [3, B, S]."""
    return positions[None].expand(3, *positions.shape)


def mixed_prompt_position_ids(batch: int, seq: int, text_before: int = 100, grid=(32, 50)) -> torch.Tensor:
    """[3, B, S] ids of a prompt = text, one image of grid (h, w) merged patches,
    text: text ids are (i, i, i); image token (r, c) is (t0, t0 + r, t0 + c);
    the trailing text continues after the largest id used."""
    gh, gw = grid
    n_img = gh * gw
    assert text_before + n_img <= seq
    ids = torch.empty(3, seq, dtype=torch.int64)
    t = torch.arange(text_before)
    ids[:, :text_before] = t
    r = torch.arange(gh).repeat_interleave(gw)
    c = torch.arange(gw).repeat(gh)
    ids[0, text_before : text_before + n_img] = text_before
    ids[1, text_before : text_before + n_img] = text_before + r
    ids[2, text_before : text_before + n_img] = text_before + c
    start = text_before + max(gh, gw)
    n_after = seq - text_before - n_img
    ids[:, text_before + n_img :] = start + torch.arange(n_after)
    return ids[:, None, :].expand(3, batch, seq).contiguous()


def rope_reference_torch(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x*cos + rotate_half(x)*sin with torch's dtype arithmetic (x [B,H,S,D], cos [B,S,D])."""
    c, s = cos[:, None], sin[:, None]
    h = x.shape[-1] // 2
    rot = torch.cat([-x[..., h:], x[..., :h]], dim=-1)
    return x * c + rot * s


# ---------------------------------------------------------------- configs


def cfg1_decode(seed: int = 0):
    """Config 1: q [1,16,1,128], k/v [1,8,1024,128] fp32 on CPU, scale 1/sqrt(128)."""
    g = generator(seed)
    q = randn((1, HQ, 1, HEAD_DIM), g)
    k = randn((1, HKV, 1024, HEAD_DIM), g)
    v = randn((1, HKV, 1024, HEAD_DIM), g)
    return q, k, v


def cfg2_lengths(seed: int = 0, batch: int = 64, lo: int = 256, hi: int = 4096) -> torch.Tensor:
    g = generator(seed)
    return torch.randint(lo, hi + 1, (batch,), generator=g, dtype=torch.int64).to(torch.int32)


@dataclass
class DecodeStepInputs:
    q: torch.Tensor         # [B, Hq, 1, D] new query (before RoPE)
    k: torch.Tensor         # [B, Hkv, 1, D] new key (before RoPE)
    v: torch.Tensor         # [B, Hkv, 1, D]
    cos: torch.Tensor       # [B, 1, D]
    sin: torch.Tensor       # [B, 1, D]
    positions: torch.Tensor  # [B] int32 slot of the new token (= current length)


def cfg2_step_inputs(lengths: torch.Tensor, layer: int, seed: int = 0, dtype=torch.bfloat16,
                     device="cpu") -> DecodeStepInputs:
    """Per-layer inputs of one decode step of config 2 (new token at slot lengths[b])."""
    B = lengths.shape[0]
    g = generator(seed * 1000 + 17 + layer, device)
    q = randn((B, HQ, 1, HEAD_DIM), g, dtype, device)
    k = randn((B, HKV, 1, HEAD_DIM), g, dtype, device)
    v = randn((B, HKV, 1, HEAD_DIM), g, dtype, device)
    pos = lengths.to(device=device, dtype=torch.int64)
    cos, sin = mrope_cos_sin(text_position_ids(pos[:, None]), dtype)
    return DecodeStepInputs(q, k, v, cos, sin, lengths.to(device=device, dtype=torch.int32))


def cfg2_cache(batch: int, capacity: int, layer: int, seed: int = 0, dtype=torch.bfloat16, device="cpu"):
    """One layer's padded caches [B, Hkv, capacity, D] (the whole capacity is
    filled with N(0,1); only the first lengths[b] slots are attended)."""
    g = generator(seed * 1000 + 500 + layer, device)
    k = randn((batch, HKV, capacity, HEAD_DIM), g, dtype, device)
    v = randn((batch, HKV, capacity, HEAD_DIM), g, dtype, device)
    return k, v


def cfg3_grids(seed: int = 0, images: int = 32, lo: int = 16, hi: int = 64) -> list[tuple[int, int]]:
    """Patch grids (h, w) ~ U[lo, hi] per side.  Attention does not need the even
    sides the 2x2 merger wants, so any integer side is drawn."""
    g = generator(seed)
    hw = torch.randint(lo, hi + 1, (images, 2), generator=g)
    return [(int(a), int(b)) for a, b in hw.tolist()]


def cu_seqlens_from_lengths(lengths) -> torch.Tensor:
    cu = [0]
    for n in lengths:
        cu.append(cu[-1] + int(n))
    return torch.tensor(cu, dtype=torch.int32)


def cfg3_varlen(seed: int = 0, images: int = 32, heads: int = VIT_HEADS, head_dim: int = VIT_HEAD_DIM,
                lo: int = 16, hi: int = 64, dtype=torch.bfloat16, device="cpu"):
    """Packed q/k/v [1, H, T, D] and int32 cu_seqlens for `images` patch grids."""
    grids = cfg3_grids(seed, images, lo, hi)
    lens = [h * w for h, w in grids]
    T = sum(lens)
    g = generator(seed + 1, device)
    q = randn((1, heads, T, head_dim), g, dtype, device)
    k = randn((1, heads, T, head_dim), g, dtype, device)
    v = randn((1, heads, T, head_dim), g, dtype, device)
    return q, k, v, cu_seqlens_from_lengths(lens).to(device), lens


def cfg4_prefill(seed: int = 0, batch: int = 8, seq: int = 2048, hq: int = HQ, hkv: int = HKV,
                 head_dim: int = HEAD_DIM, dtype=torch.bfloat16, device="cpu"):
    """q/k (rotated with multimodal RoPE) and v for causal prefill; q [B,Hq,S,D]."""
    g = generator(seed, device)
    q = randn((batch, hq, seq, head_dim), g, dtype, device)
    k = randn((batch, hkv, seq, head_dim), g, dtype, device)
    v = randn((batch, hkv, seq, head_dim), g, dtype, device)
    text_before = min(100, seq // 4)
    gh = max(1, min(32, (seq - text_before) // 64))
    gw = max(1, min(50, (seq - text_before) // (2 * gh)))
    ids = mixed_prompt_position_ids(batch, seq, text_before, (gh, gw)).to(device)
    cos, sin = mrope_cos_sin(ids, dtype, head_dim)
    return rope_reference_torch(q, cos, sin), rope_reference_torch(k, cos, sin), v


def cfg5_decode(seed: int = 0, batch: int = 4, length: int = 131072, dtype=torch.bfloat16, device="cpu"):
    g = generator(seed, device)
    q = randn((batch, HQ, 1, HEAD_DIM), g, dtype, device)
    k = randn((batch, HKV, length, HEAD_DIM), g, dtype, device)
    v = randn((batch, HKV, length, HEAD_DIM), g, dtype, device)
    return q, k, v
