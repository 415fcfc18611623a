"""Restatement of Qwen3-VL's text RoPE on CPU (test infrastructure).

Follows transformers 5.5.0 (third-party host framework of the reference,
models/qwen3_vl/modeling_qwen3_vl.py):
  * ``inv_freq``            - default RoPE init (:330-350)
  * ``mrope_cos_sin``       - Qwen3VLTextRotaryEmbedding.forward + apply_interleaved_mrope (:352-387)
  * ``apply_rope``          - apply_rotary_pos_emb / rotate_half (:410-432), with the
                              per-op rounding torch applies to 16-bit tensors
  * ``rms_norm_heads``      - Qwen3VLTextRMSNorm (:389-406) applied per head
  * ``apply_rope_vision``   - apply_rotary_pos_emb_vision (:131-142): the same rotate-half
                              form in fp32 (each product and the sum rounded as fp32), the
                              result rounded once to the tensor dtype
"""
from __future__ import annotations

import numpy as np


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Rounds float32 values to bf16 / fp16 (round-to-nearest-even) and returns
    them as float32; 'fp32' is the identity."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "fp32":
        return x
    if dtype == "fp16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        u = x.view(np.uint32).astype(np.uint64)
        nan = np.isnan(x)
        r = ((u >> 16) & 1) + 0x7FFF
        u = ((u + r) & 0xFFFF0000).astype(np.uint32)
        out = u.view(np.float32).copy()
        out[nan] = np.nan
        return out
    raise ValueError(dtype)


def inv_freq(head_dim: int, theta: float) -> np.ndarray:
    """1 / theta^(2i/D), i < D/2, in float32 as the default RoPE init computes it."""
    exps = (np.arange(0, head_dim, 2, dtype=np.int64).astype(np.float32) / np.float32(head_dim)).astype(np.float32)
    return (np.float32(1.0) / (np.float32(theta) ** exps).astype(np.float32)).astype(np.float32)


def mrope_cos_sin(position_ids: np.ndarray, head_dim: int, theta: float, mrope_section, dtype: str):
    """position_ids [3, B, S] (temporal, height, width) -> cos, sin [B, S, D].

    The D/2 frequencies are taken from the T axis except the interleaved slots
    1::3 (H, up to 3*section[1]) and 2::3 (W, up to 3*section[2]); the table is
    then duplicated to D columns (cat(freqs, freqs)) and rounded to ``dtype``."""
    inv = inv_freq(head_dim, theta)
    pos = np.asarray(position_ids, dtype=np.float32)
    freqs = (pos[..., None] * inv[None, None, None, :]).astype(np.float32)  # [3, B, S, D/2]
    ft = freqs[0].copy()
    for axis, offset in ((1, 1), (2, 2)):
        length = mrope_section[axis] * 3
        ft[..., offset:length:3] = freqs[axis][..., offset:length:3]
    emb = np.concatenate([ft, ft], axis=-1)
    return round_to(np.cos(emb), dtype), round_to(np.sin(emb), dtype)


def rotate_half(x: np.ndarray) -> np.ndarray:
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, dtype: str) -> np.ndarray:
    """x [B, H, S, D], cos/sin [B, S, D] -> x*cos + rotate_half(x)*sin, with each
    product and the sum rounded to ``dtype`` as torch does for 16-bit tensors."""
    x = np.asarray(x, dtype=np.float32)
    c = np.asarray(cos, dtype=np.float32)[:, None]
    s = np.asarray(sin, dtype=np.float32)[:, None]
    a = round_to(x * c, dtype)
    b = round_to(rotate_half(x) * s, dtype)
    return round_to(a + b, dtype)


def rms_norm_heads(x: np.ndarray, weight: np.ndarray, eps: float, dtype: str) -> np.ndarray:
    """Qwen3VLTextRMSNorm over the last dim: w * to_dtype(x * rsqrt(mean(x^2) + eps))."""
    x = np.asarray(x, dtype=np.float32)
    var = (x.astype(np.float64) ** 2).mean(axis=-1, keepdims=True).astype(np.float32)
    y = round_to(x * (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32), dtype)
    return round_to(np.asarray(weight, dtype=np.float32) * y, dtype)


def apply_rope_vision(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, dtype: str) -> np.ndarray:
    """x [T, H, D] (values of ``dtype``), cos/sin [T, D] fp32 -> rotated x as
    ``dtype`` values in float32: (x * cos) + (rotate_half(x) * sin) in fp32."""
    x = np.asarray(x, dtype=np.float32)
    c = np.asarray(cos, dtype=np.float32)[:, None, :]
    s = np.asarray(sin, dtype=np.float32)[:, None, :]
    h = x.shape[-1] // 2
    rot = np.concatenate([-x[..., h:], x[..., :h]], axis=-1)
    return round_to((x * c).astype(np.float32) + (rot * s).astype(np.float32), dtype)
