"""Restatement of the decode-side products on CPU (test infrastructure only:
the GPU tests check ``aicas_decode_linear`` against it; nothing in the package
calls it).

What the kernel computes, written out in numpy with the per-op rounding torch
applies to 16-bit tensors (transformers 5.5.0, models/qwen3_vl/modeling_qwen3_vl.py):

* ``rms_norm_rows``  - Qwen3VLTextRMSNorm.forward (:398-403): fp32 mean of
                        squares, x * rsqrt(var + eps) rounded to the dtype, then
                        weight * that, rounded again
* ``decode_linear``  - x' W^T for each weight, accumulated exactly (fp64); the
                        reference's native matrix-vector kernels accumulate in
                        fp32 (dujunbaoV1/native_cuda_ops/decode_q1_gqa_kernel.cu:
                        174-331) and so does the tensor-core kernel
  - ``residual``      residual + round(x' W^T): the two residual adds of
                        Qwen3VLTextDecoderLayer.forward (:557, :563)
  - ``swiglu``        round(silu(round(x' Wg^T))) * round(x' Wu^T):
                        Qwen3VLTextMLP.forward (:519-521) with its roundings

Results are returned before the final rounding to the output dtype, so a test
can hold the kernel to a tolerance against them.
"""
from __future__ import annotations

import numpy as np

from .rope import round_to


def rms_norm_rows(x: np.ndarray, w: np.ndarray, eps: float, dtype: str) -> np.ndarray:
    xf = np.asarray(x, dtype=np.float32)
    var = np.mean(xf.astype(np.float64) ** 2, axis=-1, keepdims=True).astype(np.float32)
    rstd = (1.0 / np.sqrt(var.astype(np.float64) + eps)).astype(np.float32)
    h = round_to(xf * rstd, dtype)
    return round_to(np.asarray(w, dtype=np.float32) * h, dtype)


def decode_linear(x, weights, *, norm_weight=None, eps=1e-6, residual=None, swiglu=False,
                  dtype: str = "bf16") -> list[np.ndarray]:
    """Per output: float64 values before the last rounding to ``dtype``."""
    xn = rms_norm_rows(x, norm_weight, eps, dtype) if norm_weight is not None else np.asarray(x, np.float32)
    xd = xn.astype(np.float64)
    accs = [xd @ np.asarray(w, dtype=np.float64).T for w in weights]
    if swiglu:
        g = round_to(accs[0], dtype).astype(np.float64)
        s = round_to(g / (1.0 + np.exp(-g)), dtype).astype(np.float64)
        u = round_to(accs[1], dtype).astype(np.float64)
        return [s * u]
    if residual is not None:
        return [np.asarray(residual, np.float64) + round_to(accs[0], dtype).astype(np.float64)]
    return accs
