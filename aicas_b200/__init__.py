"""aicas_b200: sm_100a attention backend for the Qwen3-VL-2B inference hot path.

Public surface = the reference package ``triton_qwen3vl``'s ``__all__``
(triton_qwen3vl/__init__.py:1-16 in the reference project) plus the operators
it leaves to Hugging Face or lacks: :func:`rope_kv_append`,
:func:`gqa_decode_partial` and :func:`merge_partials`, and the decode-side
products of its native decode path (:func:`decode_linear`).
"""
from . import _native
from .backends import TEXT_BACKEND_KEY, VISION_BACKEND_KEY, text_triton_attention, vision_triton_attention
from .ops import (
    decode_linear,
    gqa_decode_attention,
    gqa_decode_partial,
    gqa_flash_attention,
    merge_partials,
    rope_kv_append,
    varlen_flash_attention,
    vision_rope,
)
from .patch import install_qwen3vl_triton_attention


def __getattr__(name: str):
    """``TRITON_AVAILABLE`` / ``NATIVE_AVAILABLE``: in the reference the first
    says whether Triton imported (dense_flash_attention.py:7-15); here both say
    whether the native library loads.  They are computed on first use, so that
    importing the package (for its seeded workloads, say) maps no library."""
    if name in ("TRITON_AVAILABLE", "NATIVE_AVAILABLE"):
        return _native.available()
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")

__all__ = [
    "NATIVE_AVAILABLE",
    "TEXT_BACKEND_KEY",
    "TRITON_AVAILABLE",
    "VISION_BACKEND_KEY",
    "decode_linear",
    "gqa_decode_attention",
    "gqa_decode_partial",
    "gqa_flash_attention",
    "install_qwen3vl_triton_attention",
    "merge_partials",
    "rope_kv_append",
    "text_triton_attention",
    "varlen_flash_attention",
    "vision_rope",
    "vision_triton_attention",
]
