"""``install_qwen3vl_triton_attention``: registers the two attention backends in
Hugging Face's registries and switches a Qwen3-VL model over to them.

Same contract as triton_qwen3vl/patch.py:23-63 (path relative to the reference
project): both keys are registered in ``ALL_ATTENTION_FUNCTIONS`` and mapped to
the ``flash_attention_2`` mask function in ``ALL_MASK_ATTENTION_FUNCTIONS``;
``_attn_implementation`` is set on the four config objects that exist; the
returned dict has the same keys.  ``triton_available`` (kept under its
reference name) reports whether the sm_100a library is loadable.
"""
from __future__ import annotations

from typing import Any

from . import _native
from .backends import TEXT_BACKEND_KEY, VISION_BACKEND_KEY, text_triton_attention, vision_triton_attention


def _load_attention_registries():
    from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    return ALL_ATTENTION_FUNCTIONS, ALL_MASK_ATTENTION_FUNCTIONS


def _switch_backend(config: Any, key: str) -> bool:
    """Points one config object's ``_attn_implementation`` at ``key``; False
    (and nothing changed) when the model has no such config object."""
    has_field = config is not None and hasattr(config, "_attn_implementation")
    if has_field:
        config._attn_implementation = key
    return has_field


def install_qwen3vl_triton_attention(model: Any, fuse_vision_rope: bool = False) -> dict[str, Any]:
    """``fuse_vision_rope=True`` (an extension; the reference has no such
    switch) also runs the vision attention's QKV split + RoPE as one kernel
    (:mod:`aicas_b200.vision`) and adds ``vision_rope_fused`` (modules
    switched) to the returned dict."""
    attention_registry, mask_registry = _load_attention_registries()

    if VISION_BACKEND_KEY not in attention_registry:
        attention_registry.register(VISION_BACKEND_KEY, vision_triton_attention)
    if TEXT_BACKEND_KEY not in attention_registry:
        attention_registry.register(TEXT_BACKEND_KEY, text_triton_attention)
    if VISION_BACKEND_KEY not in mask_registry:
        mask_registry.register(VISION_BACKEND_KEY, mask_registry["flash_attention_2"])
    if TEXT_BACKEND_KEY not in mask_registry:
        mask_registry.register(TEXT_BACKEND_KEY, mask_registry["flash_attention_2"])

    base_model = getattr(model, "model", None)
    visual = getattr(base_model, "visual", None)
    language_model = getattr(base_model, "language_model", None)
    model_config = getattr(model, "config", None)
    mutated = {
        "model.model.visual.config": _switch_backend(getattr(visual, "config", None), VISION_BACKEND_KEY),
        "model.model.language_model.config": _switch_backend(getattr(language_model, "config", None), TEXT_BACKEND_KEY),
        "model.config.vision_config": _switch_backend(getattr(model_config, "vision_config", None), VISION_BACKEND_KEY),
        "model.config.text_config": _switch_backend(getattr(model_config, "text_config", None), TEXT_BACKEND_KEY),
    }
    available = _native.available()
    extra = {}
    if fuse_vision_rope:
        from .vision import install_vision_rope_fusion

        extra["vision_rope_fused"] = install_vision_rope_fusion(model)
    return {
        **extra,
        "installed": True,
        "triton_available": available,
        "vision_backend_key": VISION_BACKEND_KEY,
        "text_backend_key": TEXT_BACKEND_KEY,
        "vision_varlen_triton_enabled": available,
        "text_prefill_gqa_triton_enabled": available,
        "text_decode_triton_enabled": available,
        "mutated_configs": mutated,
    }
