"""Dispatch and API-surface tests, ported from the reference's CPU tests
(test/test_qwen3vl_triton_patch.py:22-383 in the reference project) to this
backend, which has no SDPA fallback: where the reference fell back, these
tests expect a ValueError.  CPU only (the operators are monkeypatched)."""
from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

import aicas_b200
from aicas_b200 import backends, ops, patch


class DummyRegistry(dict):
    def register(self, name, fn):
        self[name] = fn


class DummyAttentionModule(torch.nn.Module):
    def __init__(self, *, num_key_value_groups: int = 1, scaling: float = 0.125, is_causal: bool = True):
        super().__init__()
        self.num_key_value_groups = num_key_value_groups
        self.scaling = scaling
        self.is_causal = is_causal


def _build_fake_model():
    return SimpleNamespace(
        model=SimpleNamespace(
            visual=SimpleNamespace(config=SimpleNamespace(_attn_implementation="sdpa")),
            language_model=SimpleNamespace(config=SimpleNamespace(_attn_implementation="sdpa")),
        ),
        config=SimpleNamespace(
            vision_config=SimpleNamespace(_attn_implementation="sdpa"),
            text_config=SimpleNamespace(_attn_implementation="sdpa"),
        ),
    )


def test_backend_keys_are_the_reference_strings():
    assert backends.TEXT_BACKEND_KEY == "qwen3vl_triton_flash_text"
    assert backends.VISION_BACKEND_KEY == "qwen3vl_triton_flash_vision"
    # HF hands cu_seqlens to the vision attention only for "flash" implementations
    assert "flash" in backends.TEXT_BACKEND_KEY and "flash" in backends.VISION_BACKEND_KEY


def test_public_api_covers_the_reference_all():
    import triton_qwen3vl

    reference_all = {
        "TEXT_BACKEND_KEY", "TRITON_AVAILABLE", "VISION_BACKEND_KEY", "gqa_decode_attention",
        "gqa_flash_attention", "install_qwen3vl_triton_attention", "varlen_flash_attention",
    }
    assert reference_all <= set(aicas_b200.__all__)
    for name in reference_all:
        assert getattr(triton_qwen3vl, name) is getattr(aicas_b200, name)
    from triton_qwen3vl.backends import text_triton_attention, vision_triton_attention  # noqa: F401


def test_install_registers_backends_and_mutates_configs(monkeypatch):
    attention_registry = DummyRegistry()
    mask_sentinel = object()
    mask_registry = DummyRegistry({"flash_attention_2": mask_sentinel})
    monkeypatch.setattr(patch, "_load_attention_registries", lambda: (attention_registry, mask_registry))
    model = _build_fake_model()
    state = patch.install_qwen3vl_triton_attention(model)
    assert attention_registry[backends.VISION_BACKEND_KEY] is backends.vision_triton_attention
    assert attention_registry[backends.TEXT_BACKEND_KEY] is backends.text_triton_attention
    assert mask_registry[backends.VISION_BACKEND_KEY] is mask_sentinel
    assert mask_registry[backends.TEXT_BACKEND_KEY] is mask_sentinel
    assert model.model.visual.config._attn_implementation == backends.VISION_BACKEND_KEY
    assert model.model.language_model.config._attn_implementation == backends.TEXT_BACKEND_KEY
    assert model.config.vision_config._attn_implementation == backends.VISION_BACKEND_KEY
    assert model.config.text_config._attn_implementation == backends.TEXT_BACKEND_KEY
    assert state["installed"] is True
    assert set(state) == {
        "installed", "triton_available", "vision_backend_key", "text_backend_key", "vision_varlen_triton_enabled",
        "text_prefill_gqa_triton_enabled", "text_decode_triton_enabled", "mutated_configs",
    }
    assert all(state["mutated_configs"].values())


def test_install_is_idempotent_and_tolerates_missing_configs(monkeypatch):
    attention_registry = DummyRegistry()
    mask_registry = DummyRegistry({"flash_attention_2": object()})
    monkeypatch.setattr(patch, "_load_attention_registries", lambda: (attention_registry, mask_registry))
    state1 = patch.install_qwen3vl_triton_attention(SimpleNamespace())
    state2 = patch.install_qwen3vl_triton_attention(SimpleNamespace())
    assert not any(state1["mutated_configs"].values())
    assert state1["mutated_configs"] == state2["mutated_configs"]
    assert len(attention_registry) == 2


def test_install_against_real_hf_registries():
    from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    state = patch.install_qwen3vl_triton_attention(_build_fake_model())
    assert ALL_ATTENTION_FUNCTIONS[backends.TEXT_BACKEND_KEY] is backends.text_triton_attention
    assert ALL_ATTENTION_FUNCTIONS[backends.VISION_BACKEND_KEY] is backends.vision_triton_attention
    assert ALL_MASK_ATTENTION_FUNCTIONS[backends.TEXT_BACKEND_KEY] is ALL_MASK_ATTENTION_FUNCTIONS["flash_attention_2"]
    assert state["installed"]


def test_text_attention_uses_decode_kernel_for_single_token(monkeypatch):
    sentinel = torch.arange(1 * 4 * 1 * 4, dtype=torch.float32).reshape(1, 4, 1, 4)
    recorded = {}

    def fake_decode(query, key, value, **kwargs):
        recorded.update(kwargs)
        return sentinel

    def unexpected(*args, **kwargs):
        raise AssertionError("decode must not call the prefill kernel")

    monkeypatch.setattr(ops, "gqa_decode_attention", fake_decode)
    monkeypatch.setattr(ops, "gqa_flash_attention", unexpected)
    module = DummyAttentionModule(num_key_value_groups=2, scaling=0.25)
    out, weights = backends.text_triton_attention(module, torch.randn(1, 4, 1, 4), torch.randn(1, 2, 5, 4),
                                                  torch.randn(1, 2, 5, 4), attention_mask=None, dropout=0.0,
                                                  scaling=None)
    assert recorded["sm_scale"] == module.scaling
    assert recorded["num_key_value_groups"] == 2
    assert weights is None
    assert torch.equal(out, sentinel.transpose(1, 2).contiguous())


def test_text_attention_uses_gqa_prefill_kernel(monkeypatch):
    sentinel = torch.arange(1 * 4 * 5 * 4, dtype=torch.float32).reshape(1, 4, 5, 4)
    recorded = {}

    def fake_gqa(query, key, value, **kwargs):
        recorded.update(kwargs)
        return sentinel

    monkeypatch.setattr(ops, "gqa_flash_attention", fake_gqa)
    module = DummyAttentionModule(num_key_value_groups=2, scaling=0.25, is_causal=True)
    out, weights = backends.text_triton_attention(module, torch.randn(1, 4, 5, 4), torch.randn(1, 2, 5, 4),
                                                  torch.randn(1, 2, 5, 4), attention_mask=None, dropout=0.0,
                                                  scaling=None)
    assert recorded["sm_scale"] == module.scaling
    assert recorded["num_key_value_groups"] == 2
    assert recorded["causal"] is True
    assert weights is None
    assert torch.equal(out, sentinel.transpose(1, 2).contiguous())


def test_explicit_scaling_overrides_module_scaling(monkeypatch):
    recorded = {}
    monkeypatch.setattr(ops, "gqa_decode_attention", lambda q, k, v, **kw: recorded.update(kw) or q)
    backends.text_triton_attention(DummyAttentionModule(scaling=0.25), torch.randn(1, 2, 1, 4),
                                   torch.randn(1, 2, 3, 4), torch.randn(1, 2, 3, 4), None, scaling=0.5)
    assert recorded["sm_scale"] == 0.5


@pytest.mark.parametrize(
    "kwargs, q_len, kv_len, match",
    [
        ({"attention_mask": torch.ones(1, 1, 5, 5)}, 5, 5, "mask"),
        ({"attention_mask": None, "dropout": 0.1}, 5, 5, "dropout"),
        ({"attention_mask": None, "output_attentions": True}, 5, 5, "output_attentions"),
        ({"attention_mask": None}, 3, 5, "q_len == kv_len"),
    ],
)
def test_text_attention_raises_where_the_reference_fell_back(kwargs, q_len, kv_len, match):
    module = DummyAttentionModule(num_key_value_groups=2)
    with pytest.raises(ValueError, match=match):
        backends.text_triton_attention(module, torch.randn(1, 4, q_len, 8), torch.randn(1, 2, kv_len, 8),
                                       torch.randn(1, 2, kv_len, 8), **kwargs)


def test_vision_attention_uses_varlen_kernel(monkeypatch):
    sentinel = torch.arange(1 * 2 * 5 * 4, dtype=torch.float32).reshape(1, 2, 5, 4)
    recorded = {}

    def fake_varlen(query, key, value, **kwargs):
        recorded.update(kwargs)
        return sentinel

    monkeypatch.setattr(ops, "varlen_flash_attention", fake_varlen)
    module = DummyAttentionModule(num_key_value_groups=1, scaling=0.25, is_causal=False)
    cu = torch.tensor([0, 2, 5], dtype=torch.int32)
    out, weights = backends.vision_triton_attention(module, torch.randn(1, 2, 5, 4), torch.randn(1, 2, 5, 4),
                                                    torch.randn(1, 2, 5, 4), attention_mask=None, dropout=0.0,
                                                    scaling=None, cu_seq_lens_q=cu, cu_seq_lens_k=cu,
                                                    max_length_q=3, max_length_k=3, is_causal=False)
    assert recorded["sm_scale"] == module.scaling
    assert recorded["max_length_q"] == 3 and recorded["max_length_k"] == 3
    assert recorded["cu_seq_lens_q"] is cu
    assert isinstance(recorded["metadata_cache"], dict)
    assert hasattr(module, "_qwen3vl_vision_varlen_metadata_cache")
    assert weights is None
    assert torch.equal(out, sentinel.transpose(1, 2).contiguous())


def test_vision_attention_without_cu_seqlens_is_one_segment(monkeypatch):
    recorded = {}
    monkeypatch.setattr(ops, "varlen_flash_attention", lambda q, k, v, **kw: recorded.update(kw) or q)
    module = DummyAttentionModule(is_causal=False)
    backends.vision_triton_attention(module, torch.randn(1, 2, 7, 4), torch.randn(1, 2, 7, 4),
                                     torch.randn(1, 2, 7, 4), is_causal=False)
    assert recorded["cu_seq_lens_q"].tolist() == [0, 7]


def test_vision_attention_rejects_causal():
    with pytest.raises(ValueError, match="non-causal"):
        backends.vision_triton_attention(DummyAttentionModule(is_causal=True), torch.randn(1, 2, 5, 4),
                                         torch.randn(1, 2, 5, 4), torch.randn(1, 2, 5, 4))


def test_gqa_flash_attention_rejects_non_causal():
    with pytest.raises(ValueError, match="only supports causal prefill"):
        ops.gqa_flash_attention(torch.randn(1, 4, 5, 64), torch.randn(1, 2, 5, 64), torch.randn(1, 2, 5, 64),
                                causal=False, sm_scale=0.125, num_key_value_groups=2)


@pytest.mark.parametrize("op", ["decode", "prefill", "varlen"])
def test_operators_refuse_cpu_tensors(op):
    """No CPU fallback in the product path: CPU tensors are rejected."""
    with pytest.raises(ValueError, match="CUDA"):
        if op == "decode":
            ops.gqa_decode_attention(torch.randn(1, 4, 1, 64), torch.randn(1, 2, 9, 64), torch.randn(1, 2, 9, 64),
                                     sm_scale=0.125, num_key_value_groups=2)
        elif op == "prefill":
            ops.gqa_flash_attention(torch.randn(1, 4, 9, 64), torch.randn(1, 2, 9, 64), torch.randn(1, 2, 9, 64),
                                    causal=True, sm_scale=0.125, num_key_value_groups=2)
        else:
            cu = torch.tensor([0, 9], dtype=torch.int32)
            ops.varlen_flash_attention(torch.randn(1, 2, 9, 64), torch.randn(1, 2, 9, 64), torch.randn(1, 2, 9, 64),
                                       cu_seq_lens_q=cu, cu_seq_lens_k=cu, sm_scale=0.125)


def test_operators_refuse_autograd():
    q = torch.randn(1, 4, 1, 64, requires_grad=True)
    with pytest.raises(ValueError, match="inference"):
        ops.gqa_decode_attention(q, torch.randn(1, 2, 9, 64), torch.randn(1, 2, 9, 64), sm_scale=0.1,
                                 num_key_value_groups=2)
