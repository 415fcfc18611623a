"""The preallocated cache layer on CPU: in-place appends, views of the valid
prefix, mask sizes, the capacity check, and a shrunken Qwen3-VL giving the
same logits with it as with Hugging Face's DynamicCache over a prefill and
three decode steps (SDPA attention; the CUDA-graph step itself needs a GPU and
is covered by tests/test_gpu_generate.py)."""
from __future__ import annotations

import pytest
import torch
from transformers.cache_utils import DynamicCache

from aicas_b200 import integration as it
from aicas_b200.decode_graph import StaticKVCache, StaticKVLayer


def test_layer_appends_in_place_and_returns_the_prefix():
    layer = StaticKVLayer(capacity=8)
    k1, v1 = torch.randn(2, 3, 5, 4), torch.randn(2, 3, 5, 4)
    k, v = layer.update(k1, v1)
    assert k.shape == (2, 3, 5, 4) and torch.equal(k, k1) and torch.equal(v, v1)
    base = layer.keys.data_ptr()
    k2, v2 = torch.randn(2, 3, 1, 4), torch.randn(2, 3, 1, 4)
    k, v = layer.update(k2, v2)
    assert layer.keys.data_ptr() == base  # never re-allocated
    assert k.shape == (2, 3, 6, 4) and k.data_ptr() == base
    assert torch.equal(k[:, :, 5:], k2) and torch.equal(v[:, :, :5], v1)
    assert layer.get_seq_length() == 6 and layer.get_max_cache_shape() == 8
    assert layer.get_mask_sizes(1) == (7, 0)
    with pytest.raises(ValueError):
        layer.update(torch.randn(2, 3, 3, 4), torch.randn(2, 3, 3, 4))  # 9 > 8
    layer.reset()
    assert layer.get_seq_length() == 0


def test_same_logits_as_dynamic_cache_on_a_tiny_model():
    cfg = it.qwen3vl_config(
        dict(hidden_size=128, intermediate_size=256, num_hidden_layers=2, num_attention_heads=4,
             num_key_value_heads=2, head_dim=32),
        dict(depth=2, hidden_size=64, intermediate_size=128, num_heads=4, out_hidden_size=128,
             deepstack_visual_indexes=[0]))
    model = it.build_random_model(cfg, torch.float32, "cpu", seed=3)
    inp = it.synthetic_prompt(cfg, batch=2, seq_len=40, grid_hw=(4, 6), text_before=6)
    with torch.no_grad():
        outs = []
        for cache in (DynamicCache(config=cfg.text_config), StaticKVCache(cfg.text_config.num_hidden_layers, 44)):
            model.model.rope_deltas = None
            o = model(**inp, past_key_values=cache, use_cache=True)
            logits = [o.logits[:, -1]]
            tok = o.logits[:, -1].argmax(-1, keepdim=True)
            for _ in range(3):
                # a decode step: the new token only; without a mask (no padding) the
                # model places it after the cached length, plus the prompt's rope delta
                o = model(input_ids=tok, past_key_values=cache, use_cache=True)
                logits.append(o.logits[:, -1])
                tok = o.logits[:, -1].argmax(-1, keepdim=True)
            outs.append(torch.stack(logits))
            assert cache.get_seq_length() == 43
    torch.testing.assert_close(outs[1], outs[0], rtol=1e-5, atol=1e-5)
