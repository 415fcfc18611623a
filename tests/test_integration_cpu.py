"""Host side of the end-to-end integration check, on CPU with a shrunken
Qwen3-VL: the synthetic multimodal prompt, the greedy generate helper, the
comparison metrics, and the switch between SDPA and this backend."""
from __future__ import annotations

import pytest
import torch

from aicas_b200 import integration as it
from aicas_b200.backends import TEXT_BACKEND_KEY, VISION_BACKEND_KEY

TINY_TEXT = dict(hidden_size=128, intermediate_size=256, num_hidden_layers=2, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=32)
TINY_VISION = dict(depth=2, hidden_size=64, intermediate_size=128, num_heads=4, out_hidden_size=128,
                   deepstack_visual_indexes=[0])


@pytest.fixture(scope="module")
def tiny():
    cfg = it.qwen3vl_config(TINY_TEXT, TINY_VISION)
    return cfg, it.build_random_model(cfg, torch.float32, "cpu", seed=0)


def test_full_config_has_the_attention_shapes_the_kernels_serve():
    cfg = it.qwen3vl_config()
    t, v = cfg.text_config, cfg.vision_config
    assert (t.num_hidden_layers, t.num_attention_heads, t.num_key_value_heads, t.head_dim) == (28, 16, 8, 128)
    assert (v.hidden_size, v.num_heads, v.hidden_size // v.num_heads) == (1024, 16, 64)
    assert t.rope_scaling["mrope_section"] == [24, 20, 20]


def test_synthetic_prompt_layout(tiny):
    cfg, _ = tiny
    inp = it.synthetic_prompt(cfg, batch=3, seq_len=80, grid_hw=(6, 8), text_before=10)
    ids, mm = inp["input_ids"], inp["mm_token_type_ids"]
    n_img = 6 * 8 // 4
    assert ids.shape == (3, 80) and mm.shape == (3, 80)
    assert (ids[:, 10] == it.VISION_START_TOKEN_ID).all()
    assert (ids[:, 11:11 + n_img] == it.IMAGE_TOKEN_ID).all()
    assert (ids[:, 11 + n_img] == it.VISION_END_TOKEN_ID).all()
    assert int(mm.sum()) == 3 * n_img and (mm[:, 11:11 + n_img] == 1).all()
    assert inp["pixel_values"].shape == (3 * 6 * 8, 3 * 2 * 16 * 16)
    assert inp["image_grid_thw"].tolist() == [[1, 6, 8]] * 3
    with pytest.raises(ValueError):
        it.synthetic_prompt(cfg, 1, 20, grid_hw=(6, 8), text_before=10)  # too short for the image
    with pytest.raises(ValueError):
        it.synthetic_prompt(cfg, 1, 80, grid_hw=(5, 8))  # not divisible by the 2x2 merge


def test_greedy_generate_and_teacher_forced_gap(tiny):
    cfg, model = tiny
    inp = it.synthetic_prompt(cfg, batch=2, seq_len=48, grid_hw=(4, 6), text_before=8)
    run = it.greedy_generate(model, inp, 4)
    assert run.tokens.shape == (2, 4) and run.seconds > 0 and run.ttft_seconds > 0
    # the model's own greedy tokens are its argmax at every position: gap 0
    gap = it.teacher_forced_gap(model, inp, run.tokens)
    assert gap.shape == (2, 4) and float(gap.abs().max()) < 1e-4
    # a token other than the argmax shows a positive gap
    other = run.tokens.clone()
    other[:, 0] = (other[:, 0] + 1) % cfg.text_config.vocab_size
    assert float(it.teacher_forced_gap(model, inp, other)[:, 0].min()) > 0


def test_forced_choices_reproduce_the_greedy_run_and_see_a_wrong_attention(tiny):
    """Fed its own greedy tokens, the same model picks them at every position;
    a continuation that is not its own is followed all the same (each step sees
    the forced prefix), and the perturbed-attention control disagrees somewhere."""
    cfg, model = tiny
    inp = it.synthetic_prompt(cfg, batch=2, seq_len=48, grid_hw=(4, 6), text_before=8)
    it.set_attention(model, "sdpa")
    run = it.greedy_generate(model, inp, 6, timed=False)
    assert torch.equal(it.forced_choices(model, inp, run.tokens), run.tokens)
    other = torch.randint(0, 1000, run.tokens.shape)
    choices = it.forced_choices(model, inp, other)
    assert choices.shape == other.shape and torch.equal(choices[:, 0], run.tokens[:, 0])
    it.set_text_attention_control(model)
    try:
        assert it.attention_in_use(model)[1] == it.PERTURBED_KEY
        ctrl = it.forced_choices(model, inp, run.tokens)
        assert ctrl.shape == run.tokens.shape
    finally:
        it.set_attention(model, "sdpa")


def test_token_match_counts_up_to_the_first_divergence():
    a = torch.tensor([[1, 2, 3, 4], [5, 6, 7, 8]])
    b = torch.tensor([[1, 2, 0, 4], [5, 6, 7, 8]])
    assert it.token_match(a, b) == pytest.approx((2 + 4) / 8)
    assert it.token_match(a, a) == 1.0


def test_attention_switch(tiny, monkeypatch):
    _, model = tiny
    it.set_attention(model, "sdpa")
    assert it.attention_in_use(model) == ("sdpa", "sdpa")
    from aicas_b200 import _native

    monkeypatch.setattr(_native, "available", lambda: True)
    it.set_attention(model, "aicas")
    assert it.attention_in_use(model) == (VISION_BACKEND_KEY, TEXT_BACKEND_KEY)
    assert model.model.language_model.config._attn_implementation == TEXT_BACKEND_KEY
    it.set_attention(model, "sdpa")
    assert it.attention_in_use(model) == ("sdpa", "sdpa")
    monkeypatch.setattr(_native, "available", lambda: False)
    with pytest.raises(RuntimeError):
        it.set_attention(model, "aicas")  # no silent fallback when the library is missing
    it.set_attention(model, "sdpa")
    with pytest.raises(ValueError):
        it.set_attention(model, "eager")


def test_vision_rope_fusion_switch(tiny):
    """fuse_vision_rope=True puts the fused forward on every vision attention
    module and reports how many; switching back to SDPA restores Hugging
    Face's forward (no kernel runs here)."""
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLVisionAttention

    from aicas_b200 import install_qwen3vl_triton_attention
    from aicas_b200.vision import fused_vision_attention_forward

    cfg, model = tiny
    mods = [m for m in model.modules() if isinstance(m, Qwen3VLVisionAttention)]
    assert len(mods) == cfg.vision_config.depth
    state = install_qwen3vl_triton_attention(model)
    assert "vision_rope_fused" not in state and all("forward" not in m.__dict__ for m in mods)
    state = install_qwen3vl_triton_attention(model, fuse_vision_rope=True)
    assert state["vision_rope_fused"] == len(mods)
    assert all(m.forward.__func__ is fused_vision_attention_forward for m in mods)
    it.set_attention(model, "sdpa")
    assert all("forward" not in m.__dict__ for m in mods)
    assert it.attention_in_use(model) == ("sdpa", "sdpa")
