"""End-to-end integration check: greedy generation on a random-init model with
Qwen3-VL-2B's architecture, switched to this backend by
:func:`install_qwen3vl_triton_attention`, against the same weights on
PyTorch SDPA attention.

The check follows the organiser harness of the reference project
(evaluation_wrapper.py:40-66 loads the model, :380-405 installs the attention
patch, :505-516 runs ``model.generate`` greedily with the KV cache on), with
three differences forced by an offline box: the weights are random (seeded),
the prompt is synthetic (a text span, one image of ``grid_hw`` patches between
the vision start/end tokens, more text; the mixed image+text prompt of the
causal-prefill workload), and the pixels are seeded noise.  The architecture
numbers below are those of the public Qwen3-VL-2B-Instruct configuration; the
attention shapes they give are the ones the kernels are built and measured on
(text: 16 query heads over 8 KV heads at head_dim 128; vision: 16 heads at 64).

A third run generates the same tokens with :class:`GraphGreedyDecoder` (a
preallocated cache and the decode step replayed from one CUDA graph, driven by
the fused RoPE + append kernel), the serving path a deployment would use.

What is compared (the tolerances live in the tests that call these helpers):
  * ``forced_agreement``: at every position of SDPA's own greedy sequence, fed
    SDPA's tokens (teacher forcing through ``generate``, so prefill and every
    decode step run on this backend), the fraction of positions where this
    backend's greedy choice is SDPA's.  Free-running sequences of a random-init
    model part after the first near-tie and then have nothing in common, even
    between two correct attentions; this metric does not compound.  With
    ``with_control`` the same is measured for SDPA with its softmax scale off
    by 10% (``control_forced_agreement``), a wrong attention of the size a
    kernel bug makes, to show what a failing value looks like;
  * ``token_match``: the fraction of generated positions where the patched and
    the SDPA greedy sequences agree, counted up to their first divergence
    (informational: see above);
  * ``max_logit_gap``: the patched tokens fed back, teacher-forced, through
    the SDPA model: at every generated position, SDPA's best logit minus its
    logit for the patched token (0 where SDPA would pick the same token).  On
    a random-init model the top logits sit close together, so a divergence
    after a near-tie is expected; a large gap would mean the patched model
    chose a token SDPA rates as clearly worse.
"""
from __future__ import annotations

import time
from dataclasses import dataclass

import torch

from .backends import TEXT_BACKEND_KEY, VISION_BACKEND_KEY
from .patch import install_qwen3vl_triton_attention

# Qwen3-VL-2B-Instruct: language model and vision tower hyper-parameters.
QWEN3VL_2B_TEXT = dict(
    hidden_size=2048,
    intermediate_size=6144,
    num_hidden_layers=28,
    num_attention_heads=16,
    num_key_value_heads=8,
    head_dim=128,
    vocab_size=151936,
    max_position_embeddings=262144,
    rms_norm_eps=1e-6,
    rope_theta=5000000.0,
    rope_scaling={"rope_type": "default", "mrope_section": [24, 20, 20], "mrope_interleaved": True},
    tie_word_embeddings=True,
)
QWEN3VL_2B_VISION = dict(
    depth=24,
    hidden_size=1024,
    intermediate_size=4096,
    num_heads=16,
    out_hidden_size=2048,
    patch_size=16,
    spatial_merge_size=2,
    temporal_patch_size=2,
    in_channels=3,
    num_position_embeddings=2304,
    deepstack_visual_indexes=[5, 11, 17],
    hidden_act="gelu_pytorch_tanh",
)
IMAGE_TOKEN_ID = 151655
VIDEO_TOKEN_ID = 151656
VISION_START_TOKEN_ID = 151652
VISION_END_TOKEN_ID = 151653


def qwen3vl_config(text: dict | None = None, vision: dict | None = None):
    """A ``Qwen3VLConfig`` with the 2B architecture, fields overridable (the
    CPU tests shrink it)."""
    from transformers import Qwen3VLConfig

    t = dict(QWEN3VL_2B_TEXT, **(text or {}))
    v = dict(QWEN3VL_2B_VISION, **(vision or {}))
    cfg = Qwen3VLConfig(
        text_config=t,
        vision_config=v,
        image_token_id=IMAGE_TOKEN_ID,
        video_token_id=VIDEO_TOKEN_ID,
        vision_start_token_id=VISION_START_TOKEN_ID,
        vision_end_token_id=VISION_END_TOKEN_ID,
        tie_word_embeddings=t["tie_word_embeddings"],
    )
    return cfg


def build_random_model(config, dtype: torch.dtype, device: torch.device | str, seed: int = 0):
    """Random-init ``Qwen3VLForConditionalGeneration`` on ``device`` (weights
    drawn by the model's own initialiser from ``seed``), in eval mode, on SDPA."""
    from transformers import Qwen3VLForConditionalGeneration

    config._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    with torch.device(device):
        model = Qwen3VLForConditionalGeneration(config)
    model = model.to(dtype).eval()
    set_attention(model, "sdpa")
    return model


def set_attention(model, which: str) -> None:
    """Point the four config objects the patch entry point mutates at
    ``which``: "sdpa" for the unpatched baseline, "aicas" for this backend
    (through :func:`install_qwen3vl_triton_attention`, with the vision QKV
    split + RoPE fused into one kernel)."""
    from .vision import remove_vision_rope_fusion

    if which == "aicas":
        state = install_qwen3vl_triton_attention(model, fuse_vision_rope=True)
        if not state["triton_available"]:
            raise RuntimeError("the aicas_b200 native library is not loadable; the patched model cannot run")
        return
    if which != "sdpa":
        raise ValueError(f"unknown attention implementation {which!r}")
    remove_vision_rope_fusion(model)
    base = getattr(model, "model", None)
    for cfg in (
        getattr(getattr(base, "visual", None), "config", None),
        getattr(getattr(base, "language_model", None), "config", None),
        getattr(model.config, "vision_config", None),
        getattr(model.config, "text_config", None),
    ):
        if cfg is not None:
            cfg._attn_implementation = "sdpa"


def attention_in_use(model) -> tuple[str, str]:
    """(vision, text) attention implementations the model will call."""
    return model.config.vision_config._attn_implementation, model.config.text_config._attn_implementation


def synthetic_prompt(config, batch: int, seq_len: int, grid_hw: tuple[int, int] = (64, 100), text_before: int = 100,
                     seed: int = 0, dtype: torch.dtype = torch.bfloat16, device: torch.device | str = "cpu") -> dict:
    """Model inputs for ``batch`` prompts of exactly ``seq_len`` tokens, each
    ``text_before`` text tokens, <vision_start>, the image tokens of one
    ``grid_hw`` patch grid (grid_h * grid_w / merge^2 of them), <vision_end>,
    then text to fill the length.  Text ids are drawn below the special-token
    range; pixels are N(0, 1) patches as the image processor would flatten
    them (channels x temporal x patch x patch per row)."""
    vc = config.vision_config
    gh, gw = grid_hw
    merge = vc.spatial_merge_size
    if gh % merge or gw % merge:
        raise ValueError("the patch grid must be divisible by the spatial merge size")
    n_img = gh * gw // (merge * merge)
    n_after = seq_len - text_before - n_img - 2
    if n_after < 0:
        raise ValueError(f"seq_len {seq_len} cannot hold {text_before} text + {n_img} image tokens")
    g = torch.Generator().manual_seed(seed)
    text_vocab = min(config.text_config.vocab_size, VISION_START_TOKEN_ID)
    ids = torch.randint(0, text_vocab, (batch, seq_len), generator=g, dtype=torch.long)
    ids[:, text_before] = VISION_START_TOKEN_ID
    ids[:, text_before + 1:text_before + 1 + n_img] = IMAGE_TOKEN_ID
    ids[:, text_before + 1 + n_img] = VISION_END_TOKEN_ID
    mm = torch.zeros(batch, seq_len, dtype=torch.int32)
    mm[:, text_before + 1:text_before + 1 + n_img] = 1
    row = vc.in_channels * vc.temporal_patch_size * vc.patch_size * vc.patch_size
    pixels = torch.randn(batch * gh * gw, row, generator=g).to(dtype)
    thw = torch.tensor([[1, gh, gw]] * batch, dtype=torch.long)
    return {
        "input_ids": ids.to(device),
        "attention_mask": torch.ones(batch, seq_len, dtype=torch.long, device=device),
        "mm_token_type_ids": mm.to(device),
        "pixel_values": pixels.to(device),
        "image_grid_thw": thw.to(device),
    }


@dataclass
class GenerateRun:
    tokens: torch.Tensor  # [B, new] generated ids
    seconds: float  # whole generate() call, device-synchronised
    ttft_seconds: float  # generate() of one new token (prefill + first sample)
    step_ms: float = float("nan")  # device time of one decode step, where the path measures it

    @property
    def tokens_per_s(self) -> float:
        return self.tokens.numel() / self.seconds if self.seconds > 0 else float("nan")


def _sync(device) -> None:
    if torch.device(device).type == "cuda":
        torch.cuda.synchronize(device)


@torch.no_grad()
def greedy_generate(model, inputs: dict, max_new_tokens: int, timed: bool = True) -> GenerateRun:
    """``model.generate`` as the organiser harness calls it (greedy, KV cache
    on, evaluation_wrapper.py:509-516), timed on the host around
    device-synchronised calls.  TTFT is a separate one-token generate."""
    kw = dict(do_sample=False, use_cache=True, pad_token_id=0)
    device = inputs["input_ids"].device
    ttft = float("nan")
    if timed:
        _sync(device)
        t0 = time.perf_counter()
        model.generate(**inputs, max_new_tokens=1, min_new_tokens=1, **kw)
        _sync(device)
        ttft = time.perf_counter() - t0
    _sync(device)
    t0 = time.perf_counter()
    out = model.generate(**inputs, max_new_tokens=max_new_tokens, min_new_tokens=max_new_tokens, **kw)
    _sync(device)
    dt = time.perf_counter() - t0
    return GenerateRun(tokens=out[:, inputs["input_ids"].shape[1]:], seconds=dt, ttft_seconds=ttft)


class _ForceAndRecord:
    """Logits processor for ``generate``: records the model's own greedy choice
    at each step, then forces ``forced[:, step]``, so every step sees the same
    prefix as the run that produced ``forced``."""

    def __init__(self, forced: torch.Tensor):
        self.forced = forced
        self.choices: list[torch.Tensor] = []

    def __call__(self, input_ids: torch.Tensor, scores: torch.Tensor) -> torch.Tensor:
        step = len(self.choices)
        self.choices.append(scores.argmax(dim=-1))
        out = torch.full_like(scores, float("-inf"))
        out.scatter_(1, self.forced[:, step:step + 1].to(scores.device), 0.0)
        return out


@torch.no_grad()
def forced_choices(model, inputs: dict, forced: torch.Tensor) -> torch.Tensor:
    """[B, n] the model's greedy choice at each of ``forced``'s n positions when
    ``forced`` is fed back as the continuation (prefill, then n - 1 decode steps
    on the KV cache, through ``generate``)."""
    from transformers import LogitsProcessorList

    proc = _ForceAndRecord(forced)
    model.generate(**inputs, max_new_tokens=forced.shape[1], min_new_tokens=forced.shape[1], do_sample=False,
                   use_cache=True, pad_token_id=0, logits_processor=LogitsProcessorList([proc]))
    return torch.stack(proc.choices, dim=1)


def _perturbed_sdpa(module, query, key, value, attention_mask, dropout=0.0, scaling=None, **kwargs):
    """SDPA with the softmax scale off by 10%: a wrong attention of the kind a
    kernel bug would produce, for the control of the agreement metric."""
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    s = module.scaling if scaling is None else scaling
    return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout, scaling=1.1 * s, **kwargs)


PERTURBED_KEY = "aicas_control_sdpa_scale_1p1"


def set_text_attention_control(model) -> None:
    """The language model on :func:`_perturbed_sdpa` (vision stays on SDPA)."""
    from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    if PERTURBED_KEY not in ALL_ATTENTION_FUNCTIONS:
        ALL_ATTENTION_FUNCTIONS.register(PERTURBED_KEY, _perturbed_sdpa)
    if PERTURBED_KEY not in ALL_MASK_ATTENTION_FUNCTIONS:
        ALL_MASK_ATTENTION_FUNCTIONS.register(PERTURBED_KEY, ALL_MASK_ATTENTION_FUNCTIONS["sdpa"])
    set_attention(model, "sdpa")
    model.config.text_config._attn_implementation = PERTURBED_KEY
    model.model.language_model.config._attn_implementation = PERTURBED_KEY


def token_match(a: torch.Tensor, b: torch.Tensor) -> float:
    """Fraction of positions (over the batch) before each row's first
    disagreement."""
    n = min(a.shape[1], b.shape[1])
    same = (a[:, :n] == b[:, :n]).to(torch.int32)
    prefix = torch.cumprod(same, dim=1).sum(dim=1)
    return float(prefix.sum()) / float(a.shape[0] * n) if n else 1.0


@torch.no_grad()
def graph_generate(model, inputs: dict, max_new_tokens: int, timed: bool = True) -> GenerateRun:
    """The same greedy generation with :class:`GraphGreedyDecoder`; TTFT is a
    one-token run (the prefill)."""
    from .decode_graph import GraphGreedyDecoder

    dec = GraphGreedyDecoder(model)
    device = inputs["input_ids"].device
    ttft = float("nan")
    if timed:
        _sync(device)
        t0 = time.perf_counter()
        dec.generate(inputs, 1)
        _sync(device)
        ttft = time.perf_counter() - t0
    _sync(device)
    t0 = time.perf_counter()
    tokens = dec.generate(inputs, max_new_tokens)
    _sync(device)
    return GenerateRun(tokens=tokens, seconds=time.perf_counter() - t0, ttft_seconds=ttft, step_ms=dec.last_step_ms)


@torch.no_grad()
def teacher_forced_gap(model, inputs: dict, tokens: torch.Tensor) -> torch.Tensor:
    """[B, new] gaps: the model's best logit minus its logit for ``tokens``, at
    each generated position, with ``tokens`` fed back as the continuation."""
    ids = torch.cat([inputs["input_ids"], tokens], dim=1)
    n_new = tokens.shape[1]
    full = dict(inputs)
    full["input_ids"] = ids
    full["attention_mask"] = torch.ones_like(ids)
    mm = inputs["mm_token_type_ids"]
    full["mm_token_type_ids"] = torch.cat([mm, torch.zeros(mm.shape[0], n_new, dtype=mm.dtype, device=mm.device)], 1)
    model.model.rope_deltas = None
    logits = model(**full, use_cache=False, logits_to_keep=n_new + 1).logits.float()
    pred = logits[:, :-1]  # position i predicts generated token i
    best = pred.max(dim=-1).values
    chosen = pred.gather(-1, tokens.unsqueeze(-1)).squeeze(-1)
    return best - chosen


def run_check(batch: int = 8, seq_len: int = 2048, max_new_tokens: int = 128, grid_hw=(64, 100),
              dtype: torch.dtype = torch.bfloat16, device: str | torch.device = "cuda:0", seed: int = 0,
              text: dict | None = None, vision: dict | None = None, timed: bool = True,
              with_control: bool = False) -> dict:
    """Build the model, generate greedily with SDPA and with this backend, and
    compare.  Returns the numbers the integration test and the benchmark
    report."""
    config = qwen3vl_config(text, vision)
    model = build_random_model(config, dtype, device, seed)
    inputs = synthetic_prompt(config, batch, seq_len, grid_hw, seed=seed, dtype=dtype, device=device)
    # warm-up of both paths (allocator, library load, tensor-map encoder)
    warm = {k: (v[:1] if k != "pixel_values" else v[: v.shape[0] // batch]) for k, v in inputs.items()}
    set_attention(model, "sdpa")
    greedy_generate(model, warm, 2, timed=False)
    ref = greedy_generate(model, inputs, max_new_tokens, timed)
    set_attention(model, "aicas")
    assert attention_in_use(model) == (VISION_BACKEND_KEY, TEXT_BACKEND_KEY)
    greedy_generate(model, warm, 2, timed=False)
    ours = greedy_generate(model, inputs, max_new_tokens, timed)
    graph_generate(model, warm, 3, timed=False)
    graph = graph_generate(model, inputs, max_new_tokens, timed)
    # position-wise agreement: this backend's greedy choice at every position of
    # SDPA's own greedy sequence, fed SDPA's tokens (no compounding after a near-tie)
    agree = float((forced_choices(model, inputs, ref.tokens) == ref.tokens).float().mean())
    control = None
    if with_control:
        set_text_attention_control(model)
        control = float((forced_choices(model, inputs, ref.tokens) == ref.tokens).float().mean())
    set_attention(model, "sdpa")
    gap = teacher_forced_gap(model, inputs, ours.tokens)
    gap_graph = teacher_forced_gap(model, inputs, graph.tokens)
    result = {
        "batch": batch,
        "prompt_tokens": seq_len,
        "new_tokens": max_new_tokens,
        "image_grid": list(grid_hw),
        "dtype": str(dtype).replace("torch.", ""),
        "token_match": token_match(ours.tokens, ref.tokens),
        "forced_agreement": agree,
        "control_forced_agreement": control,
        "max_logit_gap": float(gap.max()),
        "mean_logit_gap": float(gap.mean()),
        "patched": {"tokens_per_s": ours.tokens_per_s, "seconds": ours.seconds, "ttft_s": ours.ttft_seconds},
        "sdpa": {"tokens_per_s": ref.tokens_per_s, "seconds": ref.seconds, "ttft_s": ref.ttft_seconds},
        "graph_decode": {"tokens_per_s": graph.tokens_per_s, "seconds": graph.seconds, "ttft_s": graph.ttft_seconds,
                         "step_ms": graph.step_ms,
                         "token_match_vs_patched": token_match(graph.tokens, ours.tokens),
                         "max_logit_gap": float(gap_graph.max()), "mean_logit_gap": float(gap_graph.mean())},
    }
    del model
    return result
