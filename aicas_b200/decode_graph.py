"""Preallocated KV cache for Hugging Face Qwen3-VL and a CUDA-graph greedy
decode step for the language model.

The semantics follow the reference's in-place cache layer and graph runner
(dujunbaoV1/evaluation_wrapper.py:54-112 ``InplaceDecodeCacheLayer``,
:210-391 ``CUDAGraphDecodeRunner``): the cache is allocated once at a fixed
capacity and appended in place (``DynamicCache`` re-allocates it with
``torch.cat`` every token, HF cache_utils.py:119-120), and one decode step of
the language model is captured in a CUDA graph and replayed.  What this
version does differently:

* the step runs the fused RoPE + q/k RMSNorm + cache append kernel
  (:func:`aicas_b200.ops.rope_kv_append`) and the split-KV decode kernel,
  which reads the cache lengths from a device vector, so the graph holds no
  per-step host value;
* every product of the step (q/k/v, o_proj, gate/up, down_proj, LM head) runs
  on :func:`aicas_b200.ops.decode_linear` with the RMSNorms, the residual adds
  and SiLU * up fused into it, as the reference's native decode ops fuse them
  (dujunbaoV1/native_cuda_ops/decode_q1_gqa_kernel.cu:127-331), for batches
  of up to 32 rows;
* the step advances its own state on the device -- cache lengths, MRoPE
  position ids, the next token (argmax of the logits) and the token log -- so
  N new tokens are one prefill and N - 1 graph replays with no host work or
  synchronisation between them;
* any batch size (the reference runner is batch 1), unpadded prompts.

Greedy only (the organiser harness generates with ``do_sample=False``,
evaluation_wrapper.py:509-516).
"""
from __future__ import annotations

import torch
from transformers.cache_utils import Cache, CacheLayerMixin

from . import _native as nat
from . import ops


class StaticKVLayer(CacheLayerMixin):
    """One decoder layer's cache: ``[B, Hkv, capacity, D]`` keys and values,
    written in place; ``update`` returns views of the valid prefix."""

    is_compileable = False
    is_sliding = False

    def __init__(self, capacity: int):
        super().__init__()
        if capacity < 1:
            raise ValueError("capacity must be positive")
        self.capacity = capacity
        self.length = 0

    def lazy_initialization(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        B, H, _, D = key_states.shape
        self.keys = torch.zeros((B, H, self.capacity, D), dtype=key_states.dtype, device=key_states.device)
        self.values = torch.zeros((B, H, self.capacity, value_states.shape[-1]), dtype=value_states.dtype,
                                  device=value_states.device)
        self.dtype, self.device = key_states.dtype, key_states.device
        self.is_initialized = True

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        n = key_states.shape[-2]
        start, end = self.length, self.length + n
        if end > self.capacity:
            raise ValueError(f"KV cache capacity {self.capacity} exceeded ({end} tokens)")
        self.keys[:, :, start:end].copy_(key_states)
        self.values[:, :, start:end].copy_(value_states)
        self.length = end
        return self.keys[:, :, :end], self.values[:, :, :end]

    def get_mask_sizes(self, query_length: int) -> tuple[int, int]:
        return self.length + query_length, 0

    def get_seq_length(self) -> int:
        return self.length

    def get_max_cache_shape(self) -> int:
        return self.capacity

    def reset(self) -> None:
        super().reset()
        self.length = 0


class StaticKVCache(Cache):
    """A :class:`transformers.cache_utils.Cache` of :class:`StaticKVLayer`s."""

    def __init__(self, num_layers: int, capacity: int):
        super().__init__(layers=[StaticKVLayer(capacity) for _ in range(num_layers)])


class GraphGreedyDecoder:
    """Greedy generation for a Qwen3-VL model whose attention is this backend:
    prefill through the model's own forward (vision tower, MRoPE, deepstack,
    the patched attention) into a :class:`StaticKVCache`, then the decode steps
    from one captured CUDA graph.

    ``model`` is a ``Qwen3VLForConditionalGeneration`` in eval mode on one GPU
    with 16-bit weights."""

    def __init__(self, model, fused: bool = True):
        self.model = model
        self.fused = fused
        self.lm = model.model.language_model
        self.lm_head = model.lm_head
        attn = self.lm.layers[0].self_attn
        self.hq = model.config.text_config.num_attention_heads
        self.hkv = model.config.text_config.num_key_value_heads
        self.head_dim = attn.head_dim
        self.group = attn.num_key_value_groups
        self.last_graph_replays = 0
        self.last_step_ms = float("nan")

    def _step(self, st: dict) -> None:
        """One decode token for the whole batch, all state on the device."""
        if self.fused and st["tok"].shape[0] <= nat.LINEAR_MAX_ROWS:
            self._step_fused(st)
        else:
            self._step_modules(st)

    def _step_fused(self, st: dict) -> None:
        """The step with every product on :func:`aicas_b200.ops.decode_linear`:
        per layer, q/k/v, the fused q/k norm + RoPE + append, decode attention,
        o_proj + residual, gate/up + SiLU*up, down_proj + residual; then the LM
        head.  Each residual product also writes the sums of squares of the
        residual stream's rows (``sumsq_out``), so the following product
        normalises its input from those statistics (``x_sumsq``) without a pass
        over x; only layer 0 computes them from the embedding itself."""
        B, D = st["tok"].shape[0], self.head_dim
        x = self.lm.embed_tokens(st["tok"]).view(B, -1)
        ss = torch.empty(B, dtype=torch.float32, device=x.device)  # row sums of squares of x
        cos, sin = self.lm.rotary_emb(x.view(B, 1, -1), st["pos"])
        layers = self.lm.layers
        for i, layer in enumerate(layers):
            attn, mlp = layer.self_attn, layer.mlp
            ln1, ln2 = layer.input_layernorm, layer.post_attention_layernorm
            q, k, v = ops.decode_linear(x, (attn.q_proj.weight, attn.k_proj.weight, attn.v_proj.weight),
                                        norm_weight=ln1.weight, eps=ln1.variance_epsilon,
                                        x_sumsq=ss if i > 0 else None)
            kc, vc = st["caches"][i]
            qr = ops.rope_kv_append(q.view(B, 1, self.hq, D).transpose(1, 2), k.view(B, 1, self.hkv, D).transpose(1, 2),
                                    v.view(B, 1, self.hkv, D).transpose(1, 2), cos, sin, kc, vc, st["lens"],
                                    kv_lens_out=st["lens_next"], q_norm_weight=attn.q_norm.weight,
                                    k_norm_weight=attn.k_norm.weight, eps=attn.q_norm.variance_epsilon)
            o = ops.gqa_decode_attention(qr, kc, vc, sm_scale=attn.scaling, num_key_value_groups=self.group,
                                         kv_lens=st["lens_next"])
            ops.decode_linear(o.reshape(B, self.hq * D), attn.o_proj.weight, residual=x, out=x, sumsq_out=ss)
            h = ops.decode_linear(x, (mlp.gate_proj.weight, mlp.up_proj.weight), norm_weight=ln2.weight,
                                  eps=ln2.variance_epsilon, x_sumsq=ss, swiglu=True)
            ops.decode_linear(h, mlp.down_proj.weight, residual=x, out=x, sumsq_out=ss)
        logits = ops.decode_linear(x, self.lm_head.weight, norm_weight=self.lm.norm.weight,
                                   eps=self.lm.norm.variance_epsilon, x_sumsq=ss)
        self._advance(st, logits)

    def _step_modules(self, st: dict) -> None:
        """The step through the model's own modules (any batch size)."""
        B, D = st["tok"].shape[0], self.head_dim
        x = self.lm.embed_tokens(st["tok"])
        cos, sin = self.lm.rotary_emb(x, st["pos"])
        for i, layer in enumerate(self.lm.layers):
            attn = layer.self_attn
            h = layer.input_layernorm(x)
            q = attn.q_proj(h).view(B, 1, self.hq, D).transpose(1, 2)
            k = attn.k_proj(h).view(B, 1, self.hkv, D).transpose(1, 2)
            v = attn.v_proj(h).view(B, 1, self.hkv, D).transpose(1, 2)
            kc, vc = st["caches"][i]
            qr = ops.rope_kv_append(q, k, v, cos, sin, kc, vc, st["lens"], kv_lens_out=st["lens_next"],
                                    q_norm_weight=attn.q_norm.weight, k_norm_weight=attn.k_norm.weight,
                                    eps=attn.q_norm.variance_epsilon)
            o = ops.gqa_decode_attention(qr, kc, vc, sm_scale=attn.scaling, num_key_value_groups=self.group,
                                         kv_lens=st["lens_next"])
            x = x + attn.o_proj(o.transpose(1, 2).reshape(B, 1, self.hq * D))
            x = x + layer.mlp(layer.post_attention_layernorm(x))
        logits = self.lm_head(self.lm.norm(x)[:, -1])
        self._advance(st, logits)

    @staticmethod
    def _advance(st: dict, logits: torch.Tensor) -> None:
        B = st["tok"].shape[0]
        nxt = logits.argmax(-1).view(B, 1)
        st["tok"].copy_(nxt)
        st["step"].add_(1)
        st["log"].index_copy_(1, st["step"], nxt)
        st["lens"].copy_(st["lens_next"])
        st["pos"].add_(1)

    @torch.no_grad()
    def generate(self, inputs: dict, max_new_tokens: int) -> torch.Tensor:
        """``[B, max_new_tokens]`` greedy tokens after the prompts in ``inputs``
        (the processor's dict: input_ids, attention_mask of ones,
        mm_token_type_ids, pixel_values, image_grid_thw).  Afterwards
        ``last_step_ms`` holds the mean device time of one replayed decode step
        (CUDA events around the replays)."""
        graph, st = self.prefill_and_capture(inputs, max_new_tokens)
        if graph is None:
            return st["log"]
        device = st["log"].device
        stream = torch.cuda.current_stream(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(max_new_tokens - 1):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize(device)
        self.last_graph_replays = max_new_tokens - 1
        self.last_step_ms = e0.elapsed_time(e1) / (max_new_tokens - 1)
        result = st["log"].clone()
        del graph
        return result

    @torch.no_grad()
    def prefill_and_capture(self, inputs: dict, max_new_tokens: int):
        """Runs the prefill and captures the decode step: ``(graph, state)``,
        the graph ``None`` when one token was asked for.  Each replay of the
        graph appends one token to ``state["log"]``; at most
        ``max_new_tokens - 1`` replays fit the cache."""
        if max_new_tokens < 1:
            raise ValueError("max_new_tokens must be at least 1")
        ids = inputs["input_ids"]
        B, S = ids.shape
        am = inputs.get("attention_mask")
        if am is not None and not bool(am.all()):
            raise ValueError("padded prompts are not supported (every prompt must fill the batch row)")
        device = ids.device
        cache = StaticKVCache(len(self.lm.layers), S + max_new_tokens)
        self.model.model.rope_deltas = None
        out = self.model(**inputs, past_key_values=cache, use_cache=True, logits_to_keep=1)
        first = out.logits[:, -1].argmax(-1)
        log = torch.zeros(B, max_new_tokens, dtype=torch.long, device=device)
        log[:, 0] = first
        if max_new_tokens == 1:
            return None, {"log": log}
        deltas = self.model.model.rope_deltas.to(device=device, dtype=torch.long).view(B)
        st = {
            "tok": first.view(B, 1).clone(),
            # MRoPE position ids of the next token: text position S plus the
            # prompt's rope delta, the same on the t/h/w axes during decode
            "pos": (S + deltas).view(1, B, 1).expand(3, B, 1).contiguous(),
            "lens": torch.full((B,), S, dtype=torch.int32, device=device),
            "lens_next": torch.empty(B, dtype=torch.int32, device=device),
            "step": torch.zeros(1, dtype=torch.long, device=device),
            "log": log,
            "caches": [(layer.keys, layer.values) for layer in cache.layers],
        }
        # warm-up run of the step on the capture stream (allocations, library
        # set-up, the decode workspace of that stream), then the state is put
        # back and the step captured
        saved = {k: st[k].clone() for k in ("tok", "pos", "lens", "step", "log")}
        saved_kv = [(kc[:, :, S].clone(), vc[:, :, S].clone()) for kc, vc in st["caches"]]
        stream = torch.cuda.Stream(device)
        stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(stream):
            self._step(st)
        torch.cuda.current_stream(device).wait_stream(stream)
        for k, v in saved.items():
            st[k].copy_(v)
        for (kc, vc), (k0, v0) in zip(st["caches"], saved_kv):
            kc[:, :, S].copy_(k0)
            vc[:, :, S].copy_(v0)
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            self._step(st)
        return graph, st
