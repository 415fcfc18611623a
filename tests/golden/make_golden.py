"""Generates the golden vectors in this directory by running the REFERENCE itself.

Run in a container that has the reference project checked out (read-only is
fine; byte-code writing is disabled):

    python tests/golden/make_golden.py --reference /path/to/AICAS

What runs, all on CPU:
  * the reference package ``triton_qwen3vl`` imported under an alias; its HF
    backends (backends.py:90-289) take their PyTorch SDPA path on CPU tensors,
    i.e. exactly the reference's own attention arithmetic;
  * ``InplaceDecodeCacheLayer`` from dujunbaoV1/evaluation_wrapper.py:54-112
    for the KV-append semantics;
  * Hugging Face's ``Qwen3VLTextRotaryEmbedding``, ``apply_rotary_pos_emb`` and
    ``Qwen3VLTextRMSNorm`` (transformers 5.5.0), the functions the reference's
    text attention is called after.

Large inputs are not stored: they are regenerated from ``aicas_b200.workloads``
seeds, and each fixture stores checksums so a test detects generator drift.
Attention references are computed on fp32 upcasts of the (16-bit) inputs:
the tolerance bar is stated against an fp32 reference.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

sys.dont_write_bytecode = True
HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from aicas_b200 import workloads as wl  # noqa: E402


def load_reference(ref_root: Path):
    spec = importlib.util.spec_from_file_location(
        "ref_triton_qwen3vl", ref_root / "triton_qwen3vl" / "__init__.py",
        submodule_search_locations=[str(ref_root / "triton_qwen3vl")],
    )
    pkg = importlib.util.module_from_spec(spec)
    sys.modules["ref_triton_qwen3vl"] = pkg
    spec.loader.exec_module(pkg)
    import ref_triton_qwen3vl.backends as backends  # noqa: E402

    spec2 = importlib.util.spec_from_file_location("ref_dujunbao_wrapper", ref_root / "dujunbaoV1" / "evaluation_wrapper.py")
    wrapper = importlib.util.module_from_spec(spec2)
    spec2.loader.exec_module(wrapper)
    return backends, wrapper


class Module(torch.nn.Module):
    def __init__(self, groups: int, scaling: float, is_causal: bool):
        super().__init__()
        self.num_key_value_groups = groups
        self.scaling = scaling
        self.is_causal = is_causal


def checksum(*tensors: torch.Tensor) -> np.ndarray:
    return np.array([float(t.double().sum()) for t in tensors] + [float(t.double().abs().sum()) for t in tensors])


def save(name: str, meta: dict, **arrays) -> None:
    path = HERE / f"{name}.npz"
    np.savez_compressed(path, meta=np.array(json.dumps(meta)), **arrays)
    print(f"wrote {path.relative_to(REPO)} ({path.stat().st_size // 1024} KiB)")


def text_ref(backends, q, k, v, groups, scale, causal=True):
    out, _ = backends.text_triton_attention(Module(groups, scale, causal), q.float(), k.float(), v.float(),
                                            attention_mask=None, dropout=0.0, scaling=None)
    return out  # [B, S, Hq, D]


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", type=Path, required=True)
    args = ap.parse_args()
    backends, wrapper = load_reference(args.reference.resolve())
    torch.set_num_threads(8)

    # -- the reference's own seeded parity cases (test/test_qwen3vl_triton_patch.py:389-491),
    #    generated on CPU (fp16 inputs) and evaluated by the reference backends in fp32
    torch.manual_seed(0)
    q = torch.randn(1, 4, 32, 64, dtype=torch.float16)
    k = torch.randn(1, 2, 32, 64, dtype=torch.float16)
    v = torch.randn(1, 2, 32, 64, dtype=torch.float16)
    out = text_ref(backends, q, k, v, 2, 64 ** -0.5)
    save("ref_prefill_seed0", {"groups": 2, "scale": 64 ** -0.5, "causal": True},
         q=q.numpy(), k=k.numpy(), v=v.numpy(), out=out.numpy())

    torch.manual_seed(1)
    q = torch.randn(1, 4, 1, 64, dtype=torch.float16)
    k = torch.randn(1, 2, 65, 64, dtype=torch.float16)
    v = torch.randn(1, 2, 65, 64, dtype=torch.float16)
    out = text_ref(backends, q, k, v, 2, 64 ** -0.5)
    save("ref_decode_seed1", {"groups": 2, "scale": 64 ** -0.5}, q=q.numpy(), k=k.numpy(), v=v.numpy(), out=out.numpy())

    torch.manual_seed(2)
    q = torch.randn(1, 2, 9, 64, dtype=torch.float16)
    k = torch.randn(1, 2, 9, 64, dtype=torch.float16)
    v = torch.randn(1, 2, 9, 64, dtype=torch.float16)
    cu = torch.tensor([0, 2, 5, 9], dtype=torch.int32)
    out, _ = backends.vision_triton_attention(Module(1, 64 ** -0.5, False), q.float(), k.float(), v.float(),
                                              attention_mask=None, cu_seq_lens_q=cu, cu_seq_lens_k=cu,
                                              max_length_q=4, max_length_k=4, is_causal=False)
    save("ref_varlen_seed2", {"scale": 64 ** -0.5}, q=q.numpy(), k=k.numpy(), v=v.numpy(), cu=cu.numpy(),
         out=out.numpy())

    # -- config 1 (fp32, CPU-runnable through the reference's PyTorch path)
    q, k, v = wl.cfg1_decode(0)
    out = text_ref(backends, q, k, v, 2, wl.SCALE_TEXT)
    save("cfg1_decode", {"seed": 0, "groups": 2, "scale": wl.SCALE_TEXT}, checksum=checksum(q, k, v), out=out.numpy())

    # -- config 2, reduced: ragged lengths including the edge lengths 1/65/127, bf16 caches
    lens = [1, 65, 127, 300]
    cap = 320
    g = wl.generator(7)
    q = wl.randn((4, wl.HQ, 1, wl.HEAD_DIM), g, torch.bfloat16)
    kc = wl.randn((4, wl.HKV, cap, wl.HEAD_DIM), g, torch.bfloat16)
    vc = wl.randn((4, wl.HKV, cap, wl.HEAD_DIM), g, torch.bfloat16)
    outs = [text_ref(backends, q[b : b + 1], kc[b : b + 1, :, :n], vc[b : b + 1, :, :n], 2, wl.SCALE_TEXT)
            for b, n in enumerate(lens)]
    save("cfg2_ragged_small", {"seed": 7, "lens": lens, "cap": cap, "groups": 2, "scale": wl.SCALE_TEXT},
         checksum=checksum(q, kc, vc), out=torch.cat(outs, 0).numpy())

    # -- config 4, reduced: causal GQA prefill with multimodal RoPE applied
    q, k, v = wl.cfg4_prefill(seed=3, batch=1, seq=160, hq=4, hkv=2)
    out = text_ref(backends, q, k, v, 2, wl.SCALE_TEXT)
    save("cfg4_prefill_small", {"seed": 3, "batch": 1, "seq": 160, "hq": 4, "hkv": 2, "groups": 2,
                                "scale": wl.SCALE_TEXT}, checksum=checksum(q, k, v), out=out.numpy())

    # -- config 3, reduced: packed ViT varlen attention
    q, k, v, cu, seg = wl.cfg3_varlen(seed=5, images=4, heads=2, lo=4, hi=16)
    out, _ = backends.vision_triton_attention(Module(1, wl.SCALE_VIT, False), q.float(), k.float(), v.float(),
                                              attention_mask=None, cu_seq_lens_q=cu, cu_seq_lens_k=cu,
                                              max_length_q=max(seg), max_length_k=max(seg), is_causal=False)
    save("cfg3_varlen_small", {"seed": 5, "images": 4, "heads": 2, "lo": 4, "hi": 16, "scale": wl.SCALE_VIT},
         checksum=checksum(q, k, v), cu=cu.numpy(), out=out.numpy())

    # -- padded text batches: the reference's masked path is sdpa_fallback
    #    (backends.py:249-260, 277-287).  Handed HF's 2-D padding mask (what its
    #    flash_attention_2 mask mapping gives it) that path raises inside SDPA, so
    #    it is run here with the 4-D mask HF builds for SDPA: key j visible to
    #    query i when j is a real token and j <= i's position.  Rows at padded
    #    query positions are stored but not compared (HF discards them).
    B, S, hq, hkv, D = 3, 40, 4, 2, 128
    g = wl.generator(13)
    mask2d = torch.ones(B, S + 1, dtype=torch.bool)
    mask2d[1, :7] = False   # left padding
    mask2d[2, :33] = False  # left padding, 7 real prompt tokens
    q = wl.randn((B, hq, S, D), g, torch.bfloat16)
    k = wl.randn((B, hkv, S + 1, D), g, torch.bfloat16)
    v = wl.randn((B, hkv, S + 1, D), g, torch.bfloat16)
    qd = wl.randn((B, hq, 1, D), g, torch.bfloat16)

    def four_d(m2, sq, skv):
        pos = torch.arange(sq) + (skv - sq)
        return m2[:, None, None, :skv] & (torch.arange(skv)[None, None, None, :] <= pos[None, None, :, None])

    def masked_ref(qq, kk, vv, m4):
        out, _ = backends.text_triton_attention(Module(2, D ** -0.5, True), qq.float(), kk.float(), vv.float(),
                                                attention_mask=m4, dropout=0.0, scaling=None)
        return out.nan_to_num(0.0)

    pre = masked_ref(q, k[:, :, :S], v[:, :, :S], four_d(mask2d[:, :S], S, S))
    dec = masked_ref(qd, k, v, four_d(mask2d, 1, S + 1))
    save("padded_text", {"seed": 13, "groups": 2, "scale": D ** -0.5, "seq": S},
         mask=mask2d.numpy(), q=q.float().numpy(), k=k.float().numpy(), v=v.float().numpy(), q_dec=qd.float().numpy(),
         out_prefill=pre.numpy(), out_decode=dec.numpy())

    # -- text RoPE (+ per-head RMSNorm) exactly as Qwen3VLTextAttention runs it before the backend
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLTextConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import (
        Qwen3VLTextRMSNorm, Qwen3VLTextRotaryEmbedding, apply_rotary_pos_emb)

    cfg = Qwen3VLTextConfig(head_dim=128, hidden_size=2048, num_attention_heads=16, num_key_value_heads=8,
                            rope_parameters={"rope_type": "default", "rope_theta": wl.ROPE_THETA,
                                             "mrope_section": list(wl.MROPE_SECTION), "mrope_interleaved": True})
    rot = Qwen3VLTextRotaryEmbedding(cfg)
    g = wl.generator(11)
    B, S = 2, 8
    qx = wl.randn((B, 4, S, 128), g, torch.bfloat16)
    kx = wl.randn((B, 2, S, 128), g, torch.bfloat16)
    ids = wl.mixed_prompt_position_ids(B, S, text_before=2, grid=(2, 2))
    ids[:, 1] += 37  # second request at other positions
    cos, sin = rot(qx, ids)
    q_rot, k_rot = apply_rotary_pos_emb(qx, kx, cos, sin)
    qn = Qwen3VLTextRMSNorm(128, eps=1e-6)
    kn = Qwen3VLTextRMSNorm(128, eps=1e-6)
    with torch.no_grad():
        qn.weight.copy_(1.0 + 0.1 * wl.randn((128,), g))
        kn.weight.copy_(1.0 + 0.1 * wl.randn((128,), g))
        qn, kn = qn.to(torch.bfloat16), kn.to(torch.bfloat16)
        qnr, knr = apply_rotary_pos_emb(qn(qx), kn(kx), cos, sin)
    f = lambda t: t.float().numpy()  # noqa: E731  (bf16 values are exact in fp32)
    save("rope_hf", {"theta": wl.ROPE_THETA, "mrope_section": list(wl.MROPE_SECTION), "eps": 1e-6},
         position_ids=ids.numpy(), q=f(qx), k=f(kx), cos=f(cos), sin=f(sin), q_rot=f(q_rot), k_rot=f(k_rot),
         q_norm_w=f(qn.weight.detach()), k_norm_w=f(kn.weight.detach()), q_norm_rot=f(qnr), k_norm_rot=f(knr))

    # -- KV append: InplaceDecodeCacheLayer.update, 5 tokens, then 1, then 12 (truncated at 16)
    layer = wrapper.InplaceDecodeCacheLayer(max_cache_len=16)
    steps = []
    for n in (5, 1, 12):
        kn_ = wl.randn((2, 2, n, 128), g, torch.bfloat16)
        vn_ = wl.randn((2, 2, n, 128), g, torch.bfloat16)
        start = layer.get_seq_length()
        kk, vv = layer.update(kn_, vn_)
        steps.append({"start": start, "n": n, "k_new": f(kn_), "v_new": f(vn_), "k_cache": f(layer.keys),
                      "v_cache": f(layer.values), "visible": int(kk.shape[2])})
    arrays = {}
    for i, st in enumerate(steps):
        for key in ("k_new", "v_new", "k_cache", "v_cache"):
            arrays[f"s{i}_{key}"] = st[key]
    save("cache_append", {"max_cache_len": 16, "steps": [{"start": s["start"], "n": s["n"], "visible": s["visible"]}
                                                         for s in steps]}, **arrays)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
