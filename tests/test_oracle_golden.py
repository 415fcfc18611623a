"""Pins the CPU oracle against the golden vectors produced by running the
reference itself (tests/golden/make_golden.py).  CPU only."""
from __future__ import annotations

import numpy as np
import torch

from aicas_b200 import workloads as wl
from oracle import attention as oa
from oracle import cache as oc
from oracle import rope as orope
from tests.conftest import checksum, load_golden

TIGHT = dict(rtol=0, atol=2e-6)


def test_reference_prefill_seed0():
    meta, a = load_golden("ref_prefill_seed0")
    out = oa.sdpa(a["q"], a["k"], a["v"], meta["scale"], True, meta["groups"])
    np.testing.assert_allclose(out.transpose(0, 2, 1, 3), a["out"], **TIGHT)


def test_reference_decode_seed1_odd_length():
    meta, a = load_golden("ref_decode_seed1")
    assert a["k"].shape[2] == 65
    out = oa.sdpa(a["q"], a["k"], a["v"], meta["scale"], False, meta["groups"])
    np.testing.assert_allclose(out.transpose(0, 2, 1, 3), a["out"], **TIGHT)


def test_reference_varlen_seed2():
    meta, a = load_golden("ref_varlen_seed2")
    out = oa.varlen(a["q"], a["k"], a["v"], a["cu"], a["cu"], meta["scale"])
    np.testing.assert_allclose(out.transpose(0, 2, 1, 3), a["out"], **TIGHT)


def test_cfg1_decode_fp32():
    meta, a = load_golden("cfg1_decode")
    q, k, v = wl.cfg1_decode(meta["seed"])
    np.testing.assert_allclose(checksum(q, k, v), a["checksum"], rtol=1e-12)
    out = oa.sdpa(q.numpy(), k.numpy(), v.numpy(), meta["scale"], False, meta["groups"])
    np.testing.assert_allclose(out.transpose(0, 2, 1, 3), a["out"], **TIGHT)


def test_cfg2_ragged_lengths():
    meta, a = load_golden("cfg2_ragged_small")
    g = wl.generator(meta["seed"])
    q = wl.randn((4, wl.HQ, 1, wl.HEAD_DIM), g, torch.bfloat16)
    kc = wl.randn((4, wl.HKV, meta["cap"], wl.HEAD_DIM), g, torch.bfloat16)
    vc = wl.randn((4, wl.HKV, meta["cap"], wl.HEAD_DIM), g, torch.bfloat16)
    np.testing.assert_allclose(checksum(q, kc, vc), a["checksum"], rtol=1e-12)
    out = oa.decode_ragged(q.float().numpy(), kc.float().numpy(), vc.float().numpy(), meta["lens"], meta["scale"], 2)
    np.testing.assert_allclose(out.transpose(0, 2, 1, 3), a["out"], **TIGHT)


def test_cfg4_prefill_with_mrope():
    meta, a = load_golden("cfg4_prefill_small")
    q, k, v = wl.cfg4_prefill(seed=meta["seed"], batch=meta["batch"], seq=meta["seq"], hq=meta["hq"], hkv=meta["hkv"])
    np.testing.assert_allclose(checksum(q, k, v), a["checksum"], rtol=1e-12)
    out = oa.sdpa(q.float().numpy(), k.float().numpy(), v.float().numpy(), meta["scale"], True, meta["groups"])
    np.testing.assert_allclose(out.transpose(0, 2, 1, 3), a["out"], **TIGHT)


def test_cfg3_varlen():
    meta, a = load_golden("cfg3_varlen_small")
    q, k, v, cu, _ = wl.cfg3_varlen(seed=meta["seed"], images=meta["images"], heads=meta["heads"],
                                    lo=meta["lo"], hi=meta["hi"])
    np.testing.assert_allclose(checksum(q, k, v), a["checksum"], rtol=1e-12)
    np.testing.assert_array_equal(cu.numpy(), a["cu"])
    out = oa.varlen(q.float().numpy(), k.float().numpy(), v.float().numpy(), a["cu"], a["cu"], meta["scale"])
    np.testing.assert_allclose(out.transpose(0, 2, 1, 3), a["out"], **TIGHT)


def test_rope_bit_exact_against_hf():
    meta, a = load_golden("rope_hf")
    np.testing.assert_array_equal(orope.apply_rope(a["q"], a["cos"], a["sin"], "bf16"), a["q_rot"])
    np.testing.assert_array_equal(orope.apply_rope(a["k"], a["cos"], a["sin"], "bf16"), a["k_rot"])


def test_mrope_tables_match_hf():
    meta, a = load_golden("rope_hf")
    cos, sin = orope.mrope_cos_sin(a["position_ids"], 128, meta["theta"], meta["mrope_section"], "bf16")
    # cos/sin of float32 arguments may differ by an ulp between libm implementations
    np.testing.assert_allclose(cos, a["cos"], rtol=0, atol=2 ** -8)
    np.testing.assert_allclose(sin, a["sin"], rtol=0, atol=2 ** -8)
    assert (cos == a["cos"]).mean() > 0.99 and (sin == a["sin"]).mean() > 0.99


def test_workload_mrope_tables_match_hf():
    meta, a = load_golden("rope_hf")
    cos, sin = wl.mrope_cos_sin(torch.from_numpy(a["position_ids"]), torch.bfloat16)
    np.testing.assert_array_equal(cos.float().numpy(), a["cos"])
    np.testing.assert_array_equal(sin.float().numpy(), a["sin"])


def test_rms_norm_then_rope_against_hf():
    meta, a = load_golden("rope_hf")
    qn = orope.rms_norm_heads(a["q"], a["q_norm_w"], meta["eps"], "bf16")
    kn = orope.rms_norm_heads(a["k"], a["k_norm_w"], meta["eps"], "bf16")
    q = orope.apply_rope(qn, a["cos"], a["sin"], "bf16")
    k = orope.apply_rope(kn, a["cos"], a["sin"], "bf16")
    # the fp32 sum of squares may round differently from torch's reduction order
    for got, ref in ((q, a["q_norm_rot"]), (k, a["k_norm_rot"])):
        assert np.abs(got - ref).max() <= 2 ** -6 * max(1.0, np.abs(ref).max())
        assert (got == ref).mean() > 0.98


def test_kv_append_matches_inplace_cache_layer():
    meta, a = load_golden("cache_append")
    cap = meta["max_cache_len"]
    kc = np.zeros_like(a["s0_k_cache"])
    vc = np.zeros_like(a["s0_v_cache"])
    for i, st in enumerate(meta["steps"]):
        positions = [st["start"]] * kc.shape[0]
        kc, vc, lens = oc.kv_append(kc, vc, a[f"s{i}_k_new"], a[f"s{i}_v_new"], positions)
        np.testing.assert_array_equal(kc, a[f"s{i}_k_cache"])
        np.testing.assert_array_equal(vc, a[f"s{i}_v_cache"])
        assert (lens == st["visible"]).all() and st["visible"] <= cap


def test_merge_of_sharded_partials_equals_full():
    q, k, v = wl.cfg1_decode(0)
    full = oa.sdpa(q.numpy(), k.numpy(), v.numpy(), wl.SCALE_TEXT, False, 2)[:, :, 0]
    for shards in (2, 4, 8):
        po, pl = oa.sharded_decode_partials(q.numpy(), k.numpy(), v.numpy(), wl.SCALE_TEXT, 2, shards)
        np.testing.assert_allclose(oa.merge(po, pl), full, rtol=0, atol=1e-12)
    lse = oa.lse_base2(q.numpy(), k.numpy(), wl.SCALE_TEXT, 2)
    po, pl = oa.sharded_decode_partials(q.numpy(), k.numpy(), v.numpy(), wl.SCALE_TEXT, 2, 4)
    m = pl.max(0)
    np.testing.assert_allclose(m + np.log2(np.exp2(pl - m).sum(0)), lse, rtol=0, atol=1e-10)


def test_decode_linear_oracle_against_hf_modules():
    """oracle.decode_linear restates Qwen3VLTextRMSNorm and Qwen3VLTextMLP:
    same values as the HF modules run in bf16 on CPU (the norm's fp32 reduction
    order and the CPU GEMM's accumulation may move a value by one unit in the
    last place)."""
    import torch
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLTextConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLTextMLP, Qwen3VLTextRMSNorm

    from oracle import decode_linear as odl

    g = torch.Generator().manual_seed(5)
    R, K, N = 6, 256, 384
    x = torch.randn(R, K, generator=g).to(torch.bfloat16)
    norm = Qwen3VLTextRMSNorm(K, eps=1e-6).to(torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_((1 + 0.1 * torch.randn(K, generator=g)).to(torch.bfloat16))
        hf_norm = norm(x).float().numpy()
    f32 = lambda t: t.float().numpy()  # noqa: E731
    ours = odl.rms_norm_rows(f32(x), f32(norm.weight.detach()), 1e-6, "bf16")
    assert (ours == hf_norm).mean() > 0.99
    assert np.abs(ours - hf_norm).max() <= 2 ** -7 * np.abs(hf_norm).max()

    cfg = Qwen3VLTextConfig(hidden_size=K, intermediate_size=N, hidden_act="silu")
    mlp = Qwen3VLTextMLP(cfg).to(torch.bfloat16)
    with torch.no_grad():
        for lin in (mlp.gate_proj, mlp.up_proj):
            lin.weight.copy_((torch.randn(N, K, generator=g) / K ** 0.5).to(torch.bfloat16))
        xn = norm(x)
        hf_h = mlp.act_fn(mlp.gate_proj(xn)) * mlp.up_proj(xn)
    (h,) = odl.decode_linear(f32(x), [f32(mlp.gate_proj.weight.detach()), f32(mlp.up_proj.weight.detach())],
                             norm_weight=f32(norm.weight.detach()), eps=1e-6, swiglu=True)
    from oracle.rope import round_to

    h = round_to(h.astype(np.float32), "bf16")
    hf_h = hf_h.float().numpy()
    assert np.abs(h - hf_h).max() <= 2 ** -6 * np.abs(hf_h).max()
    assert (h == hf_h).mean() > 0.9


def test_vision_rope_oracle_bit_exact_against_hf():
    """oracle.rope.apply_rope_vision restates apply_rotary_pos_emb_vision: the
    same bits as HF's function on CPU (bf16 q/k, fp32 cos/sin)."""
    import torch
    from transformers.models.qwen3_vl.modeling_qwen3_vl import apply_rotary_pos_emb_vision

    g = torch.Generator().manual_seed(11)
    T, H, D = 37, 4, 64
    q = torch.randn(T, H, D, generator=g).to(torch.bfloat16)
    k = torch.randn(T, H, D, generator=g).to(torch.bfloat16)
    freqs = torch.randn(T, D // 2, generator=g) * 3
    emb = torch.cat((freqs, freqs), dim=-1)
    cos, sin = emb.cos(), emb.sin()
    hq, hk = apply_rotary_pos_emb_vision(q, k, cos, sin)
    for x, ref in ((q, hq), (k, hk)):
        ours = orope.apply_rope_vision(x.float().numpy(), cos.numpy(), sin.numpy(), "bf16")
        assert np.array_equal(ours, ref.float().numpy())


def test_padded_text_oracle_against_the_reference_sdpa_path():
    """oracle.sdpa_padded restates the reference's masked path (HF SDPA with the
    4-D padding + causal mask); pinned on the rows HF uses (real query tokens)."""
    meta, a = load_golden("padded_text")
    S, mask = meta["seq"], a["mask"]
    pre, real = oa.sdpa_padded(a["q"], a["k"][:, :, :S], a["v"][:, :, :S], mask[:, :S], meta["scale"], meta["groups"])
    ref = a["out_prefill"].transpose(0, 2, 1, 3)  # the backend returns [B, S, H, D]
    rows = real[:, None, :, None] & np.ones_like(pre, dtype=bool)
    np.testing.assert_allclose(pre[rows], ref[rows], rtol=0, atol=2e-6)
    assert not real.all() and real.any()
    dec, real_d = oa.sdpa_padded(a["q_dec"], a["k"], a["v"], mask, meta["scale"], meta["groups"])
    assert real_d.all()
    np.testing.assert_allclose(dec, a["out_decode"].transpose(0, 2, 1, 3), rtol=0, atol=2e-6)
