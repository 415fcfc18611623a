"""GPU parity of the fused RoPE + KV-append kernel: bit-exact against Hugging
Face's apply_rotary_pos_emb and the reference's InplaceDecodeCacheLayer."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import aicas_b200 as ab
from aicas_b200 import workloads as wl
from oracle import cache as oc
from oracle import rope as orope
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().float().cpu().numpy()


def test_rope_and_append_bit_exact_against_hf(cuda_device):
    meta, a = load_golden("rope_hf")
    dev = cuda_device
    q = torch.from_numpy(a["q"]).to(dev, torch.bfloat16)
    k = torch.from_numpy(a["k"]).to(dev, torch.bfloat16)
    B, Hkv, S, D = k.shape
    v = torch.randn(B, Hkv, S, D, device=dev).to(torch.bfloat16)
    cos = torch.from_numpy(a["cos"]).to(dev, torch.bfloat16)
    sin = torch.from_numpy(a["sin"]).to(dev, torch.bfloat16)
    cap = 40
    kc = torch.zeros(B, Hkv, cap, D, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    positions = torch.tensor([3, 17], dtype=torch.int32, device=dev)
    lens = torch.empty(B, dtype=torch.int32, device=dev)
    q_rot = ab.rope_kv_append(q, k, v, cos, sin, kc, vc, positions, kv_lens_out=lens)
    np.testing.assert_array_equal(_np(q_rot), a["q_rot"])
    for b, p in enumerate([3, 17]):
        np.testing.assert_array_equal(_np(kc[b, :, p:p + S]), a["k_rot"][b])
        assert torch.equal(vc[b, :, p:p + S], v[b])
        assert torch.all(kc[b, :, :p] == 0) and torch.all(kc[b, :, p + S:] == 0)
    assert lens.tolist() == [3 + S, 17 + S]


def test_fused_rms_norm_rope_against_hf(cuda_device):
    meta, a = load_golden("rope_hf")
    dev = cuda_device
    q = torch.from_numpy(a["q"]).to(dev, torch.bfloat16)
    k = torch.from_numpy(a["k"]).to(dev, torch.bfloat16)
    B, Hkv, S, D = k.shape
    cos = torch.from_numpy(a["cos"]).to(dev, torch.bfloat16)
    sin = torch.from_numpy(a["sin"]).to(dev, torch.bfloat16)
    qw = torch.from_numpy(a["q_norm_w"]).to(dev, torch.bfloat16)
    kw = torch.from_numpy(a["k_norm_w"]).to(dev, torch.bfloat16)
    kc = torch.zeros(B, Hkv, S, D, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    pos = torch.zeros(B, dtype=torch.int32, device=dev)
    q_rot = ab.rope_kv_append(q, k, k, cos, sin, kc, vc, pos, q_norm_weight=qw, k_norm_weight=kw, eps=meta["eps"])
    for got, ref in ((_np(q_rot), a["q_norm_rot"]), (_np(kc), a["k_norm_rot"])):
        # rsqrt and the sum-of-squares order may move a value by one bf16 ulp
        assert np.abs(got - ref).max() <= 2 ** -6 * max(1.0, np.abs(ref).max())
        assert (got == ref).mean() > 0.98


def test_append_sequence_matches_inplace_cache_layer(cuda_device):
    """5, 1 then 12 tokens into a 16-slot cache: identical caches and lengths,
    including the truncated tail of the last payload."""
    meta, a = load_golden("cache_append")
    dev = cuda_device
    B, H, _, D = a["s0_k_new"].shape
    cap = meta["max_cache_len"]
    kc = torch.zeros(B, H, cap, D, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    for i, st in enumerate(meta["steps"]):
        kn = torch.from_numpy(a[f"s{i}_k_new"]).to(dev, torch.bfloat16)
        vn = torch.from_numpy(a[f"s{i}_v_new"]).to(dev, torch.bfloat16)
        n = kn.shape[2]
        # identity rotation (cos = 1, sin = 0) turns the kernel into a pure append
        cos = torch.ones(B, n, D, dtype=torch.bfloat16, device=dev)
        sin = torch.zeros_like(cos)
        q = torch.zeros(B, 1, n, D, dtype=torch.bfloat16, device=dev)
        pos = torch.full((B,), st["start"], dtype=torch.int32, device=dev)
        lens = torch.empty(B, dtype=torch.int32, device=dev)
        ab.rope_kv_append(q, kn, vn, cos, sin, kc, vc, pos, kv_lens_out=lens)
        np.testing.assert_array_equal(_np(kc), a[f"s{i}_k_cache"])
        np.testing.assert_array_equal(_np(vc), a[f"s{i}_v_cache"])
        assert lens.tolist() == [st["visible"]] * B


@pytest.mark.parametrize("dtype,name", [(torch.float16, "fp16"), (torch.float32, "fp32"), (torch.bfloat16, "bf16")])
def test_decode_step_rope_append_against_oracle(cuda_device, dtype, name):
    """Config-2 style step: ragged positions, one new token per request."""
    dev = cuda_device
    lens = torch.tensor([0, 5, 255, 4094], dtype=torch.int32)
    st = wl.cfg2_step_inputs(lens, layer=3, dtype=dtype, device=dev)
    cap = 4096
    kc = torch.zeros(4, wl.HKV, cap, wl.HEAD_DIM, dtype=dtype, device=dev)
    vc = torch.zeros_like(kc)
    out_lens = torch.empty(4, dtype=torch.int32, device=dev)
    q_rot = ab.rope_kv_append(st.q, st.k, st.v, st.cos, st.sin, kc, vc, st.positions, kv_lens_out=out_lens)
    ref_q = orope.apply_rope(_np(st.q), _np(st.cos), _np(st.sin), name)
    ref_k = orope.apply_rope(_np(st.k), _np(st.cos), _np(st.sin), name)
    np.testing.assert_array_equal(_np(q_rot), ref_q)
    kc_ref, vc_ref, lens_ref = oc.kv_append(np.zeros(kc.shape, np.float32), np.zeros(vc.shape, np.float32), ref_k,
                                            _np(st.v), lens.tolist())
    np.testing.assert_array_equal(_np(kc), kc_ref)
    np.testing.assert_array_equal(_np(vc), vc_ref)
    assert out_lens.cpu().numpy().tolist() == lens_ref.tolist()


def test_positions_past_capacity_are_dropped(cuda_device):
    dev = cuda_device
    B, H, S, D, cap = 2, 2, 4, 64, 6
    kn = torch.randn(B, H, S, D, device=dev).to(torch.bfloat16)
    kc = torch.zeros(B, H, cap, D, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    cos = torch.ones(B, S, D, dtype=torch.bfloat16, device=dev)
    sin = torch.zeros_like(cos)
    pos = torch.tensor([4, 6], dtype=torch.int32, device=dev)
    lens = torch.empty(B, dtype=torch.int32, device=dev)
    ab.rope_kv_append(torch.zeros(B, 1, S, D, dtype=torch.bfloat16, device=dev), kn, kn, cos, sin, kc, vc, pos,
                      kv_lens_out=lens)
    assert torch.equal(kc[0, :, 4:6], kn[0, :, :2]) and torch.all(kc[0, :, :4] == 0)
    assert torch.all(kc[1] == 0)
    assert lens.tolist() == [6, 6]
