"""GPU parity of the tcgen05 flash-attention kernels (causal GQA prefill and
packed varlen) against the reference's golden vectors and the float64 oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import aicas_b200 as ab
from aicas_b200 import _native as nat
from aicas_b200 import backends
from aicas_b200 import workloads as wl
from oracle import attention as oa
from tests.conftest import bf16_tolerance_check, checksum, load_golden

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().float().cpu().numpy()


def _dev(a, dev, dtype):
    return torch.from_numpy(np.asarray(a, dtype=np.float32)).to(dev, dtype)


def test_reference_prefill_case_seed0(cuda_device):
    """The reference's own prefill parity case: fp16, q [1,4,32,64], kv [1,2,32,64], causal."""
    meta, a = load_golden("ref_prefill_seed0")
    q, k, v = (torch.from_numpy(a[n]).to(cuda_device) for n in ("q", "k", "v"))
    out = ab.gqa_flash_attention(q, k, v, causal=True, sm_scale=meta["scale"], num_key_value_groups=2)
    assert out.shape == q.shape and out.dtype == torch.float16
    torch.testing.assert_close(out.transpose(1, 2).float().cpu(), torch.from_numpy(a["out"]), atol=1e-2, rtol=1e-2)
    bf16_tolerance_check(_np(out.transpose(1, 2)), a["out"])


def test_reference_varlen_case_seed2(cuda_device):
    """The reference's own varlen case: fp16 [1,2,9,64], cu_seqlens [0,2,5,9]."""
    meta, a = load_golden("ref_varlen_seed2")
    q, k, v = (torch.from_numpy(a[n]).to(cuda_device) for n in ("q", "k", "v"))
    cu = torch.from_numpy(a["cu"]).to(cuda_device)
    out = ab.varlen_flash_attention(q, k, v, cu_seq_lens_q=cu, cu_seq_lens_k=cu, sm_scale=meta["scale"],
                                    max_length_q=4, max_length_k=4)
    torch.testing.assert_close(out.transpose(1, 2).float().cpu(), torch.from_numpy(a["out"]), atol=1e-2, rtol=1e-2)


def test_cfg4_prefill_small_against_golden(cuda_device):
    meta, a = load_golden("cfg4_prefill_small")
    q, k, v = wl.cfg4_prefill(seed=meta["seed"], batch=meta["batch"], seq=meta["seq"], hq=meta["hq"], hkv=meta["hkv"])
    np.testing.assert_allclose(checksum(q, k, v), a["checksum"], rtol=1e-12)
    out = ab.gqa_flash_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), causal=True,
                                 sm_scale=meta["scale"], num_key_value_groups=2)
    bf16_tolerance_check(_np(out.transpose(1, 2)), a["out"])


def test_cfg3_varlen_small_against_golden(cuda_device):
    meta, a = load_golden("cfg3_varlen_small")
    q, k, v, cu, _ = wl.cfg3_varlen(seed=meta["seed"], images=meta["images"], heads=meta["heads"], lo=meta["lo"],
                                    hi=meta["hi"])
    np.testing.assert_allclose(checksum(q, k, v), a["checksum"], rtol=1e-12)
    cu = cu.to(cuda_device)
    out = ab.varlen_flash_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), cu_seq_lens_q=cu,
                                    cu_seq_lens_k=cu, sm_scale=meta["scale"])
    bf16_tolerance_check(_np(out.transpose(1, 2)), a["out"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("groups", [1, 2, 4])
@pytest.mark.parametrize("seq", [1, 7, 128, 129, 300])
def test_prefill_against_oracle(cuda_device, dtype, head_dim, groups, seq):
    torch.manual_seed(seq * 7 + groups)
    B, hkv = 2, 2
    q = torch.randn(B, hkv * groups, seq, head_dim).to(dtype)
    k = torch.randn(B, hkv, seq, head_dim).to(dtype)
    v = torch.randn(B, hkv, seq, head_dim).to(dtype)
    scale = head_dim ** -0.5
    out = ab.gqa_flash_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), causal=True,
                                 sm_scale=scale, num_key_value_groups=groups)
    bf16_tolerance_check(_np(out), oa.sdpa(_np(q), _np(k), _np(v), scale, True, groups))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("head_dim", [64, 128])
def test_varlen_against_oracle(cuda_device, dtype, head_dim):
    """Ragged sequences incl. an empty one, a 1-token one and lengths off the tile grid."""
    torch.manual_seed(head_dim)
    lens = [1, 0, 255, 256, 257, 700, 3, 130]
    cu = wl.cu_seqlens_from_lengths(lens)
    T, H = int(cu[-1]), 3
    q = torch.randn(1, H, T, head_dim).to(dtype)
    k = torch.randn(1, H, T, head_dim).to(dtype)
    v = torch.randn(1, H, T, head_dim).to(dtype)
    scale = head_dim ** -0.5
    out = ab.varlen_flash_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                                    cu_seq_lens_q=cu.to(cuda_device), cu_seq_lens_k=cu.to(cuda_device), sm_scale=scale)
    bf16_tolerance_check(_np(out), oa.varlen(_np(q), _np(k), _np(v), cu.tolist(), cu.tolist(), scale))


def test_varlen_with_distinct_q_and_k_segments(cuda_device):
    torch.manual_seed(11)
    lq, lk = [5, 130, 64], [200, 7, 300]
    cq, ck = wl.cu_seqlens_from_lengths(lq), wl.cu_seqlens_from_lengths(lk)
    q = torch.randn(1, 2, int(cq[-1]), 64).to(torch.bfloat16)
    k = torch.randn(1, 2, int(ck[-1]), 64).to(torch.bfloat16)
    v = torch.randn(1, 2, int(ck[-1]), 64).to(torch.bfloat16)
    out = ab.varlen_flash_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                                    cu_seq_lens_q=cq.to(cuda_device), cu_seq_lens_k=ck.to(cuda_device), sm_scale=0.125)
    bf16_tolerance_check(_np(out), oa.varlen(_np(q), _np(k), _np(v), cq.tolist(), ck.tolist(), 0.125))


def test_hf_layouts_through_the_backends(cuda_device):
    """The HF modules hand transposed views: text q/k/v are [B,S,H,D] storage seen
    as [B,H,S,D]; vision q/k/v come from a packed qkv projection.  No copies are
    needed and the backends return [B,S,H,D] contiguous."""
    torch.manual_seed(12)

    class M(torch.nn.Module):
        num_key_value_groups, scaling, is_causal = 2, 128 ** -0.5, True

    B, S, D = 2, 300, 128
    q = torch.randn(B, S, 16, D, device=cuda_device).to(torch.bfloat16).transpose(1, 2)
    k = torch.randn(B, S, 8, D, device=cuda_device).to(torch.bfloat16).transpose(1, 2)
    v = torch.randn(B, S, 8, D, device=cuda_device).to(torch.bfloat16).transpose(1, 2)
    out, w = backends.text_triton_attention(M(), q, k, v, None)
    assert w is None and out.shape == (B, S, 16, D) and out.is_contiguous()
    bf16_tolerance_check(_np(out.transpose(1, 2)), oa.sdpa(_np(q), _np(k), _np(v), M.scaling, True, 2))

    class V(torch.nn.Module):
        num_key_value_groups, scaling, is_causal = 1, 64 ** -0.5, False

    lens = [100, 37, 256]
    T = sum(lens)
    qkv = torch.randn(T, 3, 16, 64, device=cuda_device).to(torch.bfloat16)
    qv, kv_, vv = (x.transpose(0, 1).unsqueeze(0) for x in qkv.permute(1, 0, 2, 3).unbind(0))
    cu = wl.cu_seqlens_from_lengths(lens).to(cuda_device)
    out, w = backends.vision_triton_attention(V(), qv, kv_, vv, cu_seq_lens_q=cu, cu_seq_lens_k=cu,
                                              max_length_q=256, max_length_k=256, is_causal=False)
    assert out.shape == (1, T, 16, 64) and out.is_contiguous()
    bf16_tolerance_check(_np(out.transpose(1, 2)), oa.varlen(_np(qv), _np(kv_), _np(vv), cu.tolist(), cu.tolist(),
                                                             V.scaling))


def test_cfg4_full_size_against_fp32_torch(cuda_device):
    q, k, v = wl.cfg4_prefill(seed=0, device=cuda_device)
    out = ab.gqa_flash_attention(q, k, v, causal=True, sm_scale=wl.SCALE_TEXT, num_key_value_groups=2)
    mask = torch.ones(2048, 2048, dtype=torch.bool, device=cuda_device).tril()
    worst, tot, n = 0.0, 0.0, 0
    for b in range(8):
        for h in range(16):
            s = (q[b, h].float() @ k[b, h // 2].float().T) * wl.SCALE_TEXT
            ref = torch.softmax(s.masked_fill(~mask, float("-inf")), -1) @ v[b, h // 2].float()
            e = (out[b, h].float() - ref).abs()
            worst, tot, n = max(worst, e.max().item()), tot + e.sum().item(), n + e.numel()
    assert worst <= 2e-2 and tot / n <= 2e-3, (worst, tot / n)


def test_cfg3_full_size_against_fp32_torch(cuda_device):
    q, k, v, cu, lens = wl.cfg3_varlen(seed=0, device=cuda_device)
    out = ab.varlen_flash_attention(q, k, v, cu_seq_lens_q=cu, cu_seq_lens_k=cu, sm_scale=wl.SCALE_VIT)
    worst, tot, n = 0.0, 0.0, 0
    c = cu.tolist()
    for i in range(len(lens)):
        sl = slice(c[i], c[i + 1])
        s = torch.einsum("hqd,hkd->hqk", q[0, :, sl].float(), k[0, :, sl].float()) * wl.SCALE_VIT
        ref = torch.einsum("hqk,hkd->hqd", torch.softmax(s, -1), v[0, :, sl].float())
        e = (out[0, :, sl].float() - ref).abs()
        worst, tot, n = max(worst, e.max().item()), tot + e.sum().item(), n + e.numel()
    assert worst <= 2e-2 and tot / n <= 2e-3, (worst, tot / n)


def test_no_device_errors_after_attention(cuda_device):
    torch.cuda.synchronize()
    assert nat.device_error_flags() == 0
