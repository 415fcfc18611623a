"""GPU parity of the split-KV GQA decode kernel and the partial merge against the
reference's golden vectors and the float64 oracle."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import aicas_b200 as ab
from aicas_b200 import _native as nat
from aicas_b200 import workloads as wl
from oracle import attention as oa
from tests.conftest import bf16_tolerance_check, checksum, load_golden

pytestmark = pytest.mark.gpu

DT = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def test_reference_decode_case_seed1(cuda_device):
    """The reference's own decode parity case (odd kv length 65, fp16, group 2)."""
    meta, a = load_golden("ref_decode_seed1")
    q, k, v = (torch.from_numpy(a[n]).to(cuda_device) for n in ("q", "k", "v"))
    out = ab.gqa_decode_attention(q, k, v, sm_scale=meta["scale"], num_key_value_groups=meta["groups"])
    assert out.shape == q.shape and out.dtype == torch.float16
    bf16_tolerance_check(_np(out.transpose(1, 2)), a["out"], max_abs=1e-2, mean_abs=1e-3)


def test_cfg1_fp32_against_golden(cuda_device):
    meta, a = load_golden("cfg1_decode")
    q, k, v = wl.cfg1_decode(meta["seed"])
    np.testing.assert_allclose(checksum(q, k, v), a["checksum"], rtol=1e-12)
    out = ab.gqa_decode_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), sm_scale=meta["scale"],
                                  num_key_value_groups=2)
    np.testing.assert_allclose(_np(out.transpose(1, 2)), a["out"], rtol=0, atol=2e-6)


def test_cfg2_ragged_padded_cache_against_golden(cuda_device):
    meta, a = load_golden("cfg2_ragged_small")
    g = wl.generator(meta["seed"])
    q = wl.randn((4, wl.HQ, 1, wl.HEAD_DIM), g, torch.bfloat16)
    kc = wl.randn((4, wl.HKV, meta["cap"], wl.HEAD_DIM), g, torch.bfloat16)
    vc = wl.randn((4, wl.HKV, meta["cap"], wl.HEAD_DIM), g, torch.bfloat16)
    np.testing.assert_allclose(checksum(q, kc, vc), a["checksum"], rtol=1e-12)
    lens = torch.tensor(meta["lens"], dtype=torch.int32, device=cuda_device)
    for split in (0, 64, 128):  # one unit per request, and several split-KV merges
        out = ab.gqa_decode_attention(q.to(cuda_device), kc.to(cuda_device), vc.to(cuda_device),
                                      sm_scale=meta["scale"], num_key_value_groups=2, kv_lens=lens, split_tokens=split)
        bf16_tolerance_check(_np(out.transpose(1, 2)), a["out"])


@pytest.mark.parametrize("dtype", ["bf16", "fp16", "fp32"])
@pytest.mark.parametrize("head_dim", [16, 32, 64, 128])
@pytest.mark.parametrize("groups", [1, 2, 4, 8])
def test_decode_shapes_against_oracle(cuda_device, dtype, head_dim, groups):
    torch.manual_seed(head_dim * 10 + groups)
    B, Hkv, L = 3, 2, 777
    q = torch.randn(B, Hkv * groups, 1, head_dim).to(DT[dtype])
    k = torch.randn(B, Hkv, L, head_dim).to(DT[dtype])
    v = torch.randn(B, Hkv, L, head_dim).to(DT[dtype])
    lens = [L, 1, 401]
    scale = head_dim ** -0.5
    ref = oa.decode_ragged(_np(q), _np(k), _np(v), lens, scale, groups)
    out, lse = ab.gqa_decode_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), sm_scale=scale,
                                       num_key_value_groups=groups, kv_lens=lens, return_lse=True)
    if dtype == "fp32":
        np.testing.assert_allclose(_np(out), ref, rtol=0, atol=5e-6)
    else:
        bf16_tolerance_check(_np(out), ref)
    for b, n in enumerate(lens):
        ref_lse = oa.lse_base2(_np(q[b : b + 1]), _np(k[b : b + 1]), scale, groups, kv_len=n)
        np.testing.assert_allclose(_np(lse[b : b + 1]), ref_lse, rtol=0, atol=1e-3)


@pytest.mark.parametrize("dtype,head_dim,groups", [("bf16", 128, 2), ("fp16", 64, 1), ("fp32", 128, 4)])
def test_auto_split_halving_table_against_oracle(cuda_device, dtype, head_dim, groups):
    """Many (request, KV head) pairs with the automatic split: the halving split
    table (for bf16 at head_dim 128: 384, 256, 256, 256 tokens at capacity 1024)
    with lengths on and around every split boundary, empty and full caches."""
    torch.manual_seed(21 + head_dim + groups)
    B, Hkv, L = 24, 8, 1024
    q = torch.randn(B, Hkv * groups, 1, head_dim).to(DT[dtype])
    k = torch.randn(B, Hkv, L, head_dim).to(DT[dtype])
    v = torch.randn(B, Hkv, L, head_dim).to(DT[dtype])
    lens = [0, 1, 255, 256, 257, 383, 384, 385, 639, 640, 641, 895, 896, 897, 1023, 1024]
    lens += torch.randint(1, L + 1, (B - len(lens),)).tolist()
    scale = head_dim ** -0.5
    ref = oa.decode_ragged(_np(q), _np(k), _np(v), lens, scale, groups)
    out = ab.gqa_decode_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), sm_scale=scale,
                                  num_key_value_groups=groups, kv_lens=lens)
    if dtype == "fp32":
        np.testing.assert_allclose(_np(out), ref, rtol=0, atol=5e-6)
    else:
        bf16_tolerance_check(_np(out), ref)
    assert nat.device_error_flags() == 0


def test_workspace_reuse_across_shapes(cuda_device):
    """One workspace serves calls of different shapes and split sizes in a row:
    the split counters sit at a fixed offset and every call leaves them zeroed."""
    torch.manual_seed(8)
    cases = [(4, 2, 320, 64), (2, 8, 4096, 128), (4, 2, 320, 128), (64, 8, 512, 64), (4, 2, 320, 0), (1, 8, 2000, 64)]
    for batch, hkv, L, split in cases * 2:
        q = torch.randn(batch, hkv * 2, 1, 128, dtype=torch.bfloat16, device=cuda_device)
        k = torch.randn(batch, hkv, L, 128, dtype=torch.bfloat16, device=cuda_device)
        v = torch.randn_like(k)
        lens = torch.randint(1, L + 1, (batch,)).tolist()
        out = ab.gqa_decode_attention(q, k, v, sm_scale=0.09, num_key_value_groups=2, kv_lens=lens,
                                      split_tokens=split)
        bf16_tolerance_check(_np(out), oa.decode_ragged(_np(q), _np(k), _np(v), lens, 0.09, 2))


def test_zero_and_full_lengths(cuda_device):
    torch.manual_seed(3)
    q = torch.randn(3, 16, 1, 128, dtype=torch.bfloat16, device=cuda_device)
    k = torch.randn(3, 8, 300, 128, dtype=torch.bfloat16, device=cuda_device)
    v = torch.randn_like(k)
    out, lse = ab.gqa_decode_attention(q, k, v, sm_scale=0.1, num_key_value_groups=2, kv_lens=[0, 300, 5],
                                       return_lse=True, split_tokens=128)
    assert torch.all(out[0] == 0) and torch.all(torch.isneginf(lse[0]))
    ref = oa.decode_ragged(_np(q), _np(k), _np(v), [0, 300, 5], 0.1, 2)
    bf16_tolerance_check(_np(out), ref)


def test_strided_query_and_cache_views(cuda_device):
    """HF hands a transposed q and (with a static cache) a length-sliced cache view."""
    torch.manual_seed(4)
    B, Hq, Hkv, D, cap, L = 2, 16, 8, 128, 512, 333
    q_bshd = torch.randn(B, 1, Hq, D, dtype=torch.bfloat16, device=cuda_device)
    q = q_bshd.transpose(1, 2)
    kc = torch.randn(B, Hkv, cap, D, dtype=torch.bfloat16, device=cuda_device)
    vc = torch.randn_like(kc)
    out = ab.gqa_decode_attention(q, kc[:, :, :L], vc[:, :, :L], sm_scale=D ** -0.5, num_key_value_groups=2)
    ref = oa.sdpa(_np(q), _np(kc[:, :, :L]), _np(vc[:, :, :L]), D ** -0.5, False, 2)
    bf16_tolerance_check(_np(out), ref)


def test_partials_and_merge_equal_the_full_decode(cuda_device):
    """Sequence-sharded decode emulated on one GPU: each shard's partial (o, LSE),
    merged, equals the single-device result (the cross-GPU path of config 5)."""
    torch.manual_seed(5)
    B, Hq, Hkv, D, L = 4, 16, 8, 128, 4096
    q = torch.randn(B, Hq, 1, D, dtype=torch.bfloat16, device=cuda_device)
    k = torch.randn(B, Hkv, L, D, dtype=torch.bfloat16, device=cuda_device)
    v = torch.randn_like(k)
    full = ab.gqa_decode_attention(q, k, v, sm_scale=D ** -0.5, num_key_value_groups=2)
    ref = oa.sdpa(_np(q), _np(k), _np(v), D ** -0.5, False, 2)
    for shards in (2, 4, 8):
        step = L // shards
        parts = [ab.gqa_decode_partial(q, k[:, :, r * step:(r + 1) * step], v[:, :, r * step:(r + 1) * step],
                                       sm_scale=D ** -0.5, num_key_value_groups=2) for r in range(shards)]
        po = torch.stack([p[0] for p in parts])
        pl = torch.stack([p[1] for p in parts])
        merged, lse = ab.merge_partials(po, pl, out_dtype=torch.bfloat16, return_lse=True)
        bf16_tolerance_check(_np(merged), ref)
        assert (merged.float() - full.float()).abs().max().item() <= 2 ** -7
        ref_lse = oa.lse_base2(_np(q), _np(k), D ** -0.5, 2)
        np.testing.assert_allclose(_np(lse), ref_lse, rtol=0, atol=1e-3)


def test_cfg2_full_size_layer_against_fp32_torch(cuda_device):
    """One full config-2 layer (B=64, caches padded to 4096, lengths ~U[256,4096])
    against a float32 torch computation of each request's valid prefix."""
    lens = wl.cfg2_lengths(0)
    kc, vc = wl.cfg2_cache(64, 4096, layer=0, device=cuda_device)
    st = wl.cfg2_step_inputs(lens, layer=0, device=cuda_device)
    out = ab.gqa_decode_attention(st.q, kc, vc, sm_scale=wl.SCALE_TEXT, num_key_value_groups=2,
                                  kv_lens=lens.to(cuda_device))
    worst_max, err_sum, count = 0.0, 0.0, 0
    for b in range(64):
        n = int(lens[b])
        kk = kc[b, :, :n].float().repeat_interleave(2, 0)
        vv = vc[b, :, :n].float().repeat_interleave(2, 0)
        s = torch.einsum("hd,hkd->hk", st.q[b, :, 0].float(), kk) * wl.SCALE_TEXT
        ref = torch.einsum("hk,hkd->hd", torch.softmax(s, -1), vv)
        e = (out[b, :, 0].float() - ref).abs()
        worst_max = max(worst_max, e.max().item())
        err_sum += e.sum().item()
        count += e.numel()
    assert worst_max <= 2e-2 and err_sum / count <= 2e-3


def test_cfg5_long_context_against_fp32_torch(cuda_device):
    q, k, v = wl.cfg5_decode(0, device=cuda_device)
    out = ab.gqa_decode_attention(q, k, v, sm_scale=wl.SCALE_TEXT, num_key_value_groups=2)
    kf = k.float().repeat_interleave(2, 1)
    s = torch.einsum("bhd,bhkd->bhk", q[:, :, 0].float(), kf) * wl.SCALE_TEXT
    del kf
    ref = torch.einsum("bhk,bhkd->bhd", torch.softmax(s, -1), v.float().repeat_interleave(2, 1))
    e = (out[:, :, 0].float() - ref).abs()
    assert e.max().item() <= 2e-2 and e.mean().item() <= 2e-3


def test_direct_c_abi_call(cuda_device, native_lib):
    """The C ABI driven with raw pointers and an explicit stream, as a non-Python
    host would bind it."""
    torch.manual_seed(6)
    q = torch.randn(2, 16, 1, 128, dtype=torch.bfloat16, device=cuda_device)
    k = torch.randn(2, 8, 200, 128, dtype=torch.bfloat16, device=cuda_device)
    v = torch.randn_like(k)
    out = torch.empty_like(q)
    p = nat.DecodeParams()
    p.q, p.k, p.v, p.out = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    p.q_stride_b, p.q_stride_h = q.stride(0), q.stride(1)
    p.k_stride_b, p.k_stride_h = k.stride(0), k.stride(1)
    p.v_stride_b, p.v_stride_h = v.stride(0), v.stride(1)
    p.o_stride_b, p.o_stride_h = out.stride(0), out.stride(1)
    p.batch, p.num_q_heads, p.num_kv_heads, p.head_dim, p.kv_capacity = 2, 16, 8, 128, 200
    p.dtype, p.sm_scale, p.split_tokens = nat.DTYPE_BF16, 128 ** -0.5, 64
    need = native_lib.aicas_decode_workspace_bytes(ctypes.byref(p))
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda_device)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        rc = native_lib.aicas_decode_gqa(ctypes.byref(p), ws.data_ptr(), need, stream.cuda_stream)
    assert rc == nat.OK, nat.last_error()
    stream.synchronize()
    bf16_tolerance_check(_np(out), oa.sdpa(_np(q), _np(k), _np(v), 128 ** -0.5, False, 2))
    # the call left its split counters at zero: the same workspace serves the next call
    first = out.clone()
    rc = native_lib.aicas_decode_gqa(ctypes.byref(p), ws.data_ptr(), need, stream.cuda_stream)
    assert rc == nat.OK
    stream.synchronize()
    assert torch.equal(out, first)


def test_cuda_graph_capture_and_replay(cuda_device):
    torch.manual_seed(7)
    q = torch.randn(8, 16, 1, 128, dtype=torch.bfloat16, device=cuda_device)
    k = torch.randn(8, 8, 2048, 128, dtype=torch.bfloat16, device=cuda_device)
    v = torch.randn_like(k)
    lens = torch.full((8,), 2000, dtype=torch.int32, device=cuda_device)
    eager = ab.gqa_decode_attention(q, k, v, sm_scale=0.088, num_key_value_groups=2, kv_lens=lens)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ab.gqa_decode_attention(q, k, v, sm_scale=0.088, num_key_value_groups=2, kv_lens=lens)  # workspace
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        captured = ab.gqa_decode_attention(q, k, v, sm_scale=0.088, num_key_value_groups=2, kv_lens=lens)
    for n in (2000, 17, 1):
        lens.fill_(n)
        graph.replay()
        torch.cuda.synchronize()
        ref = oa.decode_ragged(_np(q), _np(k), _np(v), [n] * 8, 0.088, 2)
        bf16_tolerance_check(_np(captured), ref)
    lens.fill_(2000)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(captured, eager)


def test_no_device_errors_recorded(cuda_device):
    torch.cuda.synchronize()
    assert nat.device_error_flags() == 0
