"""aicas_decode_gqa_noalloc: the decode entry point for hosts that cannot
allocate device memory.

Some hosts pass this library only the pointers of tensors they already own and
have no allocator to give it (their allocator is not reachable across the C
boundary, or all device memory is reserved up front).  For them the split-KV
scratch lives in a static array inside the library.  These tests drive that
entry point through the C ABI and compare it with aicas_decode_gqa given a
workspace, on two calls in a row with different shapes (the second call
reuses the scratch the first one left behind).  The file is collected last so
that a run stopping at its first failure has run every other test before it.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from aicas_b200 import _native as nat
from oracle import attention as oa
from tests.conftest import bf16_tolerance_check

pytestmark = pytest.mark.gpu


def _params(q, k, v, out, lens, split_tokens) -> nat.DecodeParams:
    p = nat.DecodeParams()
    p.q, p.k, p.v, p.out = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    p.kv_lens = lens.data_ptr()
    p.q_stride_b, p.q_stride_h = q.stride(0), q.stride(1)
    p.k_stride_b, p.k_stride_h = k.stride(0), k.stride(1)
    p.v_stride_b, p.v_stride_h = v.stride(0), v.stride(1)
    p.o_stride_b, p.o_stride_h = out.stride(0), out.stride(1)
    p.batch, p.num_q_heads, p.num_kv_heads, p.head_dim = q.shape[0], q.shape[1], k.shape[1], q.shape[3]
    p.kv_capacity = k.shape[2]
    p.dtype = nat.DTYPE_BF16
    p.sm_scale = q.shape[3] ** -0.5
    p.split_tokens = split_tokens
    return p


def _np(t):
    return t.detach().float().cpu().numpy()


def test_noalloc_matches_the_workspace_entry_point_on_two_calls(cuda_device, native_lib):
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    cases = [(8, 8, 2048, 256, 0), (4, 8, 4096, 512, 1)]  # (B, Hkv, L, split_tokens, seed): several splits each
    for batch, hkv, L, split, seed in cases:
        g = torch.Generator(device=cuda_device).manual_seed(seed)
        q = torch.randn(batch, 2 * hkv, 1, 128, generator=g, device=cuda_device).to(torch.bfloat16)
        k = torch.randn(batch, hkv, L, 128, generator=g, device=cuda_device).to(torch.bfloat16)
        v = torch.randn(batch, hkv, L, 128, generator=g, device=cuda_device).to(torch.bfloat16)
        lens = torch.randint(1, L + 1, (batch,), generator=g, device=cuda_device, dtype=torch.int32)

        out_ws = torch.empty_like(q)
        p_ws = _params(q, k, v, out_ws, lens, split)
        need = native_lib.aicas_decode_workspace_bytes(ctypes.byref(p_ws))
        assert need > 0  # the case exercises the split-KV scratch
        ws = torch.zeros(need, dtype=torch.uint8, device=cuda_device)
        rc = native_lib.aicas_decode_gqa(ctypes.byref(p_ws), ws.data_ptr(), need, stream)
        assert rc == nat.OK, nat.last_error()

        out_na = torch.empty_like(q)
        p_na = _params(q, k, v, out_na, lens, split)
        rc = native_lib.aicas_decode_gqa_noalloc(ctypes.byref(p_na), stream)
        assert rc == nat.OK, nat.last_error()
        torch.cuda.synchronize(cuda_device)

        bf16_tolerance_check(_np(out_na), _np(out_ws))
        ref = oa.decode_ragged(_np(q), _np(k), _np(v), lens.tolist(), q.shape[3] ** -0.5, 2)
        bf16_tolerance_check(_np(out_na), ref)
    assert nat.device_error_flags() == 0


def test_noalloc_rejects_requests_beyond_its_static_scratch(cuda_device, native_lib):
    # real, correctly sized caches (every pointer the call is given stays inside
    # its allocation): 512 (request, KV head) pairs at capacity 2048 in splits of
    # 64 tokens need 512 x 32 splits x 2 heads x 129 x 4 B = ~17 MB of partials,
    # more than the 8 MiB static scratch, so the call is refused while planning
    q = torch.zeros(64, 16, 1, 128, dtype=torch.bfloat16, device=cuda_device)
    k = torch.zeros(64, 8, 2048, 128, dtype=torch.bfloat16, device=cuda_device)
    v = torch.zeros_like(k)
    lens = torch.full((64,), 2048, dtype=torch.int32, device=cuda_device)
    out = torch.empty_like(q)
    p = _params(q, k, v, out, lens, 64)
    rc = native_lib.aicas_decode_gqa_noalloc(ctypes.byref(p), torch.cuda.current_stream(cuda_device).cuda_stream)
    assert rc == nat.ERR_UNSUPPORTED
    assert "static scratch" in nat.last_error()
    del k, v


def test_noalloc_large_batch_takes_whole_caches(cuda_device, native_lib):
    """256 requests at capacity 2048 with the automatic split: the split table
    would need more partial slots than the static scratch holds, so the entry
    point takes whole caches as items (the 2048 pairs balance the CTAs on their
    own) and needs no scratch; the workspace entry point keeps the table."""
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    batch, hkv, L = 256, 8, 2048
    g = torch.Generator(device=cuda_device).manual_seed(5)
    q = torch.randn(batch, 2 * hkv, 1, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    k = torch.randn(batch, hkv, L, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    v = torch.randn(batch, hkv, L, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    lens = torch.randint(1, L + 1, (batch,), generator=g, device=cuda_device, dtype=torch.int32)
    out_ws = torch.empty_like(q)
    p_ws = _params(q, k, v, out_ws, lens, 0)
    need = native_lib.aicas_decode_workspace_bytes(ctypes.byref(p_ws))
    assert need > 8 << 20  # more than the static scratch
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda_device)
    assert native_lib.aicas_decode_gqa(ctypes.byref(p_ws), ws.data_ptr(), need, stream) == nat.OK, nat.last_error()
    out_na = torch.empty_like(q)
    p_na = _params(q, k, v, out_na, lens, 0)
    assert native_lib.aicas_decode_gqa_noalloc(ctypes.byref(p_na), stream) == nat.OK, nat.last_error()
    torch.cuda.synchronize(cuda_device)
    ref = oa.decode_ragged(_np(q), _np(k), _np(v), lens.tolist(), q.shape[3] ** -0.5, 2)
    bf16_tolerance_check(_np(out_na), ref)
    bf16_tolerance_check(_np(out_ws), ref)
    assert nat.device_error_flags() == 0
