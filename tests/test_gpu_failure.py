"""Failure detection on one GPU, without a fault: the cross-GPU exchange
waits a bounded time for peers that never publish, then reports
AICAS_DEVERR_PEER_TIMEOUT, writes zeros and returns, and the context stays
usable.  The "peer" is a second local buffer that no kernel ever publishes to
(a flag that nothing sets); only one kernel runs, so nothing waits on another
launch."""
from __future__ import annotations

import ctypes
import time

import pytest
import torch

import aicas_b200 as ab
from aicas_b200 import _native as nat
from aicas_b200 import ops

pytestmark = pytest.mark.gpu


def _buffer(lib, nbytes):
    ptr = ctypes.c_void_p()
    handle = (ctypes.c_uint8 * nat.IPC_HANDLE_BYTES)()
    nat.check(lib.aicas_peer_buffer_alloc(nbytes, ctypes.byref(ptr), handle), "aicas_peer_buffer_alloc")
    return ptr.value


def test_exchange_gives_up_on_a_silent_peer(cuda_device, native_lib):
    assert nat.device_error_flags(clear=True) == 0
    B, H, D = 2, 4, 128
    nbytes = native_lib.aicas_exchange_buffer_bytes(2, B, H, D)
    own, silent = _buffer(native_lib, nbytes), _buffer(native_lib, nbytes)
    try:
        po = torch.randn(B, H, D, device=cuda_device)
        pl = torch.randn(B, H, device=cuda_device)
        out = torch.full((B, H, 1, D), 7.0, dtype=torch.bfloat16, device=cuda_device)
        p = nat.ExchangeParams()
        p.peers[0], p.peers[1] = own, silent
        p.partial_o, p.partial_lse, p.out, p.lse = po.data_ptr(), pl.data_ptr(), out.data_ptr(), None
        p.o_stride_b, p.o_stride_h = out.stride(0), out.stride(1)
        p.world, p.rank, p.batch, p.num_heads, p.head_dim = 2, 0, B, H, D
        p.dtype = nat.DTYPE_BF16
        p.wait_budget_ns = 5_000_000  # 5 ms
        stream = torch.cuda.current_stream(cuda_device).cuda_stream
        torch.cuda.synchronize(cuda_device)
        t0 = time.perf_counter()
        for _ in range(2):  # both parities of the slots
            nat.check(native_lib.aicas_exchange_merge(ctypes.byref(p), stream), "aicas_exchange_merge")
        torch.cuda.synchronize(cuda_device)
        elapsed = time.perf_counter() - t0
        assert elapsed < 1.0, f"the bounded waits took {elapsed:.3f} s"
        assert torch.count_nonzero(out) == 0  # zeros where the peers' partials never came

        # the workspaces of the operators are zero-filled again once the error is seen
        q = torch.randn(1, 4, 1, 128, device=cuda_device).to(torch.bfloat16)
        kv = torch.randn(1, 2, 512, 128, device=cuda_device).to(torch.bfloat16)
        ab.gqa_decode_attention(q, kv, kv, sm_scale=0.088, num_key_value_groups=2, split_tokens=64)
        for ws in ops._WORKSPACES.values():
            ws.fill_(3)
        flags = nat.device_error_flags()
        assert flags & nat.DEVERR_PEER_TIMEOUT
        assert all(int(torch.count_nonzero(ws)) == 0 for ws in ops._WORKSPACES.values())

        # the context is still usable and the word clears
        assert nat.device_error_flags(clear=True) & nat.DEVERR_PEER_TIMEOUT
        assert nat.device_error_flags() == 0
        out2 = ab.gqa_decode_attention(q, kv, kv, sm_scale=0.088, num_key_value_groups=2, split_tokens=64)
        ref = ab.gqa_decode_attention(q, kv, kv, sm_scale=0.088, num_key_value_groups=2)
        torch.testing.assert_close(out2, ref, atol=2e-2, rtol=0)
    finally:
        torch.cuda.synchronize(cuda_device)
        native_lib.aicas_peer_buffer_free(own)
        native_lib.aicas_peer_buffer_free(silent)
