"""The decode kernel with the cross-GPU merge fused in, on one GPU.

With a group of one rank the kernel runs its whole exchange protocol against
its own buffer (results written into the slot, per-pair flags published, pairs
claimed and merged by CTAs whose own work is done), and the merge of one rank's
result is exact: the output must equal the plain decode's bit for bit, and the
fp64 oracle within the north-star bar.  Several calls in a row cover both slot
parities; one call through the exchange-merge kernel on the same buffer in
between checks that the two kernels share the epoch.

A group whose second "peer" is a buffer nobody publishes to (a flag that
nothing sets) checks the bounded wait: AICAS_DEVERR_PEER_TIMEOUT, zeros, and a
context that stays usable.  Only one kernel runs at a time, so nothing waits on
another launch.  The world-2..8 paths run in test_gpu_multigpu.py."""
from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest
import torch

import aicas_b200 as ab
from aicas_b200 import _native as nat
from aicas_b200 import ops

from tests.conftest import bf16_tolerance_check

pytestmark = pytest.mark.gpu


def _buffer(lib, nbytes):
    ptr = ctypes.c_void_p()
    handle = (ctypes.c_uint8 * nat.IPC_HANDLE_BYTES)()
    nat.check(lib.aicas_peer_buffer_alloc(nbytes, ctypes.byref(ptr), handle), "aicas_peer_buffer_alloc")
    return ptr.value


def _group(peers, rank, budget_ns=0):
    g = nat.PeerGroup()
    for r, p in enumerate(peers):
        g.peers[r] = p
    g.world, g.rank, g.wait_budget_ns = len(peers), rank, budget_ns
    return g


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize(
    "B,Hq,Hkv,L,lens,split",
    [
        (3, 16, 8, 12288, [12288, 7001, 1], 0),      # Qwen3-VL-2B heads; ragged, one-token cache
        (2, 16, 8, 65536, None, 0),                  # a long-context shard: splits and merges
        (64, 16, 8, 2048, "ragged", 0),              # many pairs: whole caches and halving splits
        (4, 32, 4, 4096, [0, 4096, 333, 2049], 256), # empty cache, G = 8, fixed splits
    ],
)
def test_fused_exchange_world1_matches_plain_decode(cuda_device, native_lib, dtype, B, Hq, Hkv, L, lens, split):
    from oracle import attention as oa

    assert nat.device_error_flags(clear=True) == 0
    g = torch.Generator(device=cuda_device).manual_seed(B * 1000 + L)
    D = 128
    if lens == "ragged":
        lens = torch.randint(1, L + 1, (B,), generator=torch.Generator().manual_seed(L)).tolist()
    lens_t = torch.tensor(lens, dtype=torch.int32, device=cuda_device) if lens is not None else None
    scale = D ** -0.5
    buf = _buffer(native_lib, native_lib.aicas_exchange_buffer_bytes(1, B, Hq, D))
    try:
        group = _group([buf], 0)
        for call in range(4):
            q = torch.randn(B, Hq, 1, D, generator=g, device=cuda_device).to(dtype)
            k = torch.randn(B, Hkv, L, D, generator=g, device=cuda_device).to(dtype)
            v = torch.randn(B, Hkv, L, D, generator=g, device=cuda_device).to(dtype)
            plain = ab.gqa_decode_attention(q, k, v, sm_scale=scale, num_key_value_groups=Hq // Hkv, kv_lens=lens_t,
                                            split_tokens=split)
            if call == 2:
                # the exchange-merge kernel on the same buffer (shares the epoch)
                po, pl = ops.gqa_decode_partial(q, k, v, sm_scale=scale, num_key_value_groups=Hq // Hkv,
                                                kv_lens=lens_t, split_tokens=split)
                p = nat.ExchangeParams()
                p.peers[0] = buf
                out = torch.empty(B, Hq, 1, D, dtype=dtype, device=cuda_device)
                p.partial_o, p.partial_lse, p.out, p.lse = po.data_ptr(), pl.data_ptr(), out.data_ptr(), None
                p.o_stride_b, p.o_stride_h = out.stride(0), out.stride(1)
                p.world, p.rank, p.batch, p.num_heads, p.head_dim = 1, 0, B, Hq, D
                p.dtype = ops._DTYPE_CODES[dtype]
                stream = torch.cuda.current_stream(cuda_device).cuda_stream
                nat.check(native_lib.aicas_exchange_merge(ctypes.byref(p), stream), "aicas_exchange_merge")
            else:
                out = ops.gqa_decode_exchange(q, k, v, group, sm_scale=scale, num_key_value_groups=Hq // Hkv,
                                              kv_lens=lens_t, split_tokens=split)
            torch.cuda.synchronize(cuda_device)
            if call != 2:
                assert torch.equal(out, plain), f"call {call}: fused output differs from the plain decode"
            if call == 0 and L <= 12288:
                ref = oa.decode_ragged(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                                       lens if lens is not None else [L] * B, scale, Hq // Hkv)
                bf16_tolerance_check(out.float().cpu().numpy(), ref)
        assert nat.device_error_flags() == 0
    finally:
        torch.cuda.synchronize(cuda_device)
        native_lib.aicas_peer_buffer_free(buf)


def test_fused_exchange_gives_up_on_a_silent_peer(cuda_device, native_lib):
    assert nat.device_error_flags(clear=True) == 0
    B, Hq, Hkv, L, D = 2, 16, 8, 4096, 128
    nbytes = native_lib.aicas_exchange_buffer_bytes(2, B, Hq, D)
    own, silent = _buffer(native_lib, nbytes), _buffer(native_lib, nbytes)
    try:
        group = _group([own, silent], 0, budget_ns=5_000_000)  # 5 ms
        q = torch.randn(B, Hq, 1, D, device=cuda_device).to(torch.bfloat16)
        k = torch.randn(B, Hkv, L, D, device=cuda_device).to(torch.bfloat16)
        torch.cuda.synchronize(cuda_device)
        t0 = time.perf_counter()
        for _ in range(2):  # both parities of the slots
            out = ops.gqa_decode_exchange(q, k, k, group, sm_scale=D ** -0.5, num_key_value_groups=2)
        torch.cuda.synchronize(cuda_device)
        elapsed = time.perf_counter() - t0
        assert elapsed < 1.0, f"the bounded waits took {elapsed:.3f} s"
        assert torch.count_nonzero(out) == 0  # zeros where the peer's results never came
        assert nat.device_error_flags(clear=True) & nat.DEVERR_PEER_TIMEOUT
        assert nat.device_error_flags() == 0
        # the context is still usable
        ref = ab.gqa_decode_attention(q, k, k, sm_scale=D ** -0.5, num_key_value_groups=2)
        assert np.isfinite(ref.float().cpu().numpy()).all()
    finally:
        torch.cuda.synchronize(cuda_device)
        native_lib.aicas_peer_buffer_free(own)
        native_lib.aicas_peer_buffer_free(silent)


def test_fused_exchange_rejects_bad_calls(cuda_device, native_lib):
    B, Hq, Hkv, L, D = 1, 4, 2, 256, 128
    buf = _buffer(native_lib, native_lib.aicas_exchange_buffer_bytes(1, B, Hq, D))
    try:
        q = torch.randn(B, Hq, 1, D, device=cuda_device).to(torch.bfloat16)
        k = torch.randn(B, Hkv, L, D, device=cuda_device).to(torch.bfloat16)
        with pytest.raises(ValueError, match="rank"):
            ops.gqa_decode_exchange(q, k, k, _group([buf], 1), sm_scale=0.1, num_key_value_groups=2)
        q64 = torch.randn(B, Hq, 1, 64, device=cuda_device).to(torch.bfloat16)
        k64 = torch.randn(B, Hkv, L, 64, device=cuda_device).to(torch.bfloat16)
        with pytest.raises(ValueError, match="head_dim 128"):
            ops.gqa_decode_exchange(q64, k64, k64, _group([buf], 0), sm_scale=0.1, num_key_value_groups=2)
    finally:
        torch.cuda.synchronize(cuda_device)
        native_lib.aicas_peer_buffer_free(buf)
