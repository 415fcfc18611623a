"""Padded text batches on the GPU: per-request key ranges (kv_starts / kv_lens)
in the decode and causal-prefill kernels, and HF's 2-D padding mask through
the text backend, against the reference's masked path (pinned in
tests/golden/padded_text.npz) and the float64 oracle.  Tolerance: the
north-star bf16 bar (max-abs 2e-2, mean-abs 2e-3), on the query rows Hugging
Face uses (real tokens)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import aicas_b200 as ab
from aicas_b200 import _native as nat
from aicas_b200 import backends
from oracle import attention as oa
from tests.conftest import bf16_tolerance_check, load_golden

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().float().cpu().numpy()


class _Attn(torch.nn.Module):
    def __init__(self, groups, scaling):
        super().__init__()
        self.num_key_value_groups, self.scaling, self.is_causal = groups, scaling, True


def test_golden_padded_batch_through_the_text_backend(cuda_device):
    meta, a = load_golden("padded_text")
    S, G, scale = meta["seq"], meta["groups"], meta["scale"]
    bf = lambda x: torch.from_numpy(x).to(torch.bfloat16).to(cuda_device)  # noqa: E731
    mask = torch.from_numpy(a["mask"]).to(cuda_device)
    q, k, v, qd = bf(a["q"]), bf(a["k"]), bf(a["v"]), bf(a["q_dec"])
    mod = _Attn(G, scale)
    pre, _ = backends.text_triton_attention(mod, q, k[:, :, :S], v[:, :, :S], mask[:, :S])
    _, real = oa.sdpa_padded(a["q"], a["k"][:, :, :S], a["v"][:, :, :S], a["mask"][:, :S], scale, G)
    got = _np(pre)  # [B, S, H, D]
    ref = a["out_prefill"]
    bf16_tolerance_check(got[real], ref[real])
    dec, _ = backends.text_triton_attention(mod, qd, k, v, mask)
    bf16_tolerance_check(_np(dec), a["out_decode"])


@pytest.mark.parametrize("head_dim,groups,split", [(128, 2, 0), (128, 2, 64), (128, 2, 128), (64, 4, 0), (64, 4, 128),
                                                   (64, 4, 256)])
def test_decode_with_start_offsets(cuda_device, split, head_dim, groups):
    """Request b attends to [kv_starts[b], kv_lens[b]): empty ranges, ranges off
    the tile grid, a one-token range and a whole cache."""
    g = torch.Generator().manual_seed(head_dim + split)
    B, hkv, L = 6, 2, 700
    starts = [0, 13, 640, 300, 699, 5]
    ends = [700, 500, 700, 300, 700, 6]
    q = torch.randn(B, hkv * groups, 1, head_dim, generator=g).to(torch.bfloat16)
    k = torch.randn(B, hkv, L, head_dim, generator=g).to(torch.bfloat16)
    v = torch.randn(B, hkv, L, head_dim, generator=g).to(torch.bfloat16)
    out = ab.gqa_decode_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), sm_scale=head_dim ** -0.5,
                                  num_key_value_groups=groups, split_tokens=split,
                                  kv_lens=torch.tensor(ends, dtype=torch.int32, device=cuda_device),
                                  kv_starts=torch.tensor(starts, dtype=torch.int32, device=cuda_device))
    ref = np.zeros(q.shape)
    for b, (s, e) in enumerate(zip(starts, ends)):
        if e > s:
            ref[b] = oa.sdpa(_np(q[b:b + 1]), _np(k[b:b + 1, :, s:e]), _np(v[b:b + 1, :, s:e]), head_dim ** -0.5,
                             False, groups)[0]
    bf16_tolerance_check(_np(out), ref)


@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("groups", [1, 2])
def test_prefill_with_start_offsets(cuda_device, head_dim, groups):
    """Left-padded causal prefill: row i of batch b sees keys [kv_starts[b], i];
    rows before kv_starts[b] are zero.  Starts on and off the 128-key tiles,
    one past the last row (all padding) and a batch row with no padding."""
    g = torch.Generator().manual_seed(head_dim * 3 + groups)
    B, hkv, S = 5, 2, 300
    starts = [0, 1, 128, 211, 300]
    q = torch.randn(B, hkv * groups, S, head_dim, generator=g).to(torch.bfloat16)
    k = torch.randn(B, hkv, S, head_dim, generator=g).to(torch.bfloat16)
    v = torch.randn(B, hkv, S, head_dim, generator=g).to(torch.bfloat16)
    scale = head_dim ** -0.5
    out = ab.gqa_flash_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), causal=True, sm_scale=scale,
                                 num_key_value_groups=groups,
                                 kv_starts=torch.tensor(starts, dtype=torch.int32, device=cuda_device))
    ref = np.zeros(q.shape)
    for b, s in enumerate(starts):
        if s < S:
            ref[b, :, s:] = oa.sdpa(_np(q[b:b + 1, :, s:]), _np(k[b:b + 1, :, s:]), _np(v[b:b + 1, :, s:]), scale,
                                    True, groups)[0]
    bf16_tolerance_check(_np(out), ref)


def test_left_padded_masks_of_several_shapes_through_the_backend(cuda_device):
    """HF-layout views ([B, S, H, D] storage) with a left-padded bool mask for
    prefill, then a decode step over the same cache: against the oracle."""
    g = torch.Generator().manual_seed(21)
    B, S, hq, hkv, D = 4, 257, 16, 8, 128
    pads = [0, 40, 129, 250]
    mask = torch.ones(B, S + 1, dtype=torch.bool)
    for b, p in enumerate(pads):
        mask[b, :p] = False
    qs = torch.randn(B, S, hq, D, generator=g).to(torch.bfloat16)
    ks = torch.randn(B, S + 1, hkv, D, generator=g).to(torch.bfloat16)
    vs = torch.randn(B, S + 1, hkv, D, generator=g).to(torch.bfloat16)
    qd = torch.randn(B, 1, hq, D, generator=g).to(torch.bfloat16)
    dev = lambda t: t.to(cuda_device).transpose(1, 2)  # noqa: E731
    mod = _Attn(2, D ** -0.5)
    md = mask.to(cuda_device)
    pre, _ = backends.text_triton_attention(mod, dev(qs), dev(ks)[:, :, :S], dev(vs)[:, :, :S], md[:, :S])
    ref, real = oa.sdpa_padded(_np(qs.transpose(1, 2)), _np(ks.transpose(1, 2))[:, :, :S],
                               _np(vs.transpose(1, 2))[:, :, :S], mask[:, :S].numpy(), D ** -0.5, 2)
    bf16_tolerance_check(_np(pre)[real], ref.transpose(0, 2, 1, 3)[real])
    dec, _ = backends.text_triton_attention(mod, dev(qd), dev(ks), dev(vs), md)
    ref_d, _ = oa.sdpa_padded(_np(qd.transpose(1, 2)), _np(ks.transpose(1, 2)), _np(vs.transpose(1, 2)),
                              mask.numpy(), D ** -0.5, 2)
    bf16_tolerance_check(_np(dec), ref_d.transpose(0, 2, 1, 3))
    torch.cuda.synchronize(cuda_device)
    assert nat.device_error_flags() == 0
