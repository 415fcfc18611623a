"""Decode-side products on the tensor cores (aicas_decode_linear) against the
CPU restatement in oracle/decode_linear.py.

Inputs are scaled so outputs are O(1) (x ~ N(0,1), W ~ N(0,1)/sqrt(K)); the
bar is the north-star one for 16-bit outputs, max-abs <= 2e-2 and mean-abs
<= 2e-3 against the exactly accumulated reference, plus a relative bound for
the few large outputs.  The kernel's fixed-order split reduction makes repeated
calls bit-identical, and every call leaves its tile counters at zero.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from aicas_b200 import _native as nat
from aicas_b200 import ops
from oracle import decode_linear as odl

pytestmark = pytest.mark.gpu


def _f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def _check(out: torch.Tensor, ref: np.ndarray) -> None:
    got = _f32(out).astype(np.float64)
    assert got.shape == ref.shape
    assert np.isfinite(got).all()
    err = np.abs(got - ref)
    bound = np.maximum(2e-2, 2 ** -7 * np.abs(ref))  # one bf16 unit of large values
    assert (err <= bound).all(), f"max-abs {err.max():.3e} at |ref| {np.abs(ref).flat[err.argmax()]:.3f}"
    assert err.mean() <= 2e-3, f"mean-abs {err.mean():.3e}"


def _data(R, K, rows, dtype, device, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(R, K, generator=g).to(dtype).to(device)
    ws = [(torch.randn(n, K, generator=g) / K ** 0.5).to(dtype).to(device) for n in rows]
    nw = (1 + 0.1 * torch.randn(K, generator=g)).to(dtype).to(device)
    return x, ws, nw


CASES = [
    # R, K, rows (one segment per entry)
    (1, 2048, [2048]),
    (8, 2048, [2048, 1024, 1024]),   # q/k/v of Qwen3-VL-2B
    (8, 6144, [2048]),               # down_proj
    (13, 2048, [1000]),              # rows not a multiple of 128
    (16, 512, [384, 128]),
    (17, 2048, [640]),               # 32-row padding
    (32, 1024, [4096]),
    (5, 200, [300]),                 # K not a multiple of 64
    (3, 64, [128]),                  # one K block
]


@pytest.mark.parametrize("R,K,rows", CASES)
@pytest.mark.parametrize("norm", [False, True])
@pytest.mark.parametrize("stream_k", [False, True])
def test_store_segments(cuda_device, native_lib, R, K, rows, norm, stream_k):
    """Both partitions: a CTA cluster per tile (the default below 148 tiles)
    and stream-K ranges over all SMs."""
    x, ws, nw = _data(R, K, rows, torch.bfloat16, cuda_device, seed=R * 7 + K)
    outs = ops.decode_linear(x, ws, norm_weight=nw if norm else None, eps=1e-6, stream_k=stream_k)
    outs = [outs] if isinstance(outs, torch.Tensor) else list(outs)
    refs = odl.decode_linear(_f32(x), [_f32(w) for w in ws], norm_weight=_f32(nw) if norm else None, eps=1e-6)
    for o, r in zip(outs, refs):
        _check(o, r)


@pytest.mark.parametrize("R,K,N", [(8, 2048, 2048), (8, 6144, 2048), (20, 2048, 1536), (1, 512, 200)])
@pytest.mark.parametrize("stream_k", [False, True])
def test_residual_in_place(cuda_device, native_lib, R, K, N, stream_k):
    x, (w,), _ = _data(R, K, [N], torch.bfloat16, cuda_device, seed=11 + R)
    res = torch.randn(R, N, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).to(cuda_device)
    ref = odl.decode_linear(_f32(x), [_f32(w)], residual=_f32(res))[0]
    y = ops.decode_linear(x, w, residual=res, out=res, stream_k=stream_k)
    assert y.data_ptr() == res.data_ptr()
    _check(res, ref)


@pytest.mark.parametrize("R,K,N", [(8, 2048, 6144), (1, 2048, 384), (24, 1024, 1000)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("stream_k", [False, True])
def test_swiglu_with_norm(cuda_device, native_lib, R, K, N, dtype, stream_k):
    x, (wg, wu), nw = _data(R, K, [N, N], dtype, cuda_device, seed=R + N)
    h = ops.decode_linear(x, (wg, wu), norm_weight=nw, eps=1e-6, swiglu=True, stream_k=stream_k)
    name = "bf16" if dtype == torch.bfloat16 else "fp16"
    ref = odl.decode_linear(_f32(x), [_f32(wg), _f32(wu)], norm_weight=_f32(nw), eps=1e-6, swiglu=True,
                            dtype=name)[0]
    _check(h, ref)


@pytest.mark.parametrize("R,K,N", [(8, 2048, 2048), (8, 6144, 2048), (32, 1024, 512), (3, 256, 1000)])
@pytest.mark.parametrize("stream_k", [False, True])
def test_sumsq_handoff(cuda_device, native_lib, R, K, N, stream_k):
    """The residual epilogue also returns each output row's sum of squares; the
    next product normalises its input in shared memory from those statistics
    and matches the call that computes them from x itself."""
    h, (w,), _ = _data(R, K, [N], torch.bfloat16, cuda_device, seed=5 + R)
    g = torch.Generator().manual_seed(6)
    x = torch.randn(R, N, generator=g).to(torch.bfloat16).to(cuda_device)
    w2 = (1 + 0.1 * torch.randn(N, generator=g)).to(torch.bfloat16).to(cuda_device)
    x0 = _f32(x)
    ss = torch.full((R,), -1.0, device=cuda_device)
    ops.decode_linear(h, w, residual=x, out=x, sumsq_out=ss, stream_k=stream_k)
    ref = odl.decode_linear(_f32(h), [_f32(w)], residual=x0)[0]
    _check(x, ref)
    xf = _f32(x).astype(np.float64)
    np.testing.assert_allclose(ss.cpu().numpy(), (xf ** 2).sum(axis=1), rtol=1e-5)
    # the next product: statistics from sumsq (x by TMA, normalised in place) vs
    # statistics computed from x by the kernel's own prologue
    wn = (torch.randn(384, N, generator=g) / N ** 0.5).to(torch.bfloat16).to(cuda_device)
    a = ops.decode_linear(x, wn, norm_weight=w2, eps=1e-6, x_sumsq=ss, stream_k=stream_k)
    b = ops.decode_linear(x, wn, norm_weight=w2, eps=1e-6, stream_k=stream_k)
    refn = odl.decode_linear(_f32(x), [_f32(wn)], norm_weight=_f32(w2), eps=1e-6)[0]
    _check(a, refn)
    torch.cuda.synchronize()
    assert (a != b).float().mean().item() < 0.02
    assert nat.device_error_flags() == 0


def test_lm_head_shape_and_determinism(cuda_device, native_lib):
    """151936 x 2048 (the tied LM head of Qwen3-VL-2B) with the final norm; two
    calls give identical bits, and the tile counters are zero afterwards.  A
    smaller call first leaves its partials in the shared workspace (a call of
    any shape must find its counters at zero)."""
    xs, ws_small, _ = _data(8, 2048, [2048, 1024, 1024], torch.bfloat16, cuda_device, seed=41)
    ops.decode_linear(xs, ws_small)
    x, (w,), nw = _data(8, 2048, [151936], torch.bfloat16, cuda_device, seed=42)
    a = ops.decode_linear(x, w, norm_weight=nw, eps=1e-6)
    b = ops.decode_linear(x, w, norm_weight=nw, eps=1e-6, pdl=False)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    sel = torch.arange(0, 151936, 97, device=cuda_device)
    ref = odl.decode_linear(_f32(x), [_f32(w[sel])], norm_weight=_f32(nw), eps=1e-6)[0]
    _check(a[:, sel], ref)
    ws = ops._LINEAR_WORKSPACES[(cuda_device.index, torch.cuda.current_stream(cuda_device).cuda_stream)]
    tiles = (151936 + 127) // 128
    assert int(ws[: tiles * 4].count_nonzero()) == 0
    assert nat.device_error_flags() == 0


def test_graph_capture_of_a_layer_chain(cuda_device, native_lib):
    """The decode layer's four products captured in one CUDA graph (programmatic
    dependent launches between them) give the same bits as eager calls."""
    R, H, I = 8, 1024, 3072
    g = torch.Generator().manual_seed(9)
    mk = lambda *s: (torch.randn(*s, generator=g) / s[-1] ** 0.5).to(torch.bfloat16).to(cuda_device)  # noqa: E731
    wq, wo, wg, wu, wd = mk(H, H), mk(H, H), mk(I, H), mk(I, H), mk(H, I)
    n1 = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(cuda_device)
    n2 = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(cuda_device)
    x0 = torch.randn(R, H, generator=g).to(torch.bfloat16).to(cuda_device)

    def chain(x):
        q = ops.decode_linear(x, wq, norm_weight=n1)
        ops.decode_linear(q, wo, residual=x, out=x, sumsq_out=ss)
        h = ops.decode_linear(x, (wg, wu), norm_weight=n2, x_sumsq=ss, swiglu=True)
        ops.decode_linear(h, wd, residual=x, out=x)
        return x

    ss = torch.zeros(R, device=cuda_device)

    eager = chain(x0.clone())
    xs = x0.clone()
    s = torch.cuda.Stream(cuda_device)
    s.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(s):
        chain(xs)  # warm-up on the capture stream (workspace)
    torch.cuda.current_stream(cuda_device).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        chain(xs)
    xs.copy_(x0)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(xs, eager)
    # the same chain on the oracle
    xr = _f32(x0)
    q = odl.decode_linear(xr, [_f32(wq)], norm_weight=_f32(n1))[0]
    from oracle.rope import round_to

    q = round_to(q.astype(np.float32), "bf16")
    xr = round_to(odl.decode_linear(q, [_f32(wo)], residual=xr)[0].astype(np.float32), "bf16")
    h = round_to(odl.decode_linear(xr, [_f32(wg), _f32(wu)], norm_weight=_f32(n2), swiglu=True)[0].astype(np.float32),
                 "bf16")
    ref = odl.decode_linear(h, [_f32(wd)], residual=xr)[0]
    _check(eager, ref)
    del graph


def test_rejects_what_the_kernel_cannot_take(cuda_device, native_lib):
    x, (w,), _ = _data(33, 256, [128], torch.bfloat16, cuda_device, seed=1)
    with pytest.raises(ValueError, match="at most 32 rows"):
        ops.decode_linear(x, w)
    with pytest.raises(ValueError, match="multiple of 8"):
        ops.decode_linear(x[:4, :100], w[:, :100])
    with pytest.raises(ValueError, match="one dtype"):
        ops.decode_linear(x[:4], w.half())
    with pytest.raises(ValueError, match="swiglu"):
        ops.decode_linear(x[:4], (w, w[:64]), swiglu=True)
