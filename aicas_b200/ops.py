"""PyTorch-facing operators over the sm_100a C ABI.

Names, arguments, shapes and error types follow the reference package
``triton_qwen3vl`` (paths relative to the reference project):

* :func:`gqa_decode_attention`   - triton_qwen3vl/gqa_decode_attention.py:413-430
* :func:`gqa_flash_attention`    - triton_qwen3vl/gqa_flash_attention.py:254-282
* :func:`varlen_flash_attention` - triton_qwen3vl/varlen_flash_attention.py:404-438

plus the operators the reference leaves to Hugging Face or to its native
variant: :func:`rope_kv_append` (RoPE + in-place KV-cache append),
:func:`gqa_decode_partial` / :func:`merge_partials` (split-KV across devices).

Every operator runs hand-written CUDA on the caller's current stream.  There is
no CPU or PyTorch fallback: inputs the kernels cannot take raise ``ValueError``
(as the reference's ``_*_forward`` functions do) and a missing native library
raises ``RuntimeError``.  Outputs are freshly allocated; inputs are copied only
when their strides cannot be expressed to the kernels (the reference always
calls ``.contiguous()``).
"""
from __future__ import annotations

import ctypes
from typing import Sequence

import torch

from . import _native as nat

SUPPORTED_HEAD_DIMS = frozenset({16, 32, 64, 128})
TENSOR_CORE_HEAD_DIMS = frozenset({64, 128})

_DTYPE_CODES = {torch.float32: nat.DTYPE_F32, torch.float16: nat.DTYPE_F16, torch.bfloat16: nat.DTYPE_BF16}

# split-KV workspace, one zero-initialised buffer per (device, stream); the
# decode kernel leaves it zeroed after every call
_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}


def _stream_handle(device: torch.device) -> int:
    # an integer index: torch resolves a torch.device argument through a much
    # slower path, which showed up as a large share of a decode step's host time
    idx = device.index if device.index is not None else torch.cuda.current_device()
    return torch.cuda.current_stream(idx).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _reject_grad(*tensors: torch.Tensor) -> None:
    if torch.is_grad_enabled() and any(t.requires_grad for t in tensors):
        raise ValueError(
            "aicas_b200 attention is an inference backend: autograd through these kernels is not supported"
        )


def _aligned(t: torch.Tensor, strides: Sequence[int]) -> bool:
    eb = t.element_size()
    return t.data_ptr() % 16 == 0 and all((s * eb) % 16 == 0 for s in strides)


def _heads_ready(t: torch.Tensor) -> torch.Tensor:
    """[B, H, S, D] with unit stride on D and 16-byte strides elsewhere."""
    if t.stride(3) == 1 and _aligned(t, (t.stride(0), t.stride(1), t.stride(2))):
        return t
    return t.contiguous()


def _rows_ready(t: torch.Tensor) -> torch.Tensor:
    """[B, H, L, D] whose tokens are D elements apart (a cache view)."""
    d = t.shape[3]
    if t.stride(3) == 1 and (t.shape[2] <= 1 or t.stride(2) == d) and _aligned(t, (t.stride(0), t.stride(1))):
        return t
    return t.contiguous()


def _call_in_device(device: torch.device, fn, *args):
    if torch.cuda.current_device() != device.index:
        with torch.cuda.device(device):
            return fn(*args)
    return fn(*args)


def _reset_workspaces() -> None:
    """Zero-fills every workspace of this module (after a device error: a kernel
    whose bounded wait gave up may have left split counters behind)."""
    for (dev, _), ws in list(_WORKSPACES.items()) + list(_LINEAR_WORKSPACES.items()):
        with torch.cuda.device(dev):
            ws.zero_()
            torch.cuda.synchronize(dev)


nat.add_device_error_hook(_reset_workspaces)


def _workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    key = (device.index, stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def _as_lens(kv_lens, batch: int, device: torch.device) -> torch.Tensor | None:
    if kv_lens is None:
        return None
    if not isinstance(kv_lens, torch.Tensor):
        kv_lens = torch.as_tensor(list(kv_lens), dtype=torch.int32)
    if kv_lens.ndim != 1 or kv_lens.shape[0] != batch:
        raise ValueError(f"kv_lens must have shape [{batch}], got {tuple(kv_lens.shape)}")
    return kv_lens.to(device=device, dtype=torch.int32).contiguous()


# ---------------------------------------------------------------------- decode


def _check_decode(query, key, value, num_key_value_groups: int) -> None:
    """Input contract of can_use_gqa_decode_attention (gqa_decode_attention.py:8-41),
    widened to fp32 tensors; violations raise ValueError."""
    if num_key_value_groups < 1:
        raise ValueError("num_key_value_groups must be >= 1")
    if not (query.is_cuda and key.is_cuda and value.is_cuda):
        raise ValueError("GQA decode attention needs CUDA tensors")
    if query.ndim != 4 or key.ndim != 4 or value.ndim != 4:
        raise ValueError("query, key and value must be 4-D [B, H, S, D]")
    if not (query.device == key.device == value.device):
        raise ValueError("query, key and value must be on one device")
    if query.shape[0] != key.shape[0] or key.shape[0] != value.shape[0]:
        raise ValueError("batch sizes differ")
    if query.shape[2] != 1:
        raise ValueError("GQA decode attention needs q_len == 1")
    if key.shape[2] != value.shape[2] or key.shape[1] != value.shape[1]:
        raise ValueError("key and value shapes differ")
    if query.shape[1] != key.shape[1] * num_key_value_groups:
        raise ValueError("num_q_heads != num_kv_heads * num_key_value_groups")
    if query.shape[-1] != key.shape[-1] or key.shape[-1] != value.shape[-1]:
        raise ValueError("head dims differ")
    if query.shape[-1] not in SUPPORTED_HEAD_DIMS:
        raise ValueError(f"head_dim {query.shape[-1]} not in {sorted(SUPPORTED_HEAD_DIMS)}")
    if query.dtype not in _DTYPE_CODES:
        raise ValueError(f"unsupported dtype {query.dtype}")
    if key.dtype != query.dtype or value.dtype != query.dtype:
        raise ValueError("query, key and value dtypes differ")


def _decode_call(query, key, value, *, sm_scale, num_key_value_groups, kv_lens, split_tokens, out, lse, partial_o,
                 kv_starts=None, group=None):
    B, Hq, _, D = query.shape
    Hkv, L = key.shape[1], key.shape[2]
    device = query.device
    p = nat.DecodeParams()
    p.q, p.k, p.v = query.data_ptr(), key.data_ptr(), value.data_ptr()
    p.out = _ptr(out)
    p.lse = _ptr(lse)
    p.partial_o = _ptr(partial_o)
    p.kv_lens = _ptr(kv_lens)
    p.kv_starts = _ptr(kv_starts)
    p.q_stride_b, p.q_stride_h = query.stride(0), query.stride(1)
    p.k_stride_b, p.k_stride_h = key.stride(0), key.stride(1)
    p.v_stride_b, p.v_stride_h = value.stride(0), value.stride(1)
    if out is not None:
        p.o_stride_b, p.o_stride_h = out.stride(0), out.stride(1)
    p.batch, p.num_q_heads, p.num_kv_heads, p.head_dim = B, Hq, Hkv, D
    p.kv_capacity = L
    p.dtype = _DTYPE_CODES[query.dtype]
    p.sm_scale = float(sm_scale)
    p.split_tokens = int(split_tokens)

    def run():
        lib = nat.lib()
        stream = _stream_handle(device)
        if group is not None:
            # the decode with the cross-GPU merge fused in (group: nat.PeerGroup)
            nbytes = int(lib.aicas_decode_exchange_workspace_bytes(ctypes.byref(p)))
            ws = _workspace(device, stream, nbytes) if nbytes > 0 else None
            rc = lib.aicas_decode_gqa_exchange(ctypes.byref(p), ctypes.byref(group), _ptr(ws),
                                               ws.numel() if ws is not None else 0, stream)
            nat.check(rc, "aicas_decode_gqa_exchange")
            return
        nbytes = int(lib.aicas_decode_workspace_bytes(ctypes.byref(p)))
        ws = _workspace(device, stream, nbytes) if nbytes > 0 else None
        rc = lib.aicas_decode_gqa(ctypes.byref(p), _ptr(ws), ws.numel() if ws is not None else 0, stream)
        nat.check(rc, "aicas_decode_gqa")

    _call_in_device(device, run)


def gqa_decode_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    *,
    sm_scale: float,
    num_key_value_groups: int,
    kv_lens: torch.Tensor | Sequence[int] | None = None,
    return_lse: bool = False,
    split_tokens: int = 0,
    kv_starts: torch.Tensor | Sequence[int] | None = None,
):
    """q_len == 1 GQA attention: softmax(sm_scale * q K^T) V per request.

    query ``[B, Hq, 1, D]``, key/value ``[B, Hkv, L, D]`` -> ``[B, Hq, 1, D]``
    (gqa_decode_attention.py:413-430).  Extension: ``kv_lens`` (int32 ``[B]`` on
    the device) limits request ``b`` to its first ``kv_lens[b]`` cache slots, so
    a padded preallocated cache needs no slicing and no host synchronisation;
    ``kv_starts`` (int32 ``[B]``) skips the first ``kv_starts[b]`` slots (the
    padding of a left-padded batch).  With ``return_lse`` the base-2
    log-sum-exp ``[B, Hq]`` is returned too (the ``lse`` of
    gqa_decode_attention.py:141).
    """
    _reject_grad(query, key, value)
    _check_decode(query, key, value, num_key_value_groups)
    B, Hq, _, D = query.shape
    query = _heads_ready(query)
    key = _rows_ready(key)
    value = _rows_ready(value)
    lens = _as_lens(kv_lens, B, query.device)
    starts = _as_lens(kv_starts, B, query.device)
    out = torch.empty((B, 1, Hq, D), dtype=query.dtype, device=query.device).transpose(1, 2)
    lse = torch.empty((B, Hq), dtype=torch.float32, device=query.device) if return_lse else None
    _decode_call(query, key, value, sm_scale=sm_scale, num_key_value_groups=num_key_value_groups, kv_lens=lens,
                 split_tokens=split_tokens, out=out, lse=lse, partial_o=None, kv_starts=starts)
    return (out, lse) if return_lse else out


def gqa_decode_partial(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    *,
    sm_scale: float,
    num_key_value_groups: int,
    kv_lens: torch.Tensor | Sequence[int] | None = None,
    split_tokens: int = 0,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Decode over one shard of the cache: returns the normalised fp32 partial
    output ``[B, Hq, D]`` and its base-2 LSE ``[B, Hq]`` for :func:`merge_partials`."""
    _reject_grad(query, key, value)
    _check_decode(query, key, value, num_key_value_groups)
    B, Hq, _, D = query.shape
    query = _heads_ready(query)
    key = _rows_ready(key)
    value = _rows_ready(value)
    lens = _as_lens(kv_lens, B, query.device)
    po = torch.empty((B, Hq, D), dtype=torch.float32, device=query.device)
    lse = torch.empty((B, Hq), dtype=torch.float32, device=query.device)
    _decode_call(query, key, value, sm_scale=sm_scale, num_key_value_groups=num_key_value_groups, kv_lens=lens,
                 split_tokens=split_tokens, out=None, lse=lse, partial_o=po)
    return po, lse


def gqa_decode_exchange(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    group,
    *,
    sm_scale: float,
    num_key_value_groups: int,
    kv_lens: torch.Tensor | Sequence[int] | None = None,
    split_tokens: int = 0,
) -> torch.Tensor:
    """Decode over this rank's shard of a sequence-sharded cache with the
    cross-GPU merge fused into the decode kernel (``group``: the ranks' exchange
    buffers as a ``_native.PeerGroup``).  Collective; every rank returns the
    merged ``[B, Hq, 1, D]`` output.  16-bit caches, head_dim 128."""
    _reject_grad(query, key, value)
    _check_decode(query, key, value, num_key_value_groups)
    B, Hq, _, D = query.shape
    query = _heads_ready(query)
    key = _rows_ready(key)
    value = _rows_ready(value)
    lens = _as_lens(kv_lens, B, query.device)
    out = torch.empty((B, 1, Hq, D), dtype=query.dtype, device=query.device).transpose(1, 2)
    _decode_call(query, key, value, sm_scale=sm_scale, num_key_value_groups=num_key_value_groups, kv_lens=lens,
                 split_tokens=split_tokens, out=out, lse=None, partial_o=None, group=group)
    return out


def merge_partials(
    partial_o: torch.Tensor,
    partial_lse: torch.Tensor,
    *,
    out_dtype: torch.dtype = torch.bfloat16,
    return_lse: bool = False,
):
    """Merges P partials ``[P, B, H, D]`` / ``[P, B, H]`` (base-2 LSE) into
    ``[B, H, 1, D]`` of ``out_dtype``: o = sum_p 2^(lse_p - M) o_p / sum_p 2^(lse_p - M)."""
    if not (partial_o.is_cuda and partial_lse.is_cuda):
        raise ValueError("merge_partials needs CUDA tensors")
    if partial_o.dtype != torch.float32 or partial_lse.dtype != torch.float32:
        raise ValueError("partials must be fp32")
    if partial_o.ndim != 4 or partial_lse.ndim != 3 or partial_o.shape[:3] != partial_lse.shape:
        raise ValueError("partial_o must be [P, B, H, D] and partial_lse [P, B, H]")
    if out_dtype not in _DTYPE_CODES:
        raise ValueError(f"unsupported out_dtype {out_dtype}")
    P, B, H, D = partial_o.shape
    po = partial_o.contiguous()
    pl = partial_lse.contiguous()
    out = torch.empty((B, 1, H, D), dtype=out_dtype, device=po.device).transpose(1, 2)
    lse = torch.empty((B, H), dtype=torch.float32, device=po.device) if return_lse else None
    p = nat.MergeParams()
    p.partial_o, p.partial_lse, p.out, p.lse = po.data_ptr(), pl.data_ptr(), out.data_ptr(), _ptr(lse)
    p.o_stride_b, p.o_stride_h = out.stride(0), out.stride(1)
    p.num_partials, p.batch, p.num_heads, p.head_dim = P, B, H, D
    p.dtype = _DTYPE_CODES[out_dtype]

    def run():
        nat.check(nat.lib().aicas_merge_partials(ctypes.byref(p), _stream_handle(po.device)), "aicas_merge_partials")

    _call_in_device(po.device, run)
    return (out, lse) if return_lse else out


# ---------------------------------------------------------------------- RoPE + append


def rope_kv_append(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    positions: torch.Tensor,
    *,
    q_out: torch.Tensor | None = None,
    kv_lens_out: torch.Tensor | None = None,
    q_norm_weight: torch.Tensor | None = None,
    k_norm_weight: torch.Tensor | None = None,
    eps: float = 1e-6,
) -> torch.Tensor:
    """Rotates q and the new k with HF's rotate-half RoPE, writes k/v into the
    preallocated caches at ``positions[b] + s`` and returns the rotated q.

    query ``[B, Hq, S, D]``, key/value ``[B, Hkv, S, D]``, cos/sin ``[B, S, D]``,
    caches ``[B, Hkv, C, D]``, positions int32 ``[B]``.  With ``q_norm_weight`` /
    ``k_norm_weight`` the per-head RMSNorm of Qwen3VLTextAttention is applied
    first.  Slots at or past ``C`` are dropped (the reference truncates the
    payload at ``max_cache_len``).  ``kv_lens_out[b]`` receives the new length.
    """
    _reject_grad(query, key, value)
    tensors = (query, key, value, cos, sin, k_cache, v_cache)
    if not all(t.is_cuda for t in tensors) or not positions.is_cuda:
        raise ValueError("rope_kv_append needs CUDA tensors")
    if query.ndim != 4 or key.ndim != 4 or value.ndim != 4 or k_cache.ndim != 4 or v_cache.ndim != 4:
        raise ValueError("query/key/value/caches must be 4-D")
    B, Hq, S, D = query.shape
    Hkv = key.shape[1]
    if key.shape != (B, Hkv, S, D) or value.shape != key.shape:
        raise ValueError("key/value must be [B, Hkv, S, D] matching query")
    C = k_cache.shape[2]
    if k_cache.shape != (B, Hkv, C, D) or v_cache.shape != k_cache.shape:
        raise ValueError("caches must be [B, Hkv, C, D]")
    if cos.ndim != 3 or tuple(cos.shape[1:]) != (S, D) or cos.shape[0] not in (1, B) or sin.shape != cos.shape:
        raise ValueError("cos/sin must be [B, S, D] (or [1, S, D])")
    if query.dtype not in _DTYPE_CODES or any(t.dtype != query.dtype for t in (key, value, k_cache, v_cache)):
        raise ValueError("query, key, value and caches must share a dtype")
    if cos.dtype not in (query.dtype, torch.float32):
        raise ValueError("cos/sin must have the tensor dtype or fp32")
    if D % 2 or D > 128:
        raise ValueError("head_dim must be even and <= 128")
    cos3 = cos.expand(B, S, D)
    sin3 = sin.expand(B, S, D)
    if cos3.stride(2) != 1 or sin3.stride() != cos3.stride():
        cos3 = cos3.contiguous()
        sin3 = sin3.contiguous()
    for t in (query, key, value):
        if t.stride(3) != 1:
            raise ValueError("head_dim must be the unit-stride dimension")
    if k_cache.stride(3) != 1 or k_cache.stride(2) != D or v_cache.stride(3) != 1 or v_cache.stride(2) != D:
        raise ValueError("caches must store tokens D elements apart")
    pos = positions.to(dtype=torch.int32).contiguous()
    if pos.shape != (B,):
        raise ValueError(f"positions must be [{B}]")
    if q_out is None:
        q_out = torch.empty((B, S, Hq, D), dtype=query.dtype, device=query.device).transpose(1, 2)
    for w in (q_norm_weight, k_norm_weight):
        if w is not None and (w.shape != (D,) or w.dtype != query.dtype or not w.is_contiguous()):
            raise ValueError("norm weights must be contiguous [D] of the tensor dtype")
    p = nat.RopeAppendParams()
    p.q_in, p.q_out, p.k_in, p.v_in = query.data_ptr(), q_out.data_ptr(), key.data_ptr(), value.data_ptr()
    p.cos, p.sin = cos3.data_ptr(), sin3.data_ptr()
    p.k_cache, p.v_cache, p.positions = k_cache.data_ptr(), v_cache.data_ptr(), pos.data_ptr()
    p.kv_lens_out = _ptr(kv_lens_out)
    p.q_norm_weight, p.k_norm_weight, p.norm_eps = _ptr(q_norm_weight), _ptr(k_norm_weight), float(eps)
    p.qi_stride_b, p.qi_stride_h, p.qi_stride_s = query.stride(0), query.stride(1), query.stride(2)
    p.qo_stride_b, p.qo_stride_h, p.qo_stride_s = q_out.stride(0), q_out.stride(1), q_out.stride(2)
    p.k_stride_b, p.k_stride_h, p.k_stride_s = key.stride(0), key.stride(1), key.stride(2)
    p.v_stride_b, p.v_stride_h, p.v_stride_s = value.stride(0), value.stride(1), value.stride(2)
    p.cs_stride_b, p.cs_stride_s = cos3.stride(0), cos3.stride(1)
    p.kc_stride_b, p.kc_stride_h = k_cache.stride(0), k_cache.stride(1)
    p.vc_stride_b, p.vc_stride_h = v_cache.stride(0), v_cache.stride(1)
    p.batch, p.num_q_heads, p.num_kv_heads, p.seq_len, p.head_dim, p.capacity = B, Hq, Hkv, S, D, C
    p.dtype = _DTYPE_CODES[query.dtype]
    p.cs_dtype = _DTYPE_CODES[cos3.dtype]

    def run():
        nat.check(nat.lib().aicas_rope_kv_append(ctypes.byref(p), _stream_handle(query.device)), "aicas_rope_kv_append")

    _call_in_device(query.device, run)
    return q_out


# ---------------------------------------------------------------------- tensor-core attention


def _check_fmha_common(query, key, value, what: str) -> None:
    if not (query.is_cuda and key.is_cuda and value.is_cuda):
        raise ValueError(f"{what} needs CUDA tensors")
    if query.ndim != 4 or key.ndim != 4 or value.ndim != 4:
        raise ValueError("query, key and value must be 4-D [B, H, S, D]")
    if query.shape[-1] != key.shape[-1] or key.shape[-1] != value.shape[-1]:
        raise ValueError("head dims differ")
    if query.shape[-1] not in TENSOR_CORE_HEAD_DIMS:
        raise ValueError(f"{what}: head_dim {query.shape[-1]} not in {sorted(TENSOR_CORE_HEAD_DIMS)}")
    if query.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"{what} needs fp16 or bf16 tensors")
    if key.dtype != query.dtype or value.dtype != query.dtype:
        raise ValueError("query, key and value dtypes differ")
    if key.shape[2] != value.shape[2] or key.shape[1] != value.shape[1]:
        raise ValueError("key and value shapes differ")


def _fmha_params(query, key, value, out, sm_scale) -> nat.FmhaParams:
    p = nat.FmhaParams()
    p.q, p.k, p.v, p.out = query.data_ptr(), key.data_ptr(), value.data_ptr(), out.data_ptr()
    p.q_stride_b, p.q_stride_h, p.q_stride_s = query.stride(0), query.stride(1), query.stride(2)
    p.k_stride_b, p.k_stride_h, p.k_stride_s = key.stride(0), key.stride(1), key.stride(2)
    p.v_stride_b, p.v_stride_h, p.v_stride_s = value.stride(0), value.stride(1), value.stride(2)
    p.o_stride_b, p.o_stride_h, p.o_stride_s = out.stride(0), out.stride(1), out.stride(2)
    p.batch, p.num_q_heads, p.num_kv_heads = query.shape[0], query.shape[1], key.shape[1]
    p.seq_len_q, p.seq_len_kv, p.head_dim = query.shape[2], key.shape[2], query.shape[3]
    p.dtype = _DTYPE_CODES[query.dtype]
    p.sm_scale = float(sm_scale)
    return p


def gqa_flash_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    *,
    causal: bool,
    sm_scale: float,
    num_key_value_groups: int,
    kv_starts: torch.Tensor | Sequence[int] | None = None,
) -> torch.Tensor:
    """Causal GQA prefill, q_len == kv_len (gqa_flash_attention.py:254-282), on the
    tcgen05 tensor cores.  Returns ``[B, Hq, S, D]`` whose memory is laid out as
    ``[B, S, Hq, D]``, so the HF backend's transpose back is free.

    Extension: ``kv_starts`` (int32 ``[B]``) masks the first ``kv_starts[b]``
    positions of batch row ``b`` as keys (a left-padded batch): row ``i`` attends
    to keys ``[kv_starts[b], i]``, and rows before ``kv_starts[b]`` are zero."""
    if not causal:
        raise ValueError("gqa_flash_attention only supports causal prefill attention.")
    _reject_grad(query, key, value)
    _check_fmha_common(query, key, value, "gqa_flash_attention")
    if num_key_value_groups < 1 or query.shape[1] != key.shape[1] * num_key_value_groups:
        raise ValueError("num_q_heads != num_kv_heads * num_key_value_groups")
    if query.shape[0] != key.shape[0] or query.shape[2] != key.shape[2]:
        raise ValueError("gqa_flash_attention needs square causal prefill (q_len == kv_len)")
    B, Hq, S, D = query.shape
    query, key, value = _heads_ready(query), _heads_ready(key), _heads_ready(value)
    starts = _as_lens(kv_starts, B, query.device)
    out = torch.empty((B, S, Hq, D), dtype=query.dtype, device=query.device).transpose(1, 2)
    if S == 0:
        return out
    p = _fmha_params(query, key, value, out, sm_scale)
    p.kv_starts = _ptr(starts)

    def run():
        nat.check(nat.lib().aicas_prefill_gqa_causal(ctypes.byref(p), _stream_handle(query.device)),
                  "aicas_prefill_gqa_causal")

    _call_in_device(query.device, run)
    return out


def _cu_ready(cu: torch.Tensor, device: torch.device) -> torch.Tensor:
    if not isinstance(cu, torch.Tensor):
        cu = torch.as_tensor(list(cu), dtype=torch.int32)
    if cu.ndim != 1:
        raise ValueError("cu_seqlens must be 1-D")
    return cu.to(device=device, dtype=torch.int32, non_blocking=True).contiguous()


def varlen_flash_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    *,
    cu_seq_lens_q: torch.Tensor,
    cu_seq_lens_k: torch.Tensor,
    sm_scale: float,
    max_length_q: int | torch.Tensor | None = None,
    max_length_k: int | torch.Tensor | None = None,
    metadata_cache: dict | None = None,
) -> torch.Tensor:
    """Non-causal block-diagonal attention over packed sequences
    (varlen_flash_attention.py:404-438): query/key/value ``[1, H, T, D]`` with
    int32 ``cu_seq_lens`` -> ``[1, H, T, D]``.

    The tile schedule is derived from ``cu_seq_lens`` on the device, so unlike
    the reference (varlen_flash_attention.py:102-144) no host metadata is built
    and nothing is synchronised; ``max_length_*`` and ``metadata_cache`` are
    accepted for API compatibility and not needed.
    """
    del max_length_q, max_length_k, metadata_cache
    _reject_grad(query, key, value)
    _check_fmha_common(query, key, value, "varlen_flash_attention")
    if query.shape[0] != 1 or key.shape[0] != 1:
        raise ValueError("varlen_flash_attention needs batch 1 (packed sequences)")
    if query.shape[1] != key.shape[1]:
        raise ValueError("varlen_flash_attention needs as many key heads as query heads")
    if cu_seq_lens_q is None or cu_seq_lens_k is None:
        raise ValueError("cu_seq_lens_q and cu_seq_lens_k are required")
    cq = _cu_ready(cu_seq_lens_q, query.device)
    ck = _cu_ready(cu_seq_lens_k, query.device)
    if cq.numel() != ck.numel() or cq.numel() < 1:
        raise ValueError("cu_seq_lens_q and cu_seq_lens_k must have the same (non-zero) length")
    _, H, T, D = query.shape
    query, key, value = _heads_ready(query), _heads_ready(key), _heads_ready(value)
    out = torch.empty((1, T, H, D), dtype=query.dtype, device=query.device).transpose(1, 2)
    if T == 0:
        return out
    p = _fmha_params(query, key, value, out, sm_scale)
    p.cu_seqlens_q, p.cu_seqlens_k, p.num_seqs = cq.data_ptr(), ck.data_ptr(), cq.numel() - 1

    def run():
        nat.check(nat.lib().aicas_varlen_attention(ctypes.byref(p), _stream_handle(query.device)),
                  "aicas_varlen_attention")

    _call_in_device(query.device, run)
    return out


# ---------------------------------------------------------------------- decode-side products

# workspace of the decode-side products, one zero-initialised buffer per
# (device, stream); the kernel leaves its tile counters zeroed after every call
_LINEAR_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}

_LINEAR_DTYPES = {torch.float16: nat.DTYPE_F16, torch.bfloat16: nat.DTYPE_BF16}


def _linear_workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    key = (device.index, stream)
    ws = _LINEAR_WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 4 << 20), dtype=torch.uint8, device=device)
        _LINEAR_WORKSPACES[key] = ws
    return ws


def _overlaps(a: torch.Tensor, b: torch.Tensor) -> bool:
    if a.untyped_storage().data_ptr() != b.untyped_storage().data_ptr():
        return False
    a0, b0 = a.data_ptr(), b.data_ptr()
    a1 = a0 + ((a.shape[0] - 1) * a.stride(0) + a.shape[-1]) * a.element_size() if a.numel() else a0
    b1 = b0 + ((b.shape[0] - 1) * b.stride(0) + b.shape[-1]) * b.element_size() if b.numel() else b0
    return a0 < b1 and b0 < a1


def _row_major(t: torch.Tensor, what: str) -> torch.Tensor:
    if t.ndim != 2:
        raise ValueError(f"{what} must be 2-D")
    if t.stride(1) == 1 and _aligned(t, (t.stride(0),)):
        return t
    return t.contiguous()


def decode_linear(
    x: torch.Tensor,
    weights: torch.Tensor | Sequence[torch.Tensor],
    *,
    norm_weight: torch.Tensor | None = None,
    eps: float = 1e-6,
    residual: torch.Tensor | None = None,
    swiglu: bool = False,
    out: torch.Tensor | Sequence[torch.Tensor] | None = None,
    sumsq_out: torch.Tensor | None = None,
    x_sumsq: torch.Tensor | None = None,
    pdl: bool = True,
    stream_k: bool = False,
):
    """Weight-streaming products for the few rows of a decode step, on the
    tensor cores, with the neighbouring elementwise work fused:

    * ``x`` ``[R, K]`` (R <= 32), ``weights`` one ``[N, K]`` tensor or a list of
      them (one read of x for all, as qkv_linear_matvec_kernel and
      dual_linear_matvec_kernel in dujunbaoV1/native_cuda_ops/
      decode_q1_gqa_kernel.cu:222-331 do); returns ``x' W^T`` per weight.
    * ``norm_weight``: x' = Qwen3VLTextRMSNorm(x) with that weight and ``eps``
      (rmsnorm_kernel :127-157, rounded as HF rounds), else x' = x.
    * ``residual`` ``[R, N]``: returns ``residual + x' W^T`` (one weight), the
      residual add of Qwen3VLTextDecoderLayer; ``out=residual`` updates it in
      place.
    * ``swiglu=True`` with ``weights=(gate, up)``: returns
      ``silu(x' Wg^T) * (x' Wu^T)`` (gate_up_silu_matvec_kernel :174-220,
      rounded as HF Qwen3VLTextMLP rounds).
    * ``sumsq_out`` ``[R]`` fp32 (one weight, no swiglu): receives the sum of
      squares of each row of the rounded output, the statistics of the next
      RMSNorm.  A later call passes it as ``x_sumsq`` together with
      ``norm_weight``: x then goes by TMA straight into the tensor cores'
      operand layout and is normalised there, with no statistics pass over x.

    Every tensor is fp16 or bf16 of one dtype with unit stride on the last
    dimension.  Inputs the kernel cannot take raise ``ValueError``.

    ``stream_k=True`` splits K over all SMs in stream-K ranges even when the
    output has fewer 128-feature tiles than SMs (where the default is one CTA
    cluster per tile, reducing through distributed shared memory); ``pdl=False``
    launches without programmatic dependent launch.  Both only change timing.
    """
    single = isinstance(weights, torch.Tensor)
    ws_list = [weights] if single else list(weights)
    if not ws_list:
        raise ValueError("decode_linear needs at least one weight")
    tensors = [x, *ws_list] + [t for t in (norm_weight, residual) if t is not None]
    _reject_grad(*tensors)
    if not all(t.is_cuda for t in tensors):
        raise ValueError("decode_linear needs CUDA tensors")
    if x.dtype not in _LINEAR_DTYPES or any(t.dtype != x.dtype for t in tensors):
        raise ValueError("decode_linear needs fp16 or bf16 tensors of one dtype")
    x = _row_major(x, "x")
    R, K = x.shape
    if R > nat.LINEAR_MAX_ROWS:
        raise ValueError(f"decode_linear takes at most {nat.LINEAR_MAX_ROWS} rows (got {R})")
    if len(ws_list) > nat.LINEAR_MAX_SEGMENTS:
        raise ValueError(f"decode_linear takes at most {nat.LINEAR_MAX_SEGMENTS} weights")
    ws_list = [_row_major(w, "weight") for w in ws_list]
    if any(w.shape[1] != K for w in ws_list):
        raise ValueError("every weight must be [N, in_features] with in_features == x.shape[1]")
    if swiglu and (len(ws_list) != 2 or ws_list[0].shape != ws_list[1].shape):
        raise ValueError("swiglu needs weights=(gate, up) of one shape")
    if residual is not None and (swiglu or len(ws_list) != 1):
        raise ValueError("residual takes exactly one weight")
    if norm_weight is not None and (norm_weight.shape != (K,) or not norm_weight.is_contiguous()):
        raise ValueError(f"norm_weight must be a contiguous [{K}] tensor")
    if sumsq_out is not None:
        if swiglu or len(ws_list) != 1:
            raise ValueError("sumsq_out takes exactly one weight and no swiglu")
        if sumsq_out.shape != (R,) or sumsq_out.dtype != torch.float32 or not sumsq_out.is_cuda:
            raise ValueError(f"sumsq_out must be a CUDA fp32 [{R}] tensor")
    if x_sumsq is not None:
        if norm_weight is None:
            raise ValueError("x_sumsq needs norm_weight")
        if x_sumsq.shape != (R,) or x_sumsq.dtype != torch.float32 or not x_sumsq.is_cuda:
            raise ValueError(f"x_sumsq must be a CUDA fp32 [{R}] tensor")
    n_out = 1 if swiglu else len(ws_list)
    rows = [w.shape[0] for w in ws_list]
    if out is None:
        outs = [torch.empty((R, rows[i]), dtype=x.dtype, device=x.device) for i in range(n_out)]
    else:
        outs = [out] if isinstance(out, torch.Tensor) else list(out)
        if len(outs) != n_out or any(o.shape != (R, rows[i]) or o.stride(1) != 1 or o.dtype != x.dtype
                                     for i, o in enumerate(outs)):
            raise ValueError("out does not match the outputs")
    if residual is not None and (residual.shape != (R, rows[0]) or residual.stride(1) != 1):
        raise ValueError(f"residual must be [{R}, {rows[0]}] with unit stride on the last dimension")
    # every CTA reads all of x while others already write their outputs
    for o in outs:
        if _overlaps(o, x) or (norm_weight is not None and _overlaps(o, norm_weight)):
            raise ValueError("decode_linear outputs must not overlap x or norm_weight")
    p = nat.LinearParams()
    p.x, p.x_stride, p.batch, p.in_features = x.data_ptr(), x.stride(0), R, K
    p.norm_weight, p.eps = _ptr(norm_weight), float(eps)
    p.mode = nat.LINEAR_SWIGLU if swiglu else (nat.LINEAR_RESIDUAL if residual is not None else nat.LINEAR_STORE)
    if residual is not None:
        p.residual, p.residual_stride = residual.data_ptr(), residual.stride(0)
    p.num_segments = len(ws_list)
    for i, w in enumerate(ws_list):
        p.seg[i].weight, p.seg[i].weight_stride, p.seg[i].rows = w.data_ptr(), w.stride(0), w.shape[0]
        o = outs[min(i, n_out - 1)]
        p.seg[i].out, p.seg[i].out_stride = o.data_ptr(), o.stride(0)
    p.dtype = _LINEAR_DTYPES[x.dtype]
    p.flags = (0 if pdl else nat.LINEAR_NO_PDL) | (nat.LINEAR_STREAM_K if stream_k else 0)
    p.sumsq_out, p.x_sumsq = _ptr(sumsq_out), _ptr(x_sumsq)
    device = x.device

    def run():
        lib = nat.lib()
        stream = _stream_handle(device)
        nbytes = int(lib.aicas_linear_workspace_bytes(ctypes.byref(p)))
        if nbytes == 0 and R > 0:
            nat.check(nat.ERR_UNSUPPORTED, "aicas_linear_workspace_bytes")
        ws = _linear_workspace(device, stream, nbytes)
        nat.check(lib.aicas_decode_linear(ctypes.byref(p), ws.data_ptr(), ws.numel(), stream), "aicas_decode_linear")

    if R > 0:
        _call_in_device(device, run)
    return outs[0] if (single or swiglu) else tuple(outs)


# ---------------------------------------------------------------------- vision RoPE


def vision_rope(query: torch.Tensor, key: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """HF ``apply_rotary_pos_emb_vision(q, k, cos, sin)`` (transformers
    models/qwen3_vl/modeling_qwen3_vl.py:131-142) in one kernel, bit-identical:
    q/k ``[T, H, D]`` fp16/bf16 (any strides with a unit last one, e.g. views
    of the packed qkv projection ``[T, 3, H, D]``), cos/sin ``[T, D]`` (used
    as fp32, as HF upcasts them).
    Returns new contiguous ``(q_rot, k_rot)``."""
    _reject_grad(query, key)
    if not all(t.is_cuda for t in (query, key, cos, sin)):
        raise ValueError("vision_rope needs CUDA tensors")
    if query.ndim != 3 or key.shape != query.shape:
        raise ValueError("query and key must be [T, H, D] of one shape")
    T, H, D = query.shape
    if query.dtype not in _LINEAR_DTYPES or key.dtype != query.dtype:
        raise ValueError("vision_rope needs fp16 or bf16 query and key of one dtype")
    if cos.shape != (T, D) or sin.shape != (T, D) or not (cos.is_floating_point() and sin.is_floating_point()):
        raise ValueError(f"cos/sin must be floating-point [{T}, {D}]")
    # HF upcasts cos/sin to fp32 inside apply_rotary_pos_emb_vision (exact for 16-bit values)
    cos, sin = cos.float(), sin.float()
    if D % 16 or D > 256:
        raise ValueError("head_dim must be a multiple of 16 up to 256")

    def ready(t):
        return t if t.stride(-1) == 1 and _aligned(t, t.stride()[:-1]) else t.contiguous()

    query, key = ready(query), ready(key)
    cos, sin = cos.contiguous(), sin.contiguous()
    q_out = torch.empty((T, H, D), dtype=query.dtype, device=query.device)
    k_out = torch.empty_like(q_out)
    if T == 0:
        return q_out, k_out
    p = nat.VisionRopeParams()
    p.q_in, p.k_in, p.q_out, p.k_out = query.data_ptr(), key.data_ptr(), q_out.data_ptr(), k_out.data_ptr()
    p.cos, p.sin, p.cs_stride_t = cos.data_ptr(), sin.data_ptr(), cos.stride(0)
    p.qi_stride_t, p.qi_stride_h = query.stride(0), query.stride(1)
    p.ki_stride_t, p.ki_stride_h = key.stride(0), key.stride(1)
    p.qo_stride_t, p.qo_stride_h = q_out.stride(0), q_out.stride(1)
    p.ko_stride_t, p.ko_stride_h = k_out.stride(0), k_out.stride(1)
    p.tokens, p.heads, p.head_dim, p.dtype = T, H, D, _LINEAR_DTYPES[query.dtype]

    def run():
        nat.check(nat.lib().aicas_vision_rope(ctypes.byref(p), _stream_handle(query.device)), "aicas_vision_rope")

    _call_in_device(query.device, run)
    return q_out, k_out


# ---------------------------------------------------------------------- vision QKV projection + RoPE


def vision_qkv_rope(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, cos: torch.Tensor,
                    sin: torch.Tensor, num_heads: int) -> torch.Tensor:
    """The vision attention's packed projection and RoPE in one kernel:
    ``qkv = x W^T + b`` (``nn.Linear``, transformers
    models/qwen3_vl/modeling_qwen3_vl.py:205) viewed ``[T, 3, H, D]``, with
    ``apply_rotary_pos_emb_vision`` (:131-142) applied to its q and k parts.

    x ``[T, K]``, weight ``[3*H*D, K]``, bias ``[3*H*D]`` or None (fp16/bf16,
    one dtype), cos/sin ``[T, D]`` (used as fp32).  Returns a new ``[T, 3, H, D]``
    tensor; ``[:, 0]``, ``[:, 1]``, ``[:, 2]`` are the rotated q, the rotated k
    and v.  Needs D == 64, H a multiple of 4, K a multiple of 64."""
    tensors = [x, weight] + ([bias] if bias is not None else [])
    _reject_grad(*tensors)
    if not all(t.is_cuda for t in tensors + [cos, sin]):
        raise ValueError("vision_qkv_rope needs CUDA tensors")
    if x.dtype not in _LINEAR_DTYPES or any(t.dtype != x.dtype for t in tensors):
        raise ValueError("vision_qkv_rope needs fp16 or bf16 x, weight and bias of one dtype")
    x = _row_major(x, "x")
    weight = _row_major(weight, "weight")
    T, K = x.shape
    N = weight.shape[0]
    if weight.shape[1] != K or N % (3 * num_heads) != 0:
        raise ValueError(f"weight must be [3 * heads * head_dim, {K}]")
    D = N // (3 * num_heads)
    if bias is not None:
        if bias.shape != (N,):
            raise ValueError(f"bias must be a [{N}] tensor")
        if not bias.is_contiguous() or bias.data_ptr() % 16:
            bias = bias.contiguous().clone()
    if cos.shape != (T, D) or sin.shape != (T, D):
        raise ValueError(f"cos/sin must be [{T}, {D}]")
    cos, sin = cos.float().contiguous(), sin.float().contiguous()
    out = torch.empty((T, 3, num_heads, D), dtype=x.dtype, device=x.device)
    if T == 0:
        return out
    p = nat.VisionQkvParams()
    p.x, p.x_stride, p.weight, p.weight_stride = x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0)
    p.bias = _ptr(bias)
    p.cos, p.sin, p.cs_stride_t = cos.data_ptr(), sin.data_ptr(), cos.stride(0)
    p.out, p.out_stride = out.data_ptr(), out.stride(0)
    p.tokens, p.in_features, p.heads, p.head_dim, p.dtype = T, K, num_heads, D, _LINEAR_DTYPES[x.dtype]

    def run():
        nat.check(nat.lib().aicas_vision_qkv_rope(ctypes.byref(p), _stream_handle(x.device)), "aicas_vision_qkv_rope")

    _call_in_device(x.device, run)
    return out
