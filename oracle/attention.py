"""float64 restatement of the reference's attention on CPU (test infrastructure).

All functions take numpy arrays (any float dtype; computed in float64) in the
reference layouts and return float64 arrays in the reference's op layout
``[B, H, S, D]`` (the HF backends then transpose to ``[B, S, H, D]``).
"""
from __future__ import annotations

import numpy as np

LOG2E = 1.4426950408889634


def repeat_kv(x: np.ndarray, n_rep: int) -> np.ndarray:
    """fallback.py:7-12: [B, Hkv, S, D] -> [B, Hkv*n_rep, S, D], each KV head
    repeated for the n_rep consecutive query heads of its group."""
    if n_rep == 1:
        return x
    b, h, s, d = x.shape
    return np.broadcast_to(x[:, :, None], (b, h, n_rep, s, d)).reshape(b, h * n_rep, s, d)


def sdpa(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float, causal: bool, groups: int) -> np.ndarray:
    """fallback.py:39-63 / HF sdpa_attention_forward: softmax(scale q K^T [+ causal
    mask]) V.  The causal mask is top-left aligned (query i sees keys j <= i),
    which is what SDPA's is_causal means; HF only sets it when q_len > 1."""
    q = q.astype(np.float64)
    k = repeat_kv(k.astype(np.float64), groups)
    v = repeat_kv(v.astype(np.float64), groups)
    s = np.einsum("bhqd,bhkd->bhqk", q, k) * scale
    if causal and q.shape[2] > 1:
        qi = np.arange(q.shape[2])[:, None]
        kj = np.arange(k.shape[2])[None, :]
        s = np.where(kj <= qi, s, -np.inf)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("bhqk,bhkd->bhqd", p, v)


def lse_base2(q: np.ndarray, k: np.ndarray, scale: float, groups: int, kv_len: int | None = None) -> np.ndarray:
    """LSE of one decode query in the base-2 scaled domain of
    gqa_decode_attention.py:141: log2(sum_j 2^(scale*log2(e)*q.k_j)), shape [B, Hq]."""
    k = repeat_kv(k.astype(np.float64), groups)
    if kv_len is not None:
        k = k[:, :, :kv_len]
    s = np.einsum("bhd,bhkd->bhk", q[:, :, 0].astype(np.float64), k) * scale * LOG2E
    m = s.max(axis=-1)
    return m + np.log2(np.exp2(s - m[..., None]).sum(axis=-1))


def decode_ragged(q: np.ndarray, k: np.ndarray, v: np.ndarray, lens, scale: float, groups: int) -> np.ndarray:
    """Decode branch (backends.py:207-233) applied per request to the valid
    prefix k[b, :, :lens[b]] of a padded cache.  The reference has no length
    vector, so a padded batch is the per-request loop of unpadded calls."""
    out = np.zeros(q.shape, dtype=np.float64)
    for b, n in enumerate(lens):
        n = int(n)
        if n == 0:
            continue  # empty cache: defined as a zero output
        out[b : b + 1] = sdpa(q[b : b + 1], k[b : b + 1, :, :n], v[b : b + 1, :, :n], scale, False, groups)
    return out


def sdpa_padded(q: np.ndarray, k: np.ndarray, v: np.ndarray, mask: np.ndarray, scale: float, groups: int):
    """The reference's masked text path: backends.py:249-260 (prefill) and
    277-287 (decode) send a call with a padding mask to sdpa_fallback
    (fallback.py:23-64), i.e. HF's SDPA with the 4-D mask HF builds from the
    2-D one: query i (at absolute position i + kv_len - q_len) sees key j when
    mask[b, j] is nonzero and j <= that position.

    Returns (out [B, Hq, Sq, D], real [B, Sq]): ``real`` marks the query rows at
    real-token positions, the only rows Hugging Face uses (the outputs at
    padded positions are discarded; there they are set to 0 here)."""
    q = q.astype(np.float64)
    kk = repeat_kv(k.astype(np.float64), groups)
    vv = repeat_kv(v.astype(np.float64), groups)
    sq, skv = q.shape[2], kk.shape[2]
    pos = np.arange(sq) + (skv - sq)
    allowed = (np.asarray(mask)[:, None, None, :] != 0) & (np.arange(skv)[None, None, None, :] <= pos[None, None, :, None])
    s = np.einsum("bhqd,bhkd->bhqk", q, kk) * scale
    s = np.where(allowed, s, -np.inf)
    real = np.asarray(mask)[:, pos] != 0
    rows = allowed.any(axis=-1)  # [B, 1, Sq, 1] -> rows with at least one key
    m = np.where(rows[..., None], s.max(axis=-1, keepdims=True), 0.0)
    p = np.where(allowed, np.exp(s - m), 0.0)
    den = p.sum(axis=-1, keepdims=True)
    out = np.einsum("bhqk,bhkd->bhqd", p / np.where(den > 0, den, 1.0), vv)
    out = np.where(real[:, None, :, None], out, 0.0)
    return out, real


def varlen(q: np.ndarray, k: np.ndarray, v: np.ndarray, cu_q, cu_k, scale: float) -> np.ndarray:
    """_vision_varlen_fallback (backends.py:41-87): split the packed [1, H, T, D]
    tensors by cu_seqlens and run non-causal attention per segment."""
    out = np.zeros(q.shape, dtype=np.float64)
    cu_q = [int(x) for x in cu_q]
    cu_k = [int(x) for x in cu_k]
    for i in range(len(cu_q) - 1):
        q0, q1, k0, k1 = cu_q[i], cu_q[i + 1], cu_k[i], cu_k[i + 1]
        if q1 == q0 or k1 == k0:
            continue
        out[:, :, q0:q1] = sdpa(q[:, :, q0:q1], k[:, :, k0:k1], v[:, :, k0:k1], scale, False, 1)
    return out


def merge(partial_o: np.ndarray, partial_lse: np.ndarray) -> np.ndarray:
    """Combines normalised partials [P, ...] with base-2 LSEs [P, ...]:
    o = sum_p 2^(lse_p - M) o_p / sum_p 2^(lse_p - M)."""
    lse = partial_lse.astype(np.float64)
    m = lse.max(axis=0)
    w = np.exp2(lse - m)
    return (w[..., None] * partial_o.astype(np.float64)).sum(axis=0) / w.sum(axis=0)[..., None]


def sharded_decode_partials(q, k, v, scale: float, groups: int, shards: int):
    """What each of `shards` sequence-sharded ranks computes: the normalised
    output and base-2 LSE over its contiguous slice of the cache positions."""
    L = k.shape[2]
    step = (L + shards - 1) // shards
    outs, lses = [], []
    for r in range(shards):
        sl = slice(r * step, min(L, (r + 1) * step))
        outs.append(sdpa(q, k[:, :, sl], v[:, :, sl], scale, False, groups)[:, :, 0])
        lses.append(lse_base2(q, k[:, :, sl], scale, groups))
    return np.stack(outs), np.stack(lses)
