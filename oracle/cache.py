"""KV-cache append semantics on CPU (test infrastructure).

InplaceDecodeCacheLayer.update (dujunbaoV1/evaluation_wrapper.py:84-100 in the
reference project) writes the new tokens into a preallocated cache at
``[start, min(max_cache_len, start + S))`` and drops the rest of the payload.
The sm_100a kernel generalises ``start`` to a per-request position.
"""
from __future__ import annotations

import numpy as np


def kv_append(k_cache: np.ndarray, v_cache: np.ndarray, k_new: np.ndarray, v_new: np.ndarray, positions):
    """Returns updated copies of the [B, H, C, D] caches and the new lengths."""
    k_cache = k_cache.copy()
    v_cache = v_cache.copy()
    cap = k_cache.shape[2]
    seq = k_new.shape[2]
    lens = []
    for b, start in enumerate(positions):
        start = int(start)
        end = min(cap, start + seq)
        n = max(0, end - start)
        if n > 0:
            k_cache[b, :, start:end] = k_new[b, :, :n]
            v_cache[b, :, start:end] = v_new[b, :, :n]
        lens.append(min(max(start, 0) + seq, cap))
    return k_cache, v_cache, np.asarray(lens, dtype=np.int32)
