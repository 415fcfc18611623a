"""CPU oracle for the Qwen3-VL attention hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy float64, what the reference computes on the
path the sm_100a kernels replace (paths relative to the reference project):

* ``attention.sdpa``          - triton_qwen3vl/fallback.py:7-12, 23-64 (repeat_kv + SDPA)
* ``attention.decode_ragged`` - the decode branch, backends.py:207-233, per request
* ``attention.varlen``        - backends.py:41-87 (_vision_varlen_fallback)
* ``attention.lse_base2``     - the LSE convention of gqa_decode_attention.py:141
* ``attention.merge``         - combination of split (out, LSE) partials
* ``rope.*``                  - HF apply_rotary_pos_emb / Qwen3VLTextRotaryEmbedding
                                (transformers 5.5.0, models/qwen3_vl/modeling_qwen3_vl.py)
* ``cache.kv_append``         - InplaceDecodeCacheLayer.update (dujunbaoV1/evaluation_wrapper.py:84-100)

Parity of the oracle is pinned by the golden vectors in ``tests/golden``,
produced by importing and running the reference package itself on CPU (its
operators take the PyTorch SDPA path there) with ``tests/golden/make_golden.py``.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this package, and only as the checker or the timed CPU baseline.
The product (``aicas_b200``) never imports it.
"""
