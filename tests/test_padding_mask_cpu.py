"""Padding masks through the text backend, host side (no GPU): HF's 2-D
padding mask becomes a per-request key range [start, end) on the device, for
left, right and no padding; masks the kernels cannot express raise ValueError
(the reference sends every masked call to SDPA instead, backends.py:249-260 and
277-287 in the reference project)."""
from __future__ import annotations

import pytest
import torch

from aicas_b200 import backends


def _mask(rows, width):
    m = torch.zeros(len(rows), width, dtype=torch.bool)
    for b, (s, e) in enumerate(rows):
        m[b, s:e] = True
    return m


@pytest.mark.parametrize("rows", [
    [(0, 9), (3, 9), (8, 9)],   # left padding (HF generate's default for decoder-only models)
    [(0, 9), (0, 4), (0, 1)],   # right padding
    [(2, 7), (0, 9), (5, 6)],   # both sides
    [(0, 0), (4, 9), (0, 9)],   # a row with no real token
])
def test_bounds_of_contiguous_runs(rows):
    m = _mask(rows, 9)
    start, end = backends.padding_bounds(m, 3, 9)
    assert start.dtype == torch.int32 and end.dtype == torch.int32
    for b, (s, e) in enumerate(rows):
        if s == e:
            assert int(start[b]) == int(end[b])
        else:
            assert (int(start[b]), int(end[b])) == (s, e)


def test_integer_masks_are_accepted():
    m = _mask([(2, 6), (0, 6)], 6).to(torch.int64)
    start, end = backends.padding_bounds(m, 2, 6)
    assert start.tolist() == [2, 0] and end.tolist() == [6, 6]


def test_holes_and_other_shapes_raise():
    holes = _mask([(0, 6)], 6)
    holes[0, 3] = False
    with pytest.raises(ValueError, match="contiguous run"):
        backends.padding_bounds(holes, 1, 6)
    with pytest.raises(ValueError, match="2-D padding mask"):
        backends.padding_bounds(torch.ones(1, 1, 6, 6, dtype=torch.bool), 1, 6)
    with pytest.raises(ValueError, match="2-D padding mask"):
        backends.padding_bounds(torch.ones(2, 5, dtype=torch.bool), 2, 6)


def test_one_derivation_per_mask_tensor():
    m = _mask([(1, 5), (0, 5)], 5)
    a = backends.padding_bounds(m, 2, 5)
    b = backends.padding_bounds(m, 2, 5)
    assert a[0] is b[0] and a[1] is b[1]
    m[0, 0] = True  # an in-place change bumps the version: derived again
    c = backends.padding_bounds(m, 2, 5)
    assert c[0].tolist() == [0, 0]
    other = m.clone()
    assert backends.padding_bounds(other, 2, 5)[0] is not c[0]


def test_mask_and_kv_lens_together_are_refused():
    class Attn(torch.nn.Module):
        num_key_value_groups, scaling, is_causal = 2, 0.125, True

    q = torch.randn(2, 4, 1, 16)
    k = torch.randn(2, 2, 5, 16)
    with pytest.raises(ValueError, match="either a padding mask or kv_lens"):
        backends.text_triton_attention(Attn(), q, k, k, _mask([(1, 5), (0, 5)], 5),
                                       kv_lens=torch.tensor([5, 5], dtype=torch.int32))
