"""The C-ABI library loads, exports exactly what include/aicas_b200.h declares,
its structs have the layout the ctypes binding assumes, and argument
validation rejects bad calls before anything reaches a GPU.  CPU only: no
kernel is launched."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from aicas_b200 import _native as nat
from tests.conftest import REPO

HEADER = REPO / "include" / "aicas_b200.h"


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"AICAS_API\s+[\w\s\*]+?\b(aicas_\w+)\s*\(", text))


def test_header_declares_the_binding_table():
    assert declared_functions() == set(nat.EXPORTS)


def test_library_exports_every_declared_symbol(native_lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(nat.library_path())], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert declared_functions() <= exported
    # nothing but the C ABI leaks out of the library
    assert {s for s in exported if s.startswith("aicas")} == declared_functions()


def test_version_and_capabilities(native_lib):
    v = nat.version()
    assert v.startswith("aicas_b200 ") and "sm_100a" in v
    caps = nat.capabilities()
    assert caps & nat.CAP_DECODE and caps & nat.CAP_MERGE and caps & nat.CAP_ROPE_APPEND
    assert caps & nat.CAP_PEER_EXCHANGE and caps & nat.CAP_DECODE_LINEAR and caps & nat.CAP_VISION_ROPE


STRUCTS = {
    "aicas_decode_params": nat.DecodeParams,
    "aicas_merge_params": nat.MergeParams,
    "aicas_fmha_params": nat.FmhaParams,
    "aicas_rope_append_params": nat.RopeAppendParams,
    "aicas_exchange_params": nat.ExchangeParams,
    "aicas_linear_segment": nat.LinearSegment,
    "aicas_linear_params": nat.LinearParams,
    "aicas_vision_rope_params": nat.VisionRopeParams,
    "aicas_vision_qkv_params": nat.VisionQkvParams,
    "aicas_peer_group": nat.PeerGroup,
}


def test_struct_layouts_match_the_header(tmp_path: Path):
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void) {"]
    for cname, py in STRUCTS.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-o", str(exe), str(src)], check=True)
    got = {}
    for line in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.splitlines():
        struct, field, value = line.split()
        got[(struct, field)] = int(value)
    for cname, py in STRUCTS.items():
        assert got[(cname, "size")] == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)


def _decode_params(**over) -> nat.DecodeParams:
    p = nat.DecodeParams()
    base = 1 << 20  # fake, 16-byte aligned; never dereferenced: validation fails first or only sizes are computed
    p.q, p.k, p.v, p.out = base, base * 2, base * 3, base * 4
    p.batch, p.num_q_heads, p.num_kv_heads, p.head_dim = 64, 16, 8, 128
    p.kv_capacity, p.dtype, p.sm_scale = 4096, nat.DTYPE_BF16, 128 ** -0.5
    p.q_stride_b, p.q_stride_h = 16 * 128, 128
    p.k_stride_b, p.k_stride_h = 8 * 4096 * 128, 4096 * 128
    p.v_stride_b, p.v_stride_h = 8 * 4096 * 128, 4096 * 128
    p.o_stride_b, p.o_stride_h = 16 * 128, 128
    for k, v in over.items():
        setattr(p, k, v)
    return p


@pytest.mark.parametrize(
    "over, code, text",
    [
        ({"num_q_heads": 24}, nat.ERR_UNSUPPORTED, "group size 3"),
        ({"num_q_heads": 12}, nat.ERR_INVALID, "not a multiple"),
        ({"head_dim": 96}, nat.ERR_UNSUPPORTED, "head_dim 96"),
        ({"dtype": 7}, nat.ERR_UNSUPPORTED, "dtype"),
        ({"q": (1 << 20) + 2}, nat.ERR_INVALID, "aligned"),
        ({"k_stride_h": 4096 * 128 + 4}, nat.ERR_INVALID, "16 bytes"),
        ({"out": None}, nat.ERR_INVALID, "out / partial_o"),
        ({"split_tokens": 100}, nat.ERR_UNSUPPORTED, "split_tokens"),
        ({"batch": 0}, nat.ERR_INVALID, "batch=0"),
    ],
)
def test_decode_validation(native_lib, over, code, text):
    p = _decode_params(**over)
    rc = native_lib.aicas_decode_gqa(ctypes.byref(p), None, 0, None)
    assert rc == code
    assert text in nat.last_error()
    with pytest.raises(ValueError):
        nat.check(rc, "aicas_decode_gqa")


def test_decode_workspace_is_required_for_split_kv(native_lib):
    p = _decode_params()
    need = native_lib.aicas_decode_workspace_bytes(ctypes.byref(p))
    assert need > 0
    rc = native_lib.aicas_decode_gqa(ctypes.byref(p), None, 0, None)
    assert rc == nat.ERR_WORKSPACE and str(need) in nat.last_error()


def test_decode_auto_split_table(native_lib):
    """Automatic split (148 SMs, 2 CTAs each).  Ragged batch of 512 (request,
    KV head) pairs at capacity 4096: equal splits would hold 1472 tokens; the
    halving table holds 2048, 1024, 512, 256, 256 -> 5 partial slots per pair.
    32 pairs: about one item per resident CTA (9 per pair -> 512 tokens,
    8 slots).  2048 pairs at capacity 2048: 1024, 512, 256, 256 -> 4 slots."""

    def up(x):
        return (x + 255) // 256 * 256

    def ws(units, splits):
        e = up((1 << 20) + units * splits * 2 * 128 * 4)
        return up(e + units * splits * 2 * 4)

    assert native_lib.aicas_decode_workspace_bytes(ctypes.byref(_decode_params())) == ws(512, 5)
    assert native_lib.aicas_decode_workspace_bytes(ctypes.byref(_decode_params(batch=4))) == ws(32, 8)
    p = _decode_params(batch=256, kv_capacity=2048)
    assert native_lib.aicas_decode_workspace_bytes(ctypes.byref(p)) == ws(2048, 4)


def test_decode_workspace_size_formula(native_lib):
    # split_tokens fixed -> max_splits = ceil(4096 / 512) = 8
    p = _decode_params(split_tokens=512)
    units, splits, g, d = 64 * 8, 8, 2, 128

    def up(x):
        return (x + 255) // 256 * 256

    expect = 1 << 20  # fixed counter region first
    expect = up(expect + units * splits * g * d * 4)
    expect = up(expect + units * splits * g * 4)
    assert native_lib.aicas_decode_workspace_bytes(ctypes.byref(p)) == expect
    # a single split needs no workspace
    assert native_lib.aicas_decode_workspace_bytes(ctypes.byref(_decode_params(split_tokens=4096))) == 0


def test_fmha_validation(native_lib):
    p = nat.FmhaParams()
    p.q = p.k = p.v = p.out = 1 << 20
    p.batch, p.num_q_heads, p.num_kv_heads, p.seq_len_q, p.seq_len_kv, p.head_dim = 1, 16, 8, 128, 128, 128
    p.dtype = nat.DTYPE_F32
    assert native_lib.aicas_prefill_gqa_causal(ctypes.byref(p), None) == nat.ERR_UNSUPPORTED
    p.dtype = nat.DTYPE_BF16
    p.seq_len_kv = 64
    assert native_lib.aicas_prefill_gqa_causal(ctypes.byref(p), None) == nat.ERR_UNSUPPORTED
    assert "q_len == kv_len" in nat.last_error()
    p.seq_len_kv = 128
    p.head_dim = 32
    assert native_lib.aicas_prefill_gqa_causal(ctypes.byref(p), None) == nat.ERR_UNSUPPORTED
    p.head_dim = 64
    assert native_lib.aicas_varlen_attention(ctypes.byref(p), None) == nat.ERR_UNSUPPORTED  # batch ok, Hq != Hkv
    assert "Hq == Hkv" in nat.last_error()
    p.num_kv_heads = 16
    assert native_lib.aicas_varlen_attention(ctypes.byref(p), None) == nat.ERR_INVALID  # no cu_seqlens
    assert native_lib.aicas_prefill_gqa_causal(None, None) == nat.ERR_INVALID


def test_rope_append_validation(native_lib):
    p = nat.RopeAppendParams()
    assert native_lib.aicas_rope_kv_append(ctypes.byref(p), None) == nat.ERR_INVALID
    assert "must be set" in nat.last_error()


def test_merge_validation(native_lib):
    p = nat.MergeParams()
    assert native_lib.aicas_merge_partials(ctypes.byref(p), None) == nat.ERR_INVALID


def test_exchange_buffer_size_and_validation(native_lib):
    # header (flags, epoch, then 8 per-pair flags of 8 bytes for each of the B*H
    # pairs, rounded up to 256 bytes) + 2 parities x world slots of B*H*(D+1)
    # floats rounded up to 4
    slot = (4 * 16 * 129 + 3) // 4 * 4
    header = (512 + 4 * 16 * 64 + 255) // 256 * 256
    assert native_lib.aicas_exchange_buffer_bytes(2, 4, 16, 128) == header + 2 * 2 * slot * 4
    assert native_lib.aicas_exchange_buffer_bytes(8, 4, 16, 128) == header + 2 * 8 * slot * 4
    assert native_lib.aicas_exchange_buffer_bytes(9, 4, 16, 128) == 0  # more ranks than the kernel takes
    assert native_lib.aicas_exchange_buffer_bytes(2, 0, 16, 128) == 0
    p = nat.ExchangeParams()
    p.world, p.rank, p.batch, p.num_heads, p.head_dim, p.dtype = 2, 2, 4, 16, 128, nat.DTYPE_BF16
    assert native_lib.aicas_exchange_merge(ctypes.byref(p), None) == nat.ERR_INVALID
    assert "rank 2 of world 2" in nat.last_error()
    p.rank = 0
    p.partial_o, p.partial_lse, p.out = 1 << 20, 2 << 20, 3 << 20
    p.peers[0], p.peers[1] = 4 << 20, None
    assert native_lib.aicas_exchange_merge(ctypes.byref(p), None) == nat.ERR_INVALID
    assert "rank 1" in nat.last_error()
    p.peers[1] = (5 << 20) + 16
    assert native_lib.aicas_exchange_merge(ctypes.byref(p), None) == nat.ERR_INVALID
    assert "256-byte aligned" in nat.last_error()
    p.peers[1] = 5 << 20
    p.head_dim = 130
    assert native_lib.aicas_exchange_merge(ctypes.byref(p), None) == nat.ERR_INVALID
    assert "multiple of 4" in nat.last_error()
    # the merge writes four outputs a store: out aligned, strides multiples of 16 bytes
    p.head_dim = 128
    p.out = (3 << 20) + 8
    assert native_lib.aicas_exchange_merge(ctypes.byref(p), None) == nat.ERR_INVALID
    assert "16-byte aligned" in nat.last_error()
    p.out, p.o_stride_b, p.o_stride_h = 3 << 20, 16 * 128, 132
    assert native_lib.aicas_exchange_merge(ctypes.byref(p), None) == nat.ERR_INVALID
    assert "multiples of 16 bytes" in nat.last_error()
    assert native_lib.aicas_peer_buffer_alloc(0, None, None) == nat.ERR_INVALID
    assert native_lib.aicas_peer_buffer_open(None, None) == nat.ERR_INVALID


def test_fused_exchange_validation(native_lib):
    p = _decode_params()
    g = nat.PeerGroup()
    call = lambda: native_lib.aicas_decode_gqa_exchange(ctypes.byref(p), ctypes.byref(g), 1 << 20, 1 << 20, None)
    assert native_lib.aicas_decode_gqa_exchange(ctypes.byref(p), None, None, 0, None) == nat.ERR_INVALID
    assert "group is NULL" in nat.last_error()
    g.world, g.rank = 2, 2
    assert call() == nat.ERR_INVALID and "rank 2 of world 2" in nat.last_error()
    g.world, g.rank = 9, 0
    assert call() == nat.ERR_INVALID and "at most 8 ranks" in nat.last_error()
    g.world, g.rank = 2, 0
    g.peers[0], g.peers[1] = 4 << 20, (5 << 20) + 64
    assert call() == nat.ERR_INVALID and "256-byte aligned" in nat.last_error()
    g.peers[1] = 5 << 20
    p.partial_o, p.lse = 6 << 20, 7 << 20
    assert call() == nat.ERR_INVALID and "partial_o NULL" in nat.last_error()
    p.partial_o = None
    p.head_dim = 64
    assert call() == nat.ERR_UNSUPPORTED and "head_dim 128" in nat.last_error()
    p.head_dim, p.dtype = 128, nat.DTYPE_F32
    assert call() == nat.ERR_UNSUPPORTED and "16-bit" in nat.last_error()
    # the workspace holds at least the scheduling counters (1 MiB), else the split-KV plan's size
    p.dtype = nat.DTYPE_BF16
    plain = native_lib.aicas_decode_workspace_bytes(ctypes.byref(p))
    assert native_lib.aicas_decode_exchange_workspace_bytes(ctypes.byref(p)) == max(plain, 1 << 20)
    p2 = _decode_params(split_tokens=4096)
    assert native_lib.aicas_decode_workspace_bytes(ctypes.byref(p2)) == 0
    assert native_lib.aicas_decode_exchange_workspace_bytes(ctypes.byref(p2)) == 1 << 20
    assert native_lib.aicas_decode_gqa_exchange(ctypes.byref(p2), ctypes.byref(g), 1 << 20, (1 << 20) - 1,
                                                None) == nat.ERR_WORKSPACE


def _linear_params(R=8, K=2048, rows=(2048, 1024, 1024), mode=nat.LINEAR_STORE) -> nat.LinearParams:
    p = nat.LinearParams()
    base = 1 << 20  # fake, aligned; never dereferenced (validation and sizing only)
    p.x, p.x_stride, p.batch, p.in_features = base, K, R, K
    p.mode, p.dtype, p.eps = mode, nat.DTYPE_BF16, 1e-6
    p.num_segments = len(rows)
    for i, n in enumerate(rows):
        p.seg[i].weight, p.seg[i].weight_stride, p.seg[i].rows = base * (2 + i), K, n
        p.seg[i].out, p.seg[i].out_stride = base * (8 + i), n
    return p


def test_linear_workspace_size(native_lib):
    # a fixed 64 KiB region of counters, then (stream-K only) two fp32 partial
    # slots per CTA, then (sumsq_out only) per-row sums of squares per share.
    # Fewer tiles than SMs (148 without a GPU): a CTA cluster per tile adds the
    # partials in shared memory, so no partial slots.
    base, slot16 = 65536, 16 * 128 * 4
    p = _linear_params()  # q/k/v: 32 tiles, cluster split
    assert native_lib.aicas_linear_workspace_bytes(ctypes.byref(p)) == base
    p.flags = nat.LINEAR_STREAM_K
    assert native_lib.aicas_linear_workspace_bytes(ctypes.byref(p)) == base + 2 * 148 * slot16
    p = _linear_params(R=20, K=6144, rows=(2048,), mode=nat.LINEAR_RESIDUAL)
    p.residual, p.residual_stride = 9 << 20, 2048
    assert native_lib.aicas_linear_workspace_bytes(ctypes.byref(p)) == base
    p.flags = nat.LINEAR_STREAM_K
    assert native_lib.aicas_linear_workspace_bytes(ctypes.byref(p)) == base + 2 * 148 * 2 * slot16
    # sumsq_out: 16 tiles x 8 ranks share the sums (128 shares of 32 floats)
    p.flags = 0
    p.sumsq_out = 10 << 20
    assert native_lib.aicas_linear_workspace_bytes(ctypes.byref(p)) == base + 128 * 32 * 4
    p = _linear_params(rows=(6144, 6144), mode=nat.LINEAR_SWIGLU)
    assert native_lib.aicas_linear_workspace_bytes(ctypes.byref(p)) == base
    p = _linear_params(rows=(151936,))  # the LM head: 1187 tiles, stream-K
    assert native_lib.aicas_linear_workspace_bytes(ctypes.byref(p)) == base + 2 * 148 * slot16
    p = _linear_params(rows=(16383 * 128 + 1,))  # more tiles than the counter region holds
    assert native_lib.aicas_linear_workspace_bytes(ctypes.byref(p)) == 0
    assert "exceed" in nat.last_error()


@pytest.mark.parametrize(
    "over, code, text",
    [
        ({"batch": 33}, nat.ERR_UNSUPPORTED, "0..32 rows"),
        ({"in_features": 100, "x_stride": 100}, nat.ERR_UNSUPPORTED, "multiple of 8"),
        ({"dtype": nat.DTYPE_F32}, nat.ERR_UNSUPPORTED, "fp16 or bf16"),
        ({"mode": 9}, nat.ERR_INVALID, "unknown mode"),
        ({"mode": nat.LINEAR_RESIDUAL}, nat.ERR_INVALID, "one segment"),
        ({"mode": nat.LINEAR_SWIGLU}, nat.ERR_INVALID, "two segments"),
        ({"x": (1 << 20) + 8}, nat.ERR_INVALID, "x must be"),
        ({"x_stride": 2047}, nat.ERR_INVALID, "x_stride"),
        ({"num_segments": 0}, nat.ERR_INVALID, "num_segments"),
    ],
)
def test_linear_validation(native_lib, over, code, text):
    p = _linear_params()
    for k, v in over.items():
        setattr(p, k, v)
    assert native_lib.aicas_decode_linear(ctypes.byref(p), None, 0, None) == code
    assert text in nat.last_error()
    assert native_lib.aicas_linear_workspace_bytes(ctypes.byref(p)) == 0


def test_linear_needs_its_workspace(native_lib):
    p = _linear_params()
    assert native_lib.aicas_decode_linear(ctypes.byref(p), None, 0, None) == nat.ERR_WORKSPACE
    assert "zero-initialised workspace" in nat.last_error()
    p.seg[1].weight_stride = 2044
    assert native_lib.aicas_decode_linear(ctypes.byref(p), None, 0, None) == nat.ERR_INVALID
    assert "segment 1" in nat.last_error()


def test_vision_rope_validation(native_lib):
    p = nat.VisionRopeParams()
    p.tokens, p.heads, p.head_dim, p.dtype = 8, 4, 64, nat.DTYPE_F32
    assert native_lib.aicas_vision_rope(ctypes.byref(p), None) == nat.ERR_UNSUPPORTED
    p.dtype, p.head_dim = nat.DTYPE_BF16, 40
    assert native_lib.aicas_vision_rope(ctypes.byref(p), None) == nat.ERR_UNSUPPORTED
    assert "multiple of 16" in nat.last_error()
    p.head_dim = 64
    assert native_lib.aicas_vision_rope(ctypes.byref(p), None) == nat.ERR_INVALID
    assert "must be set" in nat.last_error()
    p.tokens = 0
    assert native_lib.aicas_vision_rope(ctypes.byref(p), None) == nat.OK  # nothing to do
