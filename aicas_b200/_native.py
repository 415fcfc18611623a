"""ctypes binding of ``libaicas_b200.so`` (the C ABI in ``include/aicas_b200.h``).

The structures below mirror the C structs field by field; ``tests`` compile the
header with gcc and compare ``sizeof``/``offsetof`` against these definitions.
Loading is lazy and loud: any operator call without the library raises
``RuntimeError`` naming the build command; nothing falls back to PyTorch.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libaicas_b200.so"

DTYPE_F32 = 0
DTYPE_F16 = 1
DTYPE_BF16 = 2

OK = 0
ERR_INVALID = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_WORKSPACE = 4

DEVERR_WAIT_TIMEOUT = 1
DEVERR_TMEM = 2
DEVERR_PEER_TIMEOUT = 4

CAP_DECODE = 1
CAP_MERGE = 2
CAP_PREFILL_TCGEN05 = 4
CAP_VARLEN_TCGEN05 = 8
CAP_ROPE_APPEND = 16
CAP_PEER_EXCHANGE = 32
CAP_DECODE_LINEAR = 64
CAP_VISION_ROPE = 128
CAP_VISION_QKV = 256

LINEAR_MAX_SEGMENTS = 4
LINEAR_MAX_ROWS = 32
LINEAR_STORE = 0
LINEAR_RESIDUAL = 1
LINEAR_SWIGLU = 2
LINEAR_NO_PDL = 1
LINEAR_STREAM_K = 2

_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_vp = ctypes.c_void_p
_f32 = ctypes.c_float


class DecodeParams(ctypes.Structure):
    _fields_ = [
        ("q", _vp), ("k", _vp), ("v", _vp), ("out", _vp),
        ("lse", _vp), ("partial_o", _vp), ("kv_lens", _vp),
        ("q_stride_b", _i64), ("q_stride_h", _i64),
        ("k_stride_b", _i64), ("k_stride_h", _i64),
        ("v_stride_b", _i64), ("v_stride_h", _i64),
        ("o_stride_b", _i64), ("o_stride_h", _i64),
        ("batch", _i32), ("num_q_heads", _i32), ("num_kv_heads", _i32), ("head_dim", _i32),
        ("kv_capacity", _i32), ("dtype", _i32), ("sm_scale", _f32), ("split_tokens", _i32),
        ("kv_starts", _vp),
    ]


class MergeParams(ctypes.Structure):
    _fields_ = [
        ("partial_o", _vp), ("partial_lse", _vp), ("out", _vp), ("lse", _vp),
        ("o_stride_b", _i64), ("o_stride_h", _i64),
        ("num_partials", _i32), ("batch", _i32), ("num_heads", _i32), ("head_dim", _i32),
        ("dtype", _i32),
    ]


MAX_EXCHANGE_RANKS = 8
IPC_HANDLE_BYTES = 64


class ExchangeParams(ctypes.Structure):
    _fields_ = [
        ("peers", _vp * MAX_EXCHANGE_RANKS), ("partial_o", _vp), ("partial_lse", _vp), ("out", _vp), ("lse", _vp),
        ("o_stride_b", _i64), ("o_stride_h", _i64),
        ("world", _i32), ("rank", _i32), ("batch", _i32), ("num_heads", _i32), ("head_dim", _i32),
        ("dtype", _i32), ("wait_budget_ns", ctypes.c_uint64),
    ]


class PeerGroup(ctypes.Structure):
    _fields_ = [
        ("peers", _vp * MAX_EXCHANGE_RANKS), ("world", _i32), ("rank", _i32), ("wait_budget_ns", ctypes.c_uint64),
    ]


class FmhaParams(ctypes.Structure):
    _fields_ = [
        ("q", _vp), ("k", _vp), ("v", _vp), ("out", _vp),
        ("q_stride_b", _i64), ("q_stride_h", _i64), ("q_stride_s", _i64),
        ("k_stride_b", _i64), ("k_stride_h", _i64), ("k_stride_s", _i64),
        ("v_stride_b", _i64), ("v_stride_h", _i64), ("v_stride_s", _i64),
        ("o_stride_b", _i64), ("o_stride_h", _i64), ("o_stride_s", _i64),
        ("batch", _i32), ("num_q_heads", _i32), ("num_kv_heads", _i32), ("seq_len_q", _i32),
        ("seq_len_kv", _i32), ("head_dim", _i32), ("dtype", _i32), ("sm_scale", _f32),
        ("cu_seqlens_q", _vp), ("cu_seqlens_k", _vp), ("num_seqs", _i32), ("kv_starts", _vp),
    ]


class RopeAppendParams(ctypes.Structure):
    _fields_ = [
        ("q_in", _vp), ("q_out", _vp), ("k_in", _vp), ("v_in", _vp), ("cos", _vp), ("sin", _vp),
        ("k_cache", _vp), ("v_cache", _vp), ("positions", _vp), ("kv_lens_out", _vp),
        ("q_norm_weight", _vp), ("k_norm_weight", _vp), ("norm_eps", _f32),
        ("qi_stride_b", _i64), ("qi_stride_h", _i64), ("qi_stride_s", _i64),
        ("qo_stride_b", _i64), ("qo_stride_h", _i64), ("qo_stride_s", _i64),
        ("k_stride_b", _i64), ("k_stride_h", _i64), ("k_stride_s", _i64),
        ("v_stride_b", _i64), ("v_stride_h", _i64), ("v_stride_s", _i64),
        ("cs_stride_b", _i64), ("cs_stride_s", _i64),
        ("kc_stride_b", _i64), ("kc_stride_h", _i64),
        ("vc_stride_b", _i64), ("vc_stride_h", _i64),
        ("batch", _i32), ("num_q_heads", _i32), ("num_kv_heads", _i32), ("seq_len", _i32),
        ("head_dim", _i32), ("capacity", _i32), ("dtype", _i32), ("cs_dtype", _i32),
    ]


class VisionRopeParams(ctypes.Structure):
    _fields_ = [
        ("q_in", _vp), ("k_in", _vp), ("q_out", _vp), ("k_out", _vp), ("cos", _vp), ("sin", _vp),
        ("qi_stride_t", _i64), ("qi_stride_h", _i64), ("ki_stride_t", _i64), ("ki_stride_h", _i64),
        ("qo_stride_t", _i64), ("qo_stride_h", _i64), ("ko_stride_t", _i64), ("ko_stride_h", _i64),
        ("cs_stride_t", _i64), ("tokens", _i32), ("heads", _i32), ("head_dim", _i32), ("dtype", _i32),
    ]


class VisionQkvParams(ctypes.Structure):
    _fields_ = [
        ("x", _vp), ("x_stride", _i64), ("weight", _vp), ("weight_stride", _i64), ("bias", _vp),
        ("cos", _vp), ("sin", _vp), ("cs_stride_t", _i64), ("out", _vp), ("out_stride", _i64),
        ("tokens", _i32), ("in_features", _i32), ("heads", _i32), ("head_dim", _i32), ("dtype", _i32),
    ]


class LinearSegment(ctypes.Structure):
    _fields_ = [("weight", _vp), ("weight_stride", _i64), ("out", _vp), ("out_stride", _i64), ("rows", _i32)]


class LinearParams(ctypes.Structure):
    _fields_ = [
        ("x", _vp), ("x_stride", _i64), ("batch", _i32), ("in_features", _i32),
        ("norm_weight", _vp), ("eps", _f32), ("mode", _i32),
        ("residual", _vp), ("residual_stride", _i64),
        ("num_segments", _i32), ("seg", LinearSegment * LINEAR_MAX_SEGMENTS),
        ("dtype", _i32), ("flags", _i32),
        ("sumsq_out", _vp), ("x_sumsq", _vp),
    ]


# name -> (restype, argtypes); exactly the functions declared in include/aicas_b200.h
EXPORTS = {
    "aicas_decode_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(DecodeParams)]),
    "aicas_decode_gqa": (ctypes.c_int, [ctypes.POINTER(DecodeParams), _vp, ctypes.c_size_t, _vp]),
    "aicas_decode_gqa_noalloc": (ctypes.c_int, [ctypes.POINTER(DecodeParams), _vp]),
    "aicas_merge_partials": (ctypes.c_int, [ctypes.POINTER(MergeParams), _vp]),
    "aicas_exchange_buffer_bytes": (ctypes.c_size_t, [_i32, _i32, _i32, _i32]),
    "aicas_peer_buffer_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(_vp), _vp]),
    "aicas_peer_buffer_free": (ctypes.c_int, [_vp]),
    "aicas_peer_buffer_open": (ctypes.c_int, [_vp, ctypes.POINTER(_vp)]),
    "aicas_peer_buffer_close": (ctypes.c_int, [_vp]),
    "aicas_exchange_merge": (ctypes.c_int, [ctypes.POINTER(ExchangeParams), _vp]),
    "aicas_decode_exchange_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(DecodeParams)]),
    "aicas_decode_gqa_exchange": (ctypes.c_int, [ctypes.POINTER(DecodeParams), ctypes.POINTER(PeerGroup), _vp,
                                                 ctypes.c_size_t, _vp]),
    "aicas_prefill_gqa_causal": (ctypes.c_int, [ctypes.POINTER(FmhaParams), _vp]),
    "aicas_varlen_attention": (ctypes.c_int, [ctypes.POINTER(FmhaParams), _vp]),
    "aicas_rope_kv_append": (ctypes.c_int, [ctypes.POINTER(RopeAppendParams), _vp]),
    "aicas_vision_rope": (ctypes.c_int, [ctypes.POINTER(VisionRopeParams), _vp]),
    "aicas_vision_qkv_rope": (ctypes.c_int, [ctypes.POINTER(VisionQkvParams), _vp]),
    "aicas_linear_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(LinearParams)]),
    "aicas_decode_linear": (ctypes.c_int, [ctypes.POINTER(LinearParams), _vp, ctypes.c_size_t, _vp]),
    "aicas_version": (ctypes.c_char_p, []),
    "aicas_capabilities": (ctypes.c_uint32, []),
    "aicas_last_error": (ctypes.c_char_p, []),
    "aicas_device_error_flags": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int]),
}

_lib: ctypes.CDLL | None = None
_load_error: str | None = None


def _load() -> ctypes.CDLL:
    global _lib, _load_error
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("AICAS_B200_LIB", LIB_PATH))
    if not path.exists():
        _load_error = (
            f"native library {path} is missing; build it with `python -m aicas_b200.build` "
            "(nvcc for sm_100a). The attention operators have no CPU fallback."
        )
        raise RuntimeError(_load_error)
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in EXPORTS.items():
        try:
            fn = getattr(lib, name)
        except AttributeError as exc:
            _load_error = f"native library {path} lacks {name} (stale build?); rebuild with `python -m aicas_b200.build`"
            raise RuntimeError(_load_error) from exc
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def lib() -> ctypes.CDLL:
    """Returns the loaded library, raising RuntimeError when it is unavailable."""
    return _load()


def available() -> bool:
    try:
        _load()
        return True
    except (RuntimeError, OSError):
        return False


def library_path() -> Path:
    return Path(os.environ.get("AICAS_B200_LIB", LIB_PATH))


def last_error() -> str:
    return lib().aicas_last_error().decode(errors="replace")


def check(rc: int, what: str) -> None:
    """Turns a C-ABI status into the reference's exception types."""
    if rc == OK:
        return
    msg = f"{what}: {last_error()}"
    if rc in (ERR_INVALID, ERR_UNSUPPORTED, ERR_WORKSPACE):
        raise ValueError(msg)
    raise RuntimeError(msg)


def version() -> str:
    return lib().aicas_version().decode()


def capabilities() -> int:
    return int(lib().aicas_capabilities())


# called when the device error word is found non-zero: the workspaces whose
# counters a kernel cut short by a failed wait may have left non-zero are
# zero-filled again (the header's rule for reusing them)
_ERROR_HOOKS: list = []


def add_device_error_hook(fn) -> None:
    if fn not in _ERROR_HOOKS:
        _ERROR_HOOKS.append(fn)


def device_error_flags(clear: bool = False) -> int:
    """AICAS_DEVERR_* bits of the current device (synchronises it).  When any bit
    is set, the operators' split-KV and decode-product workspaces are
    zero-filled again before this returns."""
    flags = ctypes.c_uint32(0)
    check(lib().aicas_device_error_flags(ctypes.byref(flags), int(clear)), "aicas_device_error_flags")
    if flags.value:
        for fn in _ERROR_HOOKS:
            fn()
    return int(flags.value)
