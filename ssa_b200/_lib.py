"""ctypes binding of libssa_sm100a.so (the C ABI in include/ssa_b200.h).

The shared object is built in-tree by ``ssa_b200/build.py``.  There is no
fallback: if the library is missing or cannot be loaded, every call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libssa_sm100a.so")

# ssa_dtype / ssa_index_dtype / ssa_status (include/ssa_b200.h)
SSA_F32, SSA_BF16, SSA_F16 = 0, 1, 2
SSA_I32, SSA_I64 = 0, 1
SSA_DEVICE_INDEX_OOB = 0x1
SSA_DEVICE_BAD_CODE = 0x2
SSA_DEVICE_BAD_INDEX = 0x4
SSA_DEVICE_INDEX_FULL = 0x8
SSA_DEVICE_TIMEOUT = 0x100
STATUS_NAMES = {0: "SSA_OK", 1: "SSA_ERR_INVALID_ARG", 2: "SSA_ERR_UNSUPPORTED", 3: "SSA_ERR_WORKSPACE",
                4: "SSA_ERR_ALIGNMENT", 5: "SSA_ERR_CUDA", 6: "SSA_ERR_DEVICE"}

_c_i32 = ctypes.c_int32
_c_i64 = ctypes.c_int64
_vp = ctypes.c_void_p


class SsaRouteArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _c_i32), ("n", _c_i32), ("n_q", _c_i32), ("q_offset", _c_i32),
        ("h_q", _c_i32), ("h_kv", _c_i32), ("d", _c_i32), ("d_s", _c_i32),
        ("n_codes", _c_i32), ("a", _c_i32), ("b", _c_i32), ("top_k", _c_i32),
        ("causal", _c_i32), ("temperature", ctypes.c_float),
        ("dtype", _c_i32), ("w_dtype", _c_i32), ("codebook_heads", _c_i32),
        ("q", _vp), ("q_stride_b", _c_i64), ("q_stride_n", _c_i64), ("q_stride_h", _c_i64),
        ("k", _vp), ("k_stride_b", _c_i64), ("k_stride_n", _c_i64), ("k_stride_h", _c_i64),
        ("w_qr", _vp), ("w_kr", _vp), ("codebook", _vp),
        ("indices", _vp), ("index_dtype", _c_i32),
        ("q_codes", _vp), ("k_codes", _vp), ("cand_counts", _vp), ("status", _vp),
    ]


class SsaAttnArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _c_i32), ("n_q", _c_i32), ("n", _c_i32), ("q_offset", _c_i32),
        ("h_q", _c_i32), ("h_kv", _c_i32), ("d", _c_i32), ("top_k", _c_i32),
        ("causal", _c_i32), ("scale", ctypes.c_float), ("dtype", _c_i32),
        ("q", _vp), ("q_stride_b", _c_i64), ("q_stride_n", _c_i64), ("q_stride_h", _c_i64),
        ("k", _vp), ("k_stride_b", _c_i64), ("k_stride_n", _c_i64), ("k_stride_h", _c_i64),
        ("v", _vp), ("v_stride_b", _c_i64), ("v_stride_n", _c_i64), ("v_stride_h", _c_i64),
        ("indices", _vp), ("index_dtype", _c_i32),
        ("idx_stride_b", _c_i64), ("idx_stride_n", _c_i64), ("idx_stride_h", _c_i64),
        ("out", _vp), ("out_stride_b", _c_i64), ("out_stride_n", _c_i64), ("out_stride_h", _c_i64),
        ("status", _vp),
    ]


class SsaRopeArgs(ctypes.Structure):
    _fields_ = [
        ("cos", _vp), ("sin", _vp), ("table_stride_b", _c_i64), ("table_stride_n", _c_i64),
        ("q_out", _vp), ("q_out_stride_b", _c_i64), ("q_out_stride_n", _c_i64), ("q_out_stride_h", _c_i64),
        ("k_out", _vp), ("k_out_stride_b", _c_i64), ("k_out_stride_n", _c_i64), ("k_out_stride_h", _c_i64),
    ]


SSA_MAX_SEGMENTS = 8


class SsaQuerySegments(ctypes.Structure):
    _fields_ = [("count", _c_i32), ("rows", _c_i32 * SSA_MAX_SEGMENTS), ("positions", _c_i32 * SSA_MAX_SEGMENTS)]


class SsaDecodeIndex(ctypes.Structure):
    _fields_ = [
        ("bucket_start", _vp), ("bucket_end", _vp), ("bucket_keys", _vp), ("bucket_codes", _vp),
        ("entry_capacity", _c_i64), ("slack", _c_i32), ("min_free", _vp), ("k_codes_stride_b", _c_i64),
    ]


# exported symbol -> (restype, argtypes)
SIGNATURES = {
    "ssa_decode_index_capacity": (_c_i64, [_c_i32, _c_i32, _c_i32, _c_i32]),
    "ssa_decode_index_build": (ctypes.c_int, [ctypes.POINTER(SsaRouteArgs), ctypes.POINTER(SsaDecodeIndex), _vp,
                                              ctypes.c_size_t, _vp]),
    "ssa_decode_index_append": (ctypes.c_int, [ctypes.POINTER(SsaRouteArgs), ctypes.POINTER(SsaDecodeIndex),
                                               _c_i32, _c_i32, _vp]),
    "ssa_decode_route": (ctypes.c_int, [ctypes.POINTER(SsaRouteArgs), ctypes.POINTER(SsaDecodeIndex), _vp,
                                        ctypes.c_size_t, _vp]),
    "ssa_route_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(SsaRouteArgs)]),
    "ssa_route": (ctypes.c_int, [ctypes.POINTER(SsaRouteArgs), _vp, ctypes.c_size_t, _vp]),
    "ssa_code_assign": (ctypes.c_int, [ctypes.POINTER(SsaRouteArgs), _vp, ctypes.c_size_t, _vp]),
    "ssa_sparse_attn": (ctypes.c_int, [ctypes.POINTER(SsaAttnArgs), _vp]),
    "ssa_select_from_scores": (ctypes.c_int, [_vp, _c_i64, _c_i32, _c_i32, _vp, _vp]),
    "ssa_build_index": (ctypes.c_int, [ctypes.POINTER(SsaRouteArgs), _vp, _vp, _vp, _vp,
                                       ctypes.c_size_t, _vp]),
    "ssa_build_index_noalloc": (ctypes.c_int, [ctypes.POINTER(SsaRouteArgs), _vp, _vp, _vp, _vp]),
    "ssa_select_candidates": (ctypes.c_int, [ctypes.POINTER(SsaRouteArgs), _vp, ctypes.c_size_t, _vp]),
    "ssa_route_with_key_codes": (ctypes.c_int, [ctypes.POINTER(SsaRouteArgs), _vp, ctypes.c_size_t, _vp]),
    "ssa_route_with_index": (ctypes.c_int, [ctypes.POINTER(SsaRouteArgs), _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "ssa_route_rope": (ctypes.c_int, [ctypes.POINTER(SsaRouteArgs), ctypes.POINTER(SsaRopeArgs), _vp,
                                      ctypes.c_size_t, _vp]),
    "ssa_sparse_attn_backward": (ctypes.c_int, [ctypes.POINTER(SsaAttnArgs), _vp, _vp, _vp, _vp, _vp]),
    "ssa_l2_read_probe": (ctypes.c_int, [_vp, ctypes.c_size_t, _c_i32, _vp, _vp]),
    "ssa_route_with_index_segments": (ctypes.c_int, [ctypes.POINTER(SsaRouteArgs), ctypes.POINTER(SsaQuerySegments),
                                                     _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "ssa_sparse_attn_segments": (ctypes.c_int, [ctypes.POINTER(SsaAttnArgs), ctypes.POINTER(SsaQuerySegments), _vp]),
    "ssa_query_codes": (ctypes.c_int, [ctypes.POINTER(SsaRouteArgs), _vp, ctypes.c_size_t, _vp]),
    "ssa_select_candidates_segments": (ctypes.c_int, [ctypes.POINTER(SsaRouteArgs),
                                                      ctypes.POINTER(SsaQuerySegments), _vp, _vp, _vp,
                                                      ctypes.c_size_t, _vp]),
    "ssa_status_str": (ctypes.c_char_p, [ctypes.c_int]),
    "ssa_last_error": (ctypes.c_char_p, []),
}

_lib = None
_lock = threading.Lock()


class SSAError(RuntimeError):
    """A non-OK ssa_status returned by the library."""

    def __init__(self, fn: str, code: int, detail: str):
        self.code = code
        super().__init__(f"{fn} failed: {STATUS_NAMES.get(code, code)} ({detail})")


def lib() -> ctypes.CDLL:
    """Load libssa_sm100a.so once (raises if it is absent: there is no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m ssa_b200.build` "
                    "(nvcc, sm_100a). ssa_b200 has no CPU or non-CUDA fallback.")
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(fn: str, code: int) -> None:
    if code != 0:
        detail = lib().ssa_last_error().decode(errors="replace")
        raise SSAError(fn, code, detail)
