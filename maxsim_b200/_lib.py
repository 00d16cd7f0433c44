"""ctypes binding of ``libmaxsim_b200.so`` (declarations: ``include/maxsim_b200.h``).

The library is loaded from the package directory.  If it is missing the import
fails loudly -- there is no CPU fallback anywhere in this package.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libmaxsim_b200.so"

MSB_OK = 0
MSB_ERR_INVALID_ARGUMENT = 1
MSB_ERR_CUDA = 2
MSB_ERR_NOT_SUPPORTED = 3
MSB_ERR_INTERNAL = 4

FORMAT_INT4 = 0
FORMAT_BINARY = 1
UPLOAD_TOKEN_SCALES = 1
UPLOAD_RESIDUAL = 2
ARRAY_CODES = 0
ARRAY_TOKEN_SCALES = 1
ARRAY_RESIDUAL_CODES = 2
ARRAY_RESIDUAL_TOKEN_SCALES = 3
QUERY_F32 = 0
QUERY_I8 = 1
REDUCER_IDS = {"maxsim": 0, "weighted_maxsim": 1, "topk2": 2, "topk4": 3, "smoothsim": 4}


class ScoreOpts(ctypes.Structure):
    _fields_ = [
        ("reducer", ctypes.c_int32),
        ("query_mode", ctypes.c_int32),
        ("weights", ctypes.c_void_p),
        ("weight_rows", ctypes.c_int32),
        ("temperature", ctypes.c_float),
        ("use_residual", ctypes.c_int32),
        ("use_token_scale", ctypes.c_int32),
        ("use_doc_scale", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("doc_scale_override", ctypes.c_void_p),
    ]


class DocsInfo(ctypes.Structure):
    _fields_ = [
        ("format", ctypes.c_int32),
        ("dim", ctypes.c_int32),
        ("num_docs", ctypes.c_int64),
        ("num_tokens", ctypes.c_int64),
        ("packed_size", ctypes.c_int64),
        ("scale", ctypes.c_float),
        ("residual_scale", ctypes.c_float),
        ("has_token_scale", ctypes.c_int32),
        ("has_doc_scale", ctypes.c_int32),
        ("has_residual", ctypes.c_int32),
        ("device", ctypes.c_int32),
        ("resident_bytes", ctypes.c_int64),
        ("workspace_bytes", ctypes.c_int64),
    ]


_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float

# name -> (restype, argtypes); every symbol declared in include/maxsim_b200.h.
SIGNATURES = {
    "msb_last_error": (ctypes.c_char_p, []),
    "msb_version": (ctypes.c_int, []),
    "msb_launch_count": (_i64, []),
    "msb_set_option": (ctypes.c_int, [ctypes.c_char_p, _i64]),
    "msb_get_option": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(_i64)]),
    "msb_docs_create": (ctypes.c_int, [_i32, _i32, _vp, _i64, _vp, _i64, _f32, ctypes.POINTER(_vp)]),
    "msb_docs_create_device": (ctypes.c_int, [_i32, _i32, _vp, _i64, _vp, _vp, _i64, _f32, ctypes.POINTER(_vp)]),
    "msb_docs_destroy": (ctypes.c_int, [_vp]),
    "msb_docs_get_info": (ctypes.c_int, [_vp, ctypes.POINTER(DocsInfo)]),
    "msb_docs_set_token_scales": (ctypes.c_int, [_vp, _vp, _i64, _i32]),
    "msb_docs_set_token_scales_device": (ctypes.c_int, [_vp, _vp, _i64]),
    "msb_docs_clear_token_scales": (ctypes.c_int, [_vp]),
    "msb_docs_set_doc_scales": (ctypes.c_int, [_vp, _vp, _i64]),
    "msb_docs_clear_doc_scales": (ctypes.c_int, [_vp]),
    "msb_docs_set_residual": (ctypes.c_int, [_vp, _vp, _i64, _f32, _vp]),
    "msb_docs_clear_residual": (ctypes.c_int, [_vp]),
    "msb_docs_create_for_upload": (ctypes.c_int, [_i32, _i32, _i64, _vp, _i64, _f32, _i32, ctypes.POINTER(_vp)]),
    "msb_docs_upload": (ctypes.c_int, [_vp, _i32, _i64, _vp, _i64, ctypes.POINTER(_i64)]),
    "msb_docs_upload_wait": (ctypes.c_int, [_vp, _i64]),
    "msb_docs_upload_finish": (ctypes.c_int, [_vp, _f32]),
    "msb_pinned_alloc": (ctypes.c_int, [_i64, ctypes.POINTER(_vp)]),
    "msb_pinned_free": (ctypes.c_int, [_vp]),
    "msb_docs_score": (ctypes.c_int, [_vp, _vp, _i32, _i32, ctypes.POINTER(ScoreOpts), _vp, _i64, _vp]),
    "msb_docs_topk": (ctypes.c_int, [_vp, _vp, _i32, _i32, _i32, ctypes.POINTER(ScoreOpts), _vp, _vp]),
    "msb_docs_cascade_topk": (ctypes.c_int, [_vp, _vp, _i32, _i32, _i32, _i32, ctypes.POINTER(ScoreOpts), _vp, _vp]),
    "msb_docs_score_device": (ctypes.c_int, [_vp, _vp, _i32, _i32, ctypes.POINTER(ScoreOpts), _vp, _i64, _vp, _vp]),
    "msb_docs_topk_device": (ctypes.c_int, [_vp, _vp, _i32, _i32, _i32, ctypes.POINTER(ScoreOpts), _vp, _vp, _vp]),
    "msb_docs_topk_device_noalloc": (ctypes.c_int, [_vp, _vp, _i32, _i32, _i32, ctypes.POINTER(ScoreOpts), _vp, _vp,
                                                     _vp]),
    "msb_topk_rows_device": (ctypes.c_int, [_vp, _i64, _i32, _i64, _i32, _vp, _i32, _vp, _vp, _vp]),
    "msb_merge_shard_topk_device": (ctypes.c_int, [_vp, _i32, _i32, _i32, _vp, _vp, _vp, _vp]),
    "msb_quantize_query_int8_device": (ctypes.c_int, [_vp, _i64, _i32, _vp, _vp, _vp]),
    "msb_pack_int4_device": (ctypes.c_int, [_vp, _i64, _i32, _i32, _vp, _vp, ctypes.POINTER(_f32), _vp]),
    "msb_pack_signs_device": (ctypes.c_int, [_vp, _i64, _i32, _vp, _vp, _vp]),
}


class CudaLibraryError(RuntimeError):
    pass


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m maxsim_b200.build` "
            "(maxsim_b200 has no CPU fallback)"
        )
    lib = ctypes.CDLL(str(LIB_PATH), mode=getattr(os, "RTLD_LOCAL", 0))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def check(status: int) -> None:
    """Map a status code to the reference's Python exception types."""
    if status == MSB_OK:
        return
    message = (lib.msb_last_error() or b"").decode(errors="replace")
    if status == MSB_ERR_INVALID_ARGUMENT:
        raise ValueError(message)
    if status == MSB_ERR_NOT_SUPPORTED:
        raise NotImplementedError(message)
    raise RuntimeError(message)


def ptr(array) -> int | None:
    """Data pointer of a NumPy array or torch tensor (None for None)."""
    if array is None:
        return None
    if isinstance(array, np.ndarray):
        return array.ctypes.data
    return array.data_ptr()


def launch_count() -> int:
    return int(lib.msb_launch_count())


def set_engine(value: int) -> None:
    check(lib.msb_set_option(b"engine", int(value)))


def get_engine() -> int:
    out = ctypes.c_int64()
    check(lib.msb_get_option(b"engine", ctypes.byref(out)))
    return int(out.value)


def set_option(name: str, value: int) -> None:
    """Set a runtime knob of the library ("engine", "tc_int8_cache")."""
    check(lib.msb_set_option(name.encode(), int(value)))


def get_option(name: str) -> int:
    out = ctypes.c_int64()
    check(lib.msb_get_option(name.encode(), ctypes.byref(out)))
    return int(out.value)
