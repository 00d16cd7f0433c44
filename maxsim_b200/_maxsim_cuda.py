"""Drop-in replacement for the reference extension module ``maxsim._maxsim_cuda``.

The reference binds two pybind11 classes and a few module functions
(``cpp/maxsim/cuda_extension.cu:3416-3513``).  This module reproduces that
surface -- class names, method names, positional/keyword arguments, default
values, properties and error types -- on top of the C ABI in
``include/maxsim_b200.h`` (ctypes; the GIL is released during each call).

Arrays are accepted like pybind11's ``py::array_t<T, c_style | forcecast>``:
anything NumPy can convert, copied to a C-contiguous array of the right dtype.
"""

from __future__ import annotations

import ctypes

import numpy as np

from maxsim_b200 import _lib
from maxsim_b200._lib import check, lib

__all__ = [
    "CudaPackedDocs",
    "CudaInt4PackedDocs",
    "maxsim_cuda",
    "maxsim_cuda_batch",
    "set_dim128_unrolled_min_avg_tokens",
    "get_dim128_unrolled_min_avg_tokens",
    "set_dim128_qtile_min_packed_bytes",
    "get_dim128_qtile_min_packed_bytes",
    "set_shared_reducer_warps",
    "get_shared_reducer_warps",
    "set_residual_reducer_warps",
    "get_residual_reducer_warps",
    "set_residual_reducer_force_warps",
    "get_residual_reducer_force_warps",
    "get_effective_residual_reducer_warps",
]

# Routing knobs of the reference (cuda_extension.cu:23-74).  They select
# SIMT launch shapes that do not exist in this implementation; the values are
# kept (thread-local where the reference's are) so callers and their tests
# keep working, and ``maxsim_kernel_variant`` reports the reference's rule.
_knobs = {"dim128_unrolled_min_avg_tokens": 256, "dim128_qtile_min_packed_bytes": (1 << 64) - 1}
import threading as _threading

_tls = _threading.local()


def _tl(name, default):
    return getattr(_tls, name, default)


def _f32(a, ndim=None, name="array"):
    arr = np.ascontiguousarray(a, dtype=np.float32)
    return arr


def _u8(a):
    return np.ascontiguousarray(a, dtype=np.uint8)


def _i64(a):
    return np.ascontiguousarray(a, dtype=np.int64)


def _vp(arr):
    return None if arr is None else ctypes.c_void_p(arr.ctypes.data)


def _check_query3(query, dim):
    q = _f32(query)
    if q.ndim != 3:
        raise ValueError("query must have shape [batch, query_tokens, dim]")
    if q.shape[2] != dim:
        raise ValueError("query shape does not match dim")
    return q


def _reducer_opts(reducer, query_weights, temperature, batch, qtok):
    if not isinstance(reducer, str) or reducer not in _lib.REDUCER_IDS:
        raise ValueError("reducer must be one of 'maxsim', 'weighted_maxsim', 'topk2', 'topk4', or 'smoothsim'")
    rid = _lib.REDUCER_IDS[reducer]
    temperature = float(np.float32(temperature))
    if not (temperature > 0.0) or not np.isfinite(temperature):
        raise ValueError("temperature must be finite and > 0")
    weights = None
    rows = 1
    if query_weights is None:
        if rid == 1:
            raise ValueError("query_weights are required for reducer='weighted_maxsim'")
    else:
        if rid != 1:
            raise ValueError("query_weights are only valid for reducer='weighted_maxsim'")
        try:
            weights = np.ascontiguousarray(query_weights, dtype=np.float32)
        except (TypeError, ValueError) as exc:
            raise ValueError("query_weights must be convertible to a float32 array") from exc
        if weights.ndim == 1 and weights.shape[0] == qtok:
            rows = 1
        elif weights.ndim == 2 and weights.shape[1] == qtok and weights.shape[0] in (1, batch):
            rows = weights.shape[0]
        else:
            raise ValueError("query_weights must have shape [query_tokens] or [batch, query_tokens]")
        if weights.size == 0:
            weights = np.zeros(1, np.float32)  # nothing to read; keeps the pointer non-NULL
    return rid, weights, rows, temperature


def _opts(reducer=0, query_mode=0, weights=None, weight_rows=1, temperature=1.0, use_residual=False,
          use_token_scale=False, use_doc_scale=False, scale=1.0, override=None):
    o = _lib.ScoreOpts()
    o.reducer = reducer
    o.query_mode = query_mode
    # host arrays for the synchronous calls; torch CUDA tensors for the *_device calls
    o.weights = None if weights is None else (weights.data_ptr() if hasattr(weights, "data_ptr")
                                              else weights.ctypes.data)
    o.weight_rows = weight_rows
    o.temperature = temperature
    o.use_residual = int(bool(use_residual))
    o.use_token_scale = int(bool(use_token_scale))
    o.use_doc_scale = int(bool(use_doc_scale))
    o.scale = float(scale)
    o.doc_scale_override = None if override is None else (override.data_ptr() if hasattr(override, "data_ptr")
                                                          else override.ctypes.data)
    return o


class _Handle:
    """Owns one ``msb_docs`` handle."""

    _format = None
    _bytes_div = None

    def __init__(self, packed, offsets, dim, scale):
        packed = _u8(packed)
        offsets = _i64(offsets)
        if packed.ndim != 2:
            raise ValueError(f"packed must have shape [num_doc_tokens, dim / {self._bytes_div}]")
        if offsets.ndim != 1:
            raise ValueError("offsets must be a 1-D array")
        dim = int(dim)
        if self._format == _lib.FORMAT_INT4:
            if dim <= 0 or dim % 2 != 0:
                raise ValueError("dim must be positive and divisible by 2")
        elif dim <= 0 or dim % 8 != 0:
            raise ValueError("dim must be positive and divisible by 8")
        if packed.shape[1] != dim // self._bytes_div:
            raise ValueError("packed shape does not match dim")
        if offsets.shape[0] < 2:
            raise ValueError("offsets must contain at least [0, num_doc_tokens]")
        self._h = ctypes.c_void_p()
        self._dim = dim
        check(lib.msb_docs_create(self._format, dim, _vp(packed), packed.shape[0], _vp(offsets),
                                  offsets.shape[0] - 1, ctypes.c_float(scale), ctypes.byref(self._h)))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                lib.msb_docs_destroy(h)
            except Exception:  # pragma: no cover - interpreter shutdown
                pass
            self._h = None

    # -- info ------------------------------------------------------------
    def _info(self):
        info = _lib.DocsInfo()
        check(lib.msb_docs_get_info(self._h, ctypes.byref(info)))
        return info

    @property
    def dim(self):
        return self._dim

    @property
    def num_docs(self):
        return int(self._info().num_docs)

    @property
    def num_tokens(self):
        return int(self._info().num_tokens)

    @property
    def packed_size(self):
        return int(self._info().packed_size)

    @property
    def has_token_scale_vector(self):
        return bool(self._info().has_token_scale)

    @property
    def token_scale_vector_size(self):
        info = self._info()
        return int(info.num_tokens) if info.has_token_scale else 0

    @property
    def resident_bytes(self):
        return int(self._info().resident_bytes)

    @property
    def workspace_bytes(self):
        return int(self._info().workspace_bytes)

    @property
    def device_handle(self):
        """Raw ``msb_docs*`` for the device-pointer entry points."""
        return self._h

    # -- core calls --------------------------------------------------------
    def _score(self, query, opts, candidates=None):
        q = query
        batch, qtok = q.shape[0], q.shape[1]
        if candidates is not None:
            cands = _i64(candidates)
            if cands.ndim != 1:
                raise ValueError("candidate_indices must be a 1-D array")
            n_targets = cands.shape[0]
        else:
            cands = None
            n_targets = self.num_docs
        out = np.empty((batch, n_targets), dtype=np.float32)
        if batch == 0 or n_targets == 0:
            if cands is not None:
                bad = (cands < 0) | (cands >= self.num_docs)
                if bad.any():
                    raise ValueError("candidate_indices entries must be between 0 and num_docs - 1")
            return out
        check(lib.msb_docs_score(self._h, _vp(q), batch, qtok, ctypes.byref(opts), _vp(cands),
                                 0 if cands is None else n_targets, _vp(out)))
        return out

    def _topk(self, query, k, opts):
        k = int(k)
        if k < 1 or k > self.num_docs:
            raise ValueError("k must be between 1 and num_docs")
        batch, qtok = query.shape[0], query.shape[1]
        scores = np.empty((batch, k), dtype=np.float32)
        ids = np.empty((batch, k), dtype=np.int64)
        check(lib.msb_docs_topk(self._h, _vp(query), batch, qtok, k, ctypes.byref(opts), _vp(scores), _vp(ids)))
        return scores, ids

    def _require_int8_dim(self):
        if self._dim != 128:
            raise ValueError("int8 query scoring currently requires dim=128")

    def set_token_scale_vector(self, token_scales):
        ts = _f32(token_scales)
        if ts.ndim != 1 or ts.shape[0] != self.num_tokens:
            raise ValueError("token scale vector must have shape [num_doc_tokens]")
        check(lib.msb_docs_set_token_scales(self._h, _vp(ts), ts.shape[0],
                                            1 if self._format == _lib.FORMAT_INT4 else 0))

    def clear_token_scale_vector(self):
        check(lib.msb_docs_clear_token_scales(self._h))

    # -- device-pointer fast path (used by the SDK batch APIs and bench.py) --
    def topk_batch_device(self, query, k, out_scores, out_ids, *, int8_query=False, stream=None, **kw):
        """Enqueue scan + top-k on device tensors (torch) without synchronising."""
        opts = _opts(query_mode=_lib.QUERY_I8 if int8_query else _lib.QUERY_F32, **kw)
        check(lib.msb_docs_topk_device(self._h, ctypes.c_void_p(query.data_ptr()), query.shape[0], query.shape[1],
                                       int(k), ctypes.byref(opts), ctypes.c_void_p(out_scores.data_ptr()),
                                       ctypes.c_void_p(out_ids.data_ptr()),
                                       None if stream is None else ctypes.c_void_p(stream)))

    def score_batch_device(self, query, out, *, candidates=None, int8_query=False, stream=None, **kw):
        opts = _opts(query_mode=_lib.QUERY_I8 if int8_query else _lib.QUERY_F32, **kw)
        check(lib.msb_docs_score_device(self._h, ctypes.c_void_p(query.data_ptr()), query.shape[0],
                                        query.shape[1], ctypes.byref(opts),
                                        None if candidates is None else ctypes.c_void_p(candidates.data_ptr()),
                                        0 if candidates is None else candidates.shape[0],
                                        ctypes.c_void_p(out.data_ptr()),
                                        None if stream is None else ctypes.c_void_p(stream)))


class CudaPackedDocs(_Handle):
    """Binary sign-code corpus resident on the GPU (reference ``CudaPackedDocs``)."""

    _format = _lib.FORMAT_BINARY
    _bytes_div = 8

    def __init__(self, packed, offsets, dim):
        super().__init__(packed, offsets, dim, 1.0)

    @property
    def has_scale_vector(self):
        return bool(self._info().has_doc_scale)

    @property
    def scale_vector_size(self):
        info = self._info()
        return int(info.num_docs) if info.has_doc_scale else 0

    @property
    def maxsim_kernel_variant(self):
        """The reference's routing label (cuda_extension.cu:2342-2347, :2625-2634)."""
        if self._dim == 128 and self.packed_size >= _knobs["dim128_qtile_min_packed_bytes"]:
            return "dim128_qtile"
        if self._dim != 128:
            return "generic"
        if self.num_docs <= 128:
            return "dim128_unrolled"
        avg = self.num_tokens // max(self.num_docs, 1)
        return "dim128_unrolled" if avg >= _knobs["dim128_unrolled_min_avg_tokens"] else "generic"

    def set_scale_vector(self, scale):
        s = _f32(scale)
        if s.ndim != 1 or s.shape[0] != self.num_docs:
            raise ValueError("scale vector must have shape [num_docs]")
        check(lib.msb_docs_set_doc_scales(self._h, _vp(s), s.shape[0]))

    def clear_scale_vector(self):
        check(lib.msb_docs_clear_doc_scales(self._h))

    def _binary_opts(self, scale, use_scale_vector, use_token_scale, **kw):
        return _opts(use_token_scale=use_token_scale, use_doc_scale=use_scale_vector, scale=float(np.float32(scale)),
                     **kw)

    def maxsim_batch(self, query, scale=1.0, use_scale_vector=False, use_token_scale=False):
        q = _check_query3(query, self._dim)
        return self._score(q, self._binary_opts(scale, use_scale_vector, use_token_scale))

    def _generic(self, query, candidates, reducer, query_weights, temperature, scale, use_scale_vector,
                 use_token_scale, scale_vector_override):
        q = _check_query3(query, self._dim)
        rid, w, rows, temp = _reducer_opts(reducer, query_weights, temperature, q.shape[0], q.shape[1])
        override = None
        if scale_vector_override is not None:
            if use_scale_vector:
                raise ValueError("scale_vector_override and use_scale_vector cannot both be set")
            override = _f32(scale_vector_override)
            if override.ndim != 1 or override.shape[0] != self.num_docs:
                raise ValueError("scale_vector_override must have shape [num_docs]")
        opts = self._binary_opts(scale, use_scale_vector, use_token_scale, reducer=rid, weights=w, weight_rows=rows,
                                 temperature=temp, override=override)
        return self._score(q, opts, candidates)

    def score_batch(self, query, reducer="maxsim", query_weights=None, temperature=1.0, scale=1.0,
                    use_scale_vector=False, use_token_scale=False, scale_vector_override=None):
        return self._generic(query, None, reducer, query_weights, temperature, scale, use_scale_vector,
                             use_token_scale, scale_vector_override)

    def score_candidates_batch(self, query, candidate_indices, reducer="maxsim", query_weights=None,
                               temperature=1.0, scale=1.0, use_scale_vector=False, use_token_scale=False,
                               scale_vector_override=None):
        cands = _i64(candidate_indices)
        if cands.ndim != 1:
            raise ValueError("candidate_indices must be a 1-D array")
        return self._generic(query, cands, reducer, query_weights, temperature, scale, use_scale_vector,
                             use_token_scale, scale_vector_override)

    def topk_batch(self, query, k, scale=1.0, use_scale_vector=False, use_token_scale=False):
        q = _check_query3(query, self._dim)
        return self._topk(q, k, self._binary_opts(scale, use_scale_vector, use_token_scale))

    def topk_lut_batch(self, query, k, scale=1.0, use_scale_vector=False, use_token_scale=False):
        """The reference's byte-LUT variant; the same scan serves both here (exact for integer-valued queries)."""
        if self._dim != 128:
            raise ValueError("topk_lut_batch currently requires dim=128")
        return self.topk_batch(query, k, scale, use_scale_vector, use_token_scale)

    def streaming_topk_batch(self, query, k, scale=1.0, use_scale_vector=False):
        """The reference's lock-based streaming variant; same results via the fused scan + top-k."""
        return self.topk_batch(query, k, scale, use_scale_vector, False)

    def topk_centroid_batch(self, query, weights, k, scale=1.0, use_scale_vector=False, use_token_scale=False):
        q = _check_query3(query, self._dim)
        w = _f32(weights)
        if w.ndim != 1 or w.shape[0] != self._dim:
            raise ValueError("weights must have shape [dim]")
        return self.topk_batch(np.ascontiguousarray(q * w[None, None, :], dtype=np.float32), k, scale,
                               use_scale_vector, use_token_scale)

    def maxsim_batch_int8q(self, query, scale=1.0, use_scale_vector=False, use_token_scale=False):
        self._require_int8_dim()
        q = _check_query3(query, self._dim)
        return self._score(q, self._binary_opts(scale, use_scale_vector, use_token_scale, query_mode=_lib.QUERY_I8))

    def topk_batch_int8q(self, query, k, scale=1.0, use_scale_vector=False, use_token_scale=False):
        self._require_int8_dim()
        q = _check_query3(query, self._dim)
        return self._topk(q, k, self._binary_opts(scale, use_scale_vector, use_token_scale, query_mode=_lib.QUERY_I8))


    # -- sign-bit prefix + int4 residual (two-stream format with no counterpart in the reference) --
    @property
    def has_residual_int4(self):
        return bool(self._info().has_residual)

    def set_residual_int4(self, packed, token_scales):
        """Per-token int4 residual [num_doc_tokens, dim / 2] completing the sign prefix, whose per-token
        reconstruction scale is this handle's token scale vector."""
        p = _u8(packed)
        if p.ndim != 2 or p.shape[0] != self.num_tokens or p.shape[1] != self._dim // 2:
            raise ValueError("residual packed data must have shape [num_doc_tokens, dim / 2]")
        ts = _f32(token_scales)
        if ts.ndim != 1 or ts.shape[0] != self.num_tokens:
            raise ValueError("residual token scale vector must have shape [num_doc_tokens]")
        check(lib.msb_docs_set_residual(self._h, _vp(p), p.shape[0], ctypes.c_float(1.0), _vp(ts)))

    def clear_residual_int4(self):
        check(lib.msb_docs_clear_residual(self._h))

    def _residual(self, query, candidates, reducer, query_weights, temperature):
        q = _check_query3(query, self._dim)
        rid, w, rows, temp = _reducer_opts(reducer, query_weights, temperature, q.shape[0], q.shape[1])
        if not self.has_residual_int4 and q.shape[0] and q.shape[1]:
            raise ValueError("residual int4 data was requested but is not loaded on this CUDA handle")
        return self._score(q, _opts(reducer=rid, weights=w, weight_rows=rows, temperature=temp, use_residual=True),
                           candidates)

    def score_residual_batch(self, query, reducer="maxsim", query_weights=None, temperature=1.0):
        return self._residual(query, None, reducer, query_weights, temperature)

    def score_residual_candidates_batch(self, query, candidate_indices, reducer="maxsim", query_weights=None,
                                        temperature=1.0):
        cands = _i64(candidate_indices)
        if cands.ndim != 1:
            raise ValueError("candidate_indices must be a 1-D array")
        return self._residual(query, cands, reducer, query_weights, temperature)

    def cascade_topk_batch(self, query, k, candidates, reducer="maxsim", query_weights=None, temperature=1.0):
        """Sign-prefix scan -> per-row top-M -> fused residual rescoring -> top-k, on the device."""
        q = _check_query3(query, self._dim)
        rid, w, rows, temp = _reducer_opts(reducer, query_weights, temperature, q.shape[0], q.shape[1])
        k, m = int(k), int(candidates)
        scores = np.empty((q.shape[0], k), dtype=np.float32)
        ids = np.empty((q.shape[0], k), dtype=np.int64)
        opts = _opts(reducer=rid, weights=w, weight_rows=rows, temperature=temp)
        check(lib.msb_docs_cascade_topk(self._h, _vp(q), q.shape[0], q.shape[1], k, m, ctypes.byref(opts),
                                        _vp(scores), _vp(ids)))
        return scores, ids


class CudaInt4PackedDocs(_Handle):
    """int4 (tensor or per-token scale, optional residual stream) corpus on the GPU
    (reference ``CudaInt4PackedDocs``)."""

    _format = _lib.FORMAT_INT4
    _bytes_div = 2

    def __init__(self, packed, offsets, dim, scale):
        scale = float(np.float32(scale))
        if not (scale > 0.0) or not np.isfinite(scale):
            raise ValueError("scale must be finite and > 0")
        super().__init__(packed, offsets, dim, scale)

    @classmethod
    def _for_upload(cls, offsets, num_tokens, dim, scale, flags):
        """A handle whose arrays are allocated but not filled (``msb_docs_create_for_upload``); the
        streaming loader fills them and finishes the upload before any scoring call."""
        scale = float(np.float32(scale))
        if not (scale > 0.0) or not np.isfinite(scale):
            raise ValueError("scale must be finite and > 0")
        offsets = _i64(offsets)
        self = cls.__new__(cls)
        self._h = ctypes.c_void_p()
        self._dim = int(dim)
        check(lib.msb_docs_create_for_upload(cls._format, int(dim), int(num_tokens), _vp(offsets),
                                             offsets.shape[0] - 1, ctypes.c_float(scale), int(flags),
                                             ctypes.byref(self._h)))
        return self

    @property
    def scale(self):
        return float(self._info().scale)

    @property
    def has_residual_int4(self):
        return bool(self._info().has_residual)

    def set_residual_int4(self, packed, scale, token_scales):
        p = _u8(packed)
        if p.ndim != 2 or p.shape[0] != self.num_tokens or p.shape[1] != self._dim // 2:
            raise ValueError("residual packed data must have shape [num_doc_tokens, dim / 2]")
        scale = float(np.float32(scale))
        if not (scale > 0.0) or not np.isfinite(scale):
            raise ValueError("residual scale must be finite and > 0")
        ts = _f32(token_scales)
        if ts.ndim != 1 or ts.shape[0] != self.num_tokens:
            raise ValueError("residual token scale vector must have shape [num_doc_tokens]")
        check(lib.msb_docs_set_residual(self._h, _vp(p), p.shape[0], ctypes.c_float(scale), _vp(ts)))

    def clear_residual_int4(self):
        check(lib.msb_docs_clear_residual(self._h))

    def maxsim_batch(self, query):
        q = _check_query3(query, self._dim)
        return self._score(q, _opts())

    def _generic(self, query, candidates, reducer, query_weights, temperature, residual):
        q = _check_query3(query, self._dim)
        rid, w, rows, temp = _reducer_opts(reducer, query_weights, temperature, q.shape[0], q.shape[1])
        if residual and not self.has_residual_int4 and q.shape[0] and q.shape[1]:
            raise ValueError("residual int4 data was requested but is not loaded on this CUDA handle")
        return self._score(q, _opts(reducer=rid, weights=w, weight_rows=rows, temperature=temp,
                                    use_residual=residual), candidates)

    def score_batch(self, query, reducer="maxsim", query_weights=None, temperature=1.0):
        return self._generic(query, None, reducer, query_weights, temperature, False)

    def score_candidates_batch(self, query, candidate_indices, reducer="maxsim", query_weights=None,
                               temperature=1.0):
        cands = _i64(candidate_indices)
        if cands.ndim != 1:
            raise ValueError("candidate_indices must be a 1-D array")
        return self._generic(query, cands, reducer, query_weights, temperature, False)

    def score_residual_batch(self, query, reducer="maxsim", query_weights=None, temperature=1.0):
        return self._generic(query, None, reducer, query_weights, temperature, True)

    def score_residual_candidates_batch(self, query, candidate_indices, reducer="maxsim", query_weights=None,
                                        temperature=1.0):
        cands = _i64(candidate_indices)
        if cands.ndim != 1:
            raise ValueError("candidate_indices must be a 1-D array")
        return self._generic(query, cands, reducer, query_weights, temperature, True)

    def topk_batch(self, query, k):
        q = _check_query3(query, self._dim)
        return self._topk(q, k, _opts())

    def maxsim_batch_int8q(self, query):
        self._require_int8_dim()
        q = _check_query3(query, self._dim)
        return self._score(q, _opts(query_mode=_lib.QUERY_I8))

    def topk_batch_int8q(self, query, k):
        self._require_int8_dim()
        q = _check_query3(query, self._dim)
        return self._topk(q, k, _opts(query_mode=_lib.QUERY_I8))

    def cascade_topk_batch(self, query, k, candidates, reducer="maxsim", query_weights=None, temperature=1.0):
        """Residual cascade fully on the device (no host round trip between stages)."""
        q = _check_query3(query, self._dim)
        rid, w, rows, temp = _reducer_opts(reducer, query_weights, temperature, q.shape[0], q.shape[1])
        k, m = int(k), int(candidates)
        scores = np.empty((q.shape[0], k), dtype=np.float32)
        ids = np.empty((q.shape[0], k), dtype=np.int64)
        opts = _opts(reducer=rid, weights=w, weight_rows=rows, temperature=temp)
        check(lib.msb_docs_cascade_topk(self._h, _vp(q), q.shape[0], q.shape[1], k, m, ctypes.byref(opts),
                                        _vp(scores), _vp(ids)))
        return scores, ids


def _host_packed_scan(query, packed, offsets, dim, scale, squeeze):
    handle = CudaPackedDocs(packed, offsets, dim)
    out = handle.maxsim_batch(query, scale)
    return out[0] if squeeze else out


def maxsim_cuda(query, packed, offsets, dim, scale=1.0):
    """Single-query binary MaxSim from host arrays (reference :3308-3359)."""
    q = _f32(query)
    if q.ndim != 2:
        raise ValueError("query must have shape [query_tokens, dim]")
    p = _u8(packed)
    if p.ndim != 2:
        raise ValueError("packed must have shape [num_doc_tokens, dim / 8]")
    if int(dim) <= 0 or int(dim) % 8 != 0:
        raise ValueError("dim must be positive and divisible by 8")
    if q.shape[1] != dim or p.shape[1] != dim // 8:
        raise ValueError("query/packed shapes do not match dim")
    return _host_packed_scan(q[None], p, offsets, dim, scale, True)


def maxsim_cuda_batch(query, packed, offsets, dim, scale=1.0):
    """Batched binary MaxSim from host arrays (reference :3361-3412)."""
    q = _f32(query)
    if q.ndim != 3:
        raise ValueError("query must have shape [batch, query_tokens, dim]")
    p = _u8(packed)
    if p.ndim != 2:
        raise ValueError("packed must have shape [num_doc_tokens, dim / 8]")
    if int(dim) <= 0 or int(dim) % 8 != 0:
        raise ValueError("dim must be positive and divisible by 8")
    if q.shape[2] != dim or p.shape[1] != dim // 8:
        raise ValueError("query/packed shapes do not match dim")
    return _host_packed_scan(q, p, offsets, dim, scale, False)


def set_dim128_unrolled_min_avg_tokens(value):
    _knobs["dim128_unrolled_min_avg_tokens"] = int(value)


def get_dim128_unrolled_min_avg_tokens():
    return _knobs["dim128_unrolled_min_avg_tokens"]


def set_dim128_qtile_min_packed_bytes(value):
    _knobs["dim128_qtile_min_packed_bytes"] = int(value)


def get_dim128_qtile_min_packed_bytes():
    return _knobs["dim128_qtile_min_packed_bytes"]


def set_shared_reducer_warps(value):
    if value not in (0, 4, 8):
        raise ValueError("shared reducer warps must be one of 0, 4, or 8")
    _tls.shared = int(value)


def get_shared_reducer_warps():
    return _tl("shared", 4)


def set_residual_reducer_warps(value):
    if value not in (0, 4, 8):
        raise ValueError("residual reducer warps must be one of 0, 4, or 8")
    _tls.residual = int(value)


def get_residual_reducer_warps():
    return _tl("residual", 8)


def set_residual_reducer_force_warps(value):
    if value not in (-1, 0, 4, 8):
        raise ValueError("residual reducer force warps must be one of -1, 0, 4, or 8")
    _tls.force = int(value)


def get_residual_reducer_force_warps():
    return _tl("force", -1)


def get_effective_residual_reducer_warps(query_tokens):
    """Reference launch-shape policy (cuda_extension.cu:58-74), reported for compatibility."""
    if query_tokens <= 0:
        raise ValueError("query tokens must be positive")
    force = get_residual_reducer_force_warps()
    if force >= 0:
        return force
    warps = get_residual_reducer_warps()
    if warps == 8:
        return 8 if query_tokens >= 8 else 4
    return warps if warps <= query_tokens else 0


def _topk_with_options(handle, query, k, reducer="maxsim", query_weights=None, temperature=1.0, scale=1.0,
                       use_scale_vector=False, use_token_scale=False, scale_vector_override=None, residual=False):
    """Scan with any reducer + device top-k in one call (no [B, D] round trip to the host)."""
    q = _check_query3(query, handle.dim)
    rid, w, rows, temp = _reducer_opts(reducer, query_weights, temperature, q.shape[0], q.shape[1])
    override = None if scale_vector_override is None else _f32(scale_vector_override)
    opts = _opts(reducer=rid, weights=w, weight_rows=rows, temperature=temp, use_residual=residual,
                 use_token_scale=use_token_scale, use_doc_scale=use_scale_vector, scale=float(np.float32(scale)),
                 override=override)
    return handle._topk(q, k, opts)
