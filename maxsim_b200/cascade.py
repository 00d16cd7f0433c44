"""Residual int4 format and the prefix -> residual rescoring cascade.

Public surface of the reference's ``src/maxsim/cascade.py``.  The cascade runs
entirely on the GPU (prefix scan, per-row top-M, fused two-stream rescoring of
each row's candidates, final top-k) in one library call -- the reference copies
the full prefix score matrix to the host and loops over batch rows there.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from maxsim_b200._api import _as_numpy, _effective_device, _normalize_candidate_indices, _normalize_reducer_options
from maxsim_b200.experimental import (
    Int4PackedDocs,
    _pack_nibbles,
    _validate_int4_data_matches_values,
    _validate_int4_packed,
    int4_maxsim,
    int4_to_device,
    pack_int4_symmetric,
    topk_int4_maxsim,
)


@dataclass(frozen=True)
class ResidualInt4PackedDocs:
    prefix_data: object
    prefix_values: np.ndarray | None
    prefix_scale: float
    prefix_token_scale: np.ndarray
    residual_data: object
    residual_values: np.ndarray | None
    residual_scale: float
    residual_token_scale: np.ndarray
    doc_offsets: np.ndarray
    dim: int
    num_docs: int
    device: str = "cpu"

    @property
    def num_tokens(self) -> int:
        return int(self.doc_offsets[-1])

    @property
    def storage_bytes(self) -> int:
        code_bytes = self.num_tokens * self.dim // 2
        p = self.prefix_data.nbytes if isinstance(self.prefix_data, np.ndarray) else code_bytes
        r = self.residual_data.nbytes if isinstance(self.residual_data, np.ndarray) else code_bytes
        return int(p + r + 8 + self.prefix_token_scale.nbytes + self.residual_token_scale.nbytes)


def _reconstruct(values, scale, token_scale):
    return values.astype(np.float32, copy=False) * np.float32(scale) * token_scale[:, np.newaxis]


def pack_residual_int4(doc_embeddings, doc_offsets=None) -> ResidualInt4PackedDocs:
    """Per-token int4 prefix plus per-token int4 of (x - prefix reconstruction)."""
    docs = _as_numpy(doc_embeddings).astype(np.float32, copy=False)
    prefix = pack_int4_symmetric(docs, doc_offsets, scale_granularity="token")
    residual = np.asarray(docs - _reconstruct(prefix.values, prefix.scale, prefix.token_scale), dtype=np.float32)
    second = pack_int4_symmetric(residual, prefix.doc_offsets, scale_granularity="token")
    out = ResidualInt4PackedDocs(
        prefix_data=prefix.data, prefix_values=prefix.values, prefix_scale=prefix.scale,
        prefix_token_scale=prefix.token_scale, residual_data=second.data, residual_values=second.values,
        residual_scale=second.scale, residual_token_scale=second.token_scale, doc_offsets=prefix.doc_offsets,
        dim=prefix.dim, num_docs=prefix.num_docs, device="cpu")
    _validate_residual_packed(out)
    return out


def _prefix_view(packed: ResidualInt4PackedDocs) -> Int4PackedDocs:
    return Int4PackedDocs(data=packed.prefix_data, values=packed.prefix_values, doc_offsets=packed.doc_offsets,
                          dim=packed.dim, num_docs=packed.num_docs, scale=packed.prefix_scale, device=packed.device,
                          token_scale=packed.prefix_token_scale)


def _validate_residual_packed(packed: ResidualInt4PackedDocs, *, verify_packed_values: bool = False) -> None:
    if not isinstance(packed, ResidualInt4PackedDocs):
        raise TypeError("packed must be a ResidualInt4PackedDocs instance")
    if packed.device == "cuda" and getattr(packed, "_msb_validated", False):
        return  # a resident corpus is immutable once validated: no O(N) host checks per call
    prefix = _prefix_view(packed)
    _validate_int4_packed(prefix)
    if verify_packed_values:
        _validate_int4_data_matches_values(prefix)
    if packed.prefix_token_scale is None:
        raise ValueError("prefix_token_scale must have shape [num_doc_tokens]")
    if packed.device == "cpu":
        rd, rv = packed.residual_data, packed.residual_values
        if not isinstance(rd, np.ndarray):
            raise ValueError("CPU residual_data must be a NumPy array")
        if rd.dtype != np.uint8:
            raise ValueError("CPU residual_data must have dtype uint8")
        if rd.shape != (packed.num_tokens, packed.dim // 2):
            raise ValueError("residual_data must have shape [num_doc_tokens, dim / 2]")
        if not isinstance(rv, np.ndarray):
            raise ValueError("CPU residual_values must be a NumPy array")
        if rv.shape != (packed.num_tokens, packed.dim):
            raise ValueError("residual_values must have shape [num_doc_tokens, dim]")
        if rv.dtype != np.int8:
            raise ValueError("residual_values must have dtype int8")
        if np.any(rv < -7) or np.any(rv > 7):
            raise ValueError("residual_values must be symmetric int4 values in [-7, 7]")
        if verify_packed_values and not np.array_equal(rd, _pack_nibbles(rv)):
            raise ValueError("residual_data does not encode residual_values")
    elif packed.device == "cuda":
        if packed.residual_values is not None:
            raise ValueError("CUDA residual_values must be None")
        if packed.prefix_data is not packed.residual_data:
            raise ValueError("CUDA prefix_data and residual_data must share one handle")
        handle = packed.prefix_data
        for name, expected in (("dim", packed.dim), ("num_docs", packed.num_docs), ("num_tokens", packed.num_tokens)):
            actual = getattr(handle, name, None)
            if actual is None or int(actual) != int(expected):
                raise ValueError(f"CUDA residual handle {name} does not match metadata")
        if getattr(handle, "has_token_scale_vector", None) is not True:
            raise ValueError("CUDA residual handle is missing prefix token scales")
        if getattr(handle, "has_residual_int4", None) is not True:
            raise ValueError("CUDA residual handle is missing residual int4 data")
    else:
        raise ValueError("device must be 'cpu' or 'cuda'")
    try:
        rs = float(packed.residual_scale)
    except (TypeError, ValueError) as exc:
        raise ValueError("residual_scale must be a finite scalar > 0") from exc
    if not np.isfinite(rs) or rs <= 0.0:
        raise ValueError("residual_scale must be a finite scalar > 0")
    rts = packed.residual_token_scale
    if not isinstance(rts, np.ndarray) or rts.ndim != 1 or rts.shape[0] != packed.num_tokens:
        raise ValueError("residual_token_scale must have shape [num_doc_tokens]")
    if rts.dtype != np.float32:
        raise ValueError("residual_token_scale must have dtype float32")
    if not np.all(np.isfinite(rts)) or np.any(rts <= 0.0):
        raise ValueError("residual_token_scale values must be finite and > 0")


def residual_int4_to_device(packed: ResidualInt4PackedDocs, device: str = "cuda") -> ResidualInt4PackedDocs:
    if device != "cuda":
        raise ValueError("device must be 'cuda'")
    _validate_residual_packed(packed, verify_packed_values=True)
    if packed.device == "cuda":
        return packed
    prefix = int4_to_device(_prefix_view(packed))
    prefix.data.set_residual_int4(np.ascontiguousarray(packed.residual_data, dtype=np.uint8),
                                  float(packed.residual_scale),
                                  np.ascontiguousarray(packed.residual_token_scale, dtype=np.float32))
    resident = ResidualInt4PackedDocs(
        prefix_data=prefix.data, prefix_values=None, prefix_scale=prefix.scale, prefix_token_scale=prefix.token_scale,
        residual_data=prefix.data, residual_values=None, residual_scale=packed.residual_scale,
        residual_token_scale=packed.residual_token_scale.copy(), doc_offsets=packed.doc_offsets.copy(),
        dim=packed.dim, num_docs=packed.num_docs, device="cuda")
    _validate_residual_packed(resident)
    object.__setattr__(resident, "_msb_validated", True)
    return resident


def _normalize_query(query_tokens, dim: int):
    query = _as_numpy(query_tokens).astype(np.float32, copy=False)
    if query.ndim == 1:
        batches, squeeze = query[np.newaxis, np.newaxis, :], True
    elif query.ndim == 2:
        batches, squeeze = query[np.newaxis], True
    elif query.ndim == 3:
        batches, squeeze = query, False
    else:
        raise ValueError("query_tokens must have shape [dim], [query_tokens, dim], or [batch, query_tokens, dim]")
    if batches.shape[2] != dim:
        raise ValueError(f"query dim={batches.shape[2]} does not match packed dim={dim}")
    if not np.all(np.isfinite(batches)):
        raise ValueError("query_tokens must contain only finite values")
    return np.ascontiguousarray(batches, dtype=np.float32), squeeze


def _resident(packed: ResidualInt4PackedDocs, device: str) -> ResidualInt4PackedDocs:
    _validate_residual_packed(packed)
    _effective_device(device, packed)
    return packed if packed.device == "cuda" else residual_int4_to_device(packed)


def prefix_score(query_tokens, packed: ResidualInt4PackedDocs, *, device: str = "auto", reducer: str = "maxsim",
                 query_weights=None, temperature: float = 1.0, candidate_indices=None) -> np.ndarray:
    _validate_residual_packed(packed)
    batches, squeeze = _normalize_query(query_tokens, packed.dim)
    resident = _resident(packed, device)
    return int4_maxsim(batches[0] if squeeze else batches, _prefix_view(resident), device=device, reducer=reducer,
                       query_weights=query_weights, temperature=temperature, candidate_indices=candidate_indices)


def prefix_topk(query_tokens, packed: ResidualInt4PackedDocs, k: int, *, device: str = "auto",
                reducer: str = "maxsim", query_weights=None, temperature: float = 1.0):
    _validate_residual_packed(packed)
    if not isinstance(k, (int, np.integer)) or isinstance(k, (bool, np.bool_)):
        raise ValueError("k must be an integer")
    if k < 1 or k > packed.num_docs:
        raise ValueError("k must satisfy 1 <= k <= num_docs")
    batches, squeeze = _normalize_query(query_tokens, packed.dim)
    resident = _resident(packed, device)
    return topk_int4_maxsim(batches[0] if squeeze else batches, _prefix_view(resident), k, device=device,
                            reducer=reducer, query_weights=query_weights, temperature=temperature)


def residual_score(query_tokens, packed: ResidualInt4PackedDocs, *, device: str = "auto", reducer: str = "maxsim",
                   query_weights=None, temperature: float = 1.0, candidate_indices=None) -> np.ndarray:
    """Fused ``dot(q,p)*ps*pts + dot(q,r)*rs*rts`` scores, any reducer, on the GPU."""
    _validate_residual_packed(packed)
    if device not in {"auto", "cpu", "cuda"}:
        raise ValueError("device must be 'auto', 'cpu', or 'cuda'")
    resident = _resident(packed, device)
    batches, squeeze = _normalize_query(query_tokens, packed.dim)
    reducer_value, weights, temperature_value = _normalize_reducer_options(
        reducer, query_weights, temperature, batch=batches.shape[0], query_tokens=batches.shape[1])
    candidates = _normalize_candidate_indices(candidate_indices, packed.num_docs)
    num_targets = packed.num_docs if candidates is None else int(candidates.shape[0])
    if batches.shape[0] == 0 or num_targets == 0:
        out = np.empty((batches.shape[0], num_targets), dtype=np.float32)
        return out[0] if squeeze else out
    if batches.shape[1] == 0:
        out = np.zeros((batches.shape[0], num_targets), dtype=np.float32)
        return out[0] if squeeze else out
    handle = resident.prefix_data
    if candidates is None:
        out = handle.score_residual_batch(batches, reducer_value, weights, float(temperature_value))
    else:
        out = handle.score_residual_candidates_batch(batches, candidates, reducer_value, weights,
                                                     float(temperature_value))
    return out[0] if squeeze else out


def _stable_topk(scores: np.ndarray, k: int):
    """Score descending, lower index first on ties (host helper for host-resident score matrices)."""
    values = np.asarray(scores, dtype=np.float32)
    if values.ndim == 1:
        order = np.lexsort((np.arange(values.shape[0]), -values))[:k].astype(np.int64)
        return values[order], order
    if values.ndim != 2:
        raise ValueError("scores must be one- or two-dimensional")
    if values.shape[0] == 0:
        return np.empty((0, k), np.float32), np.empty((0, k), np.int64)
    idx = np.stack([np.lexsort((np.arange(r.shape[0]), -r))[:k] for r in values]).astype(np.int64)
    return np.take_along_axis(values, idx, axis=1), idx


def cascade_topk(query_tokens, packed: ResidualInt4PackedDocs, k: int, *, candidates: int, device: str = "auto",
                 reducer: str = "maxsim", query_weights=None, temperature: float = 1.0):
    """Prefix scan -> per-row top-``candidates`` -> fused residual rescoring -> top-``k``, on the GPU."""
    _validate_residual_packed(packed)
    if device not in {"auto", "cpu", "cuda"}:
        raise ValueError("device must be 'auto', 'cpu', or 'cuda'")
    if not isinstance(k, (int, np.integer)) or isinstance(k, (bool, np.bool_)):
        raise ValueError("k must be an integer")
    if not isinstance(candidates, (int, np.integer)) or isinstance(candidates, (bool, np.bool_)):
        raise ValueError("candidates must be an integer")
    if k < 1 or k > candidates or candidates > packed.num_docs:
        raise ValueError("cascade sizes must satisfy 1 <= k <= candidates <= num_docs")
    resident = _resident(packed, device)
    batches, squeeze = _normalize_query(query_tokens, packed.dim)
    _, weights, temperature_value = _normalize_reducer_options(
        reducer, query_weights, temperature, batch=batches.shape[0], query_tokens=batches.shape[1])
    if batches.shape[0] == 0:
        return np.empty((0, k), np.float32), np.empty((0, k), np.int64)
    scores, ids = resident.prefix_data.cascade_topk_batch(batches, int(k), int(candidates), reducer, weights,
                                                          temperature_value)
    return (scores[0], ids[0]) if squeeze else (scores, ids)


# ---------------------------------------------------------------------------
# Binary-prefix cascade: sign bits scaled by a per-token reconstruction scale,
# plus a per-token int4 residual.  The reference's residual cascade uses an int4
# prefix only; this two-stream format is the benchmark's binary-prefix variant
# (16 B + 4 B per token for the prefix scan, 32 B + 4 B more for rescoring).
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class BinaryResidualPackedDocs:
    prefix_data: object                 # sign bits uint8 [N, dim/8] (bit i of byte i/8, x >= 0 -> 1) or a handle
    prefix_token_scale: np.ndarray      # per-token mean |x|: the sign reconstruction scale
    residual_data: object | None        # int4 [N, dim/2] of x - mean|x| * sign(x)
    residual_values: np.ndarray | None
    residual_token_scale: np.ndarray
    doc_offsets: np.ndarray
    dim: int
    num_docs: int
    device: str = "cpu"

    @property
    def num_tokens(self) -> int:
        return int(self.doc_offsets[-1])

    @property
    def storage_bytes(self) -> int:
        n = self.num_tokens
        return int(n * self.dim // 8 + n * self.dim // 2 + self.prefix_token_scale.nbytes +
                   self.residual_token_scale.nbytes)


def pack_binary_residual_int4(doc_embeddings, doc_offsets=None) -> BinaryResidualPackedDocs:
    """Sign bits with per-token mean |x| reconstruction scale, and the per-token int4 residual."""
    from maxsim_b200._api import _mean_abs, _normalize_offsets, _sign_bits

    x = _as_numpy(doc_embeddings).astype(np.float32, copy=False)
    if x.ndim != 2:
        raise ValueError("doc_embeddings must have shape [num_doc_tokens, dim]")
    if x.shape[1] % 8 != 0:
        raise ValueError("dim must be divisible by 8")
    offsets = _normalize_offsets(doc_offsets, x.shape[0])
    ps = _mean_abs(x)
    signs = np.where(x >= 0, np.float32(1.0), np.float32(-1.0))
    residual = (x - ps[:, np.newaxis] * signs).astype(np.float32)
    rpk = pack_int4_symmetric(residual, offsets, scale_granularity="token")
    return BinaryResidualPackedDocs(prefix_data=_sign_bits(x), prefix_token_scale=ps, residual_data=rpk.data,
                                    residual_values=rpk.values, residual_token_scale=rpk.token_scale,
                                    doc_offsets=offsets, dim=int(x.shape[1]), num_docs=int(offsets.shape[0] - 1))


def binary_residual_to_device(packed: BinaryResidualPackedDocs, device: str = "cuda") -> BinaryResidualPackedDocs:
    """Upload both streams to one resident binary handle."""
    if device != "cuda":
        raise ValueError("device must be 'cuda'")
    if packed.device == "cuda":
        return packed
    from maxsim_b200 import _maxsim_cuda

    handle = _maxsim_cuda.CudaPackedDocs(np.ascontiguousarray(packed.prefix_data, dtype=np.uint8),
                                         np.ascontiguousarray(packed.doc_offsets, dtype=np.int64), packed.dim)
    handle.set_token_scale_vector(np.ascontiguousarray(packed.prefix_token_scale, dtype=np.float32))
    handle.set_residual_int4(np.ascontiguousarray(packed.residual_data, dtype=np.uint8),
                             np.ascontiguousarray(packed.residual_token_scale, dtype=np.float32))
    return BinaryResidualPackedDocs(prefix_data=handle, prefix_token_scale=packed.prefix_token_scale,
                                    residual_data=None, residual_values=None,
                                    residual_token_scale=packed.residual_token_scale,
                                    doc_offsets=packed.doc_offsets.copy(), dim=packed.dim, num_docs=packed.num_docs,
                                    device="cuda")


def _binary_resident(packed: BinaryResidualPackedDocs, device) -> BinaryResidualPackedDocs:
    if not isinstance(packed, BinaryResidualPackedDocs):
        raise TypeError("packed must be a BinaryResidualPackedDocs instance")
    _effective_device(device, packed)
    return packed if packed.device == "cuda" else binary_residual_to_device(packed)


def binary_prefix_score(query_tokens, packed: BinaryResidualPackedDocs, *, device: str = "auto",
                        reducer: str = "maxsim", query_weights=None, temperature: float = 1.0,
                        candidate_indices=None) -> np.ndarray:
    """Scores of the sign prefix alone (sign dot times the per-token reconstruction scale)."""
    resident = _binary_resident(packed, device)
    q, squeeze = _normalize_query(query_tokens, packed.dim)
    rv, w, t = _normalize_reducer_options(reducer, query_weights, temperature, batch=q.shape[0],
                                          query_tokens=q.shape[1])
    cands = _normalize_candidate_indices(candidate_indices, packed.num_docs)
    h = resident.prefix_data
    out = (h.score_batch(q, rv, w, t, 1.0, False, True) if cands is None
           else h.score_candidates_batch(q, cands, rv, w, t, 1.0, False, True))
    return out[0] if squeeze else out


def binary_residual_score(query_tokens, packed: BinaryResidualPackedDocs, *, device: str = "auto",
                          reducer: str = "maxsim", query_weights=None, temperature: float = 1.0,
                          candidate_indices=None) -> np.ndarray:
    """Fused two-stream scores: (sign . q) * prefix scale + (residual . q) * residual scale, then the reducer."""
    resident = _binary_resident(packed, device)
    q, squeeze = _normalize_query(query_tokens, packed.dim)
    rv, w, t = _normalize_reducer_options(reducer, query_weights, temperature, batch=q.shape[0],
                                          query_tokens=q.shape[1])
    cands = _normalize_candidate_indices(candidate_indices, packed.num_docs)
    h = resident.prefix_data
    out = (h.score_residual_batch(q, rv, w, t) if cands is None
           else h.score_residual_candidates_batch(q, cands, rv, w, t))
    return out[0] if squeeze else out


def binary_cascade_topk(query_tokens, packed: BinaryResidualPackedDocs, k: int, *, candidates: int,
                        device: str = "auto", reducer: str = "maxsim", query_weights=None,
                        temperature: float = 1.0):
    """Sign-prefix scan -> per-query top-M -> fused residual rescoring -> top-k, in one device call."""
    resident = _binary_resident(packed, device)
    q, squeeze = _normalize_query(query_tokens, packed.dim)
    if not 1 <= int(k) <= int(candidates) <= packed.num_docs:
        raise ValueError("cascade sizes must satisfy 1 <= k <= candidates <= num_docs")
    rv, w, t = _normalize_reducer_options(reducer, query_weights, temperature, batch=q.shape[0],
                                          query_tokens=q.shape[1])
    s, i = resident.prefix_data.cascade_topk_batch(q, int(k), int(candidates), rv, w, t)
    return (s[0], i[0]) if squeeze else (s, i)
