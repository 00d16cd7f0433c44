"""int4 formats (tensor and per-token scale) and their GPU scoring API.

Public surface of the reference's int4 part of ``src/maxsim/experimental.py``
(``Int4PackedDocs``, ``pack_int4_symmetric``, ``int4_to_device``,
``int4_maxsim``, ``int4_maxsim_int8q``, ``topk_int4_maxsim``).  The
centroid (``binary_q40``) and ternary experiments of that module are not part
of this package.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from maxsim_b200._api import (
    _as_batches,
    _as_numpy,
    _effective_device,
    _normalize_candidate_indices,
    _normalize_offsets,
    _normalize_reducer_options,
)


@dataclass(frozen=True)
class Int4PackedDocs:
    """int4 corpus: ``data`` uint8 ``[N, dim/2]`` (even dim in the low nibble) or a CUDA handle."""

    data: object
    values: np.ndarray | None
    doc_offsets: np.ndarray
    dim: int
    num_docs: int
    scale: float
    device: str = "cpu"
    token_scale: np.ndarray | None = None

    @property
    def storage_bytes(self) -> int:
        if isinstance(self.data, np.ndarray):
            packed_bytes = int(self.data.nbytes)
        else:
            packed_bytes = int(getattr(self.data, "packed_size", 0))
        token_bytes = 0 if self.token_scale is None else int(self.token_scale.nbytes)
        return packed_bytes + 4 + token_bytes


def _pack_nibbles(values: np.ndarray) -> np.ndarray:
    v = values.astype(np.int16)
    return np.ascontiguousarray(((v[:, 0::2] & 0x0F) | ((v[:, 1::2] & 0x0F) << 4)).astype(np.uint8))


def pack_int4_symmetric(doc_embeddings, doc_offsets=None, *, scale: float | None = None,
                        scale_granularity: str = "tensor") -> Int4PackedDocs:
    """Symmetric int4 codes in [-7, 7] with a tensor or per-token scale."""
    docs = _as_numpy(doc_embeddings).astype(np.float32, copy=False)
    if docs.ndim != 2:
        raise ValueError("doc_embeddings must have shape [num_doc_tokens, dim]")
    if docs.shape[1] <= 0:
        raise ValueError("dim must be positive")
    if docs.shape[1] % 2 != 0:
        raise ValueError("dim must be divisible by 2 for int4 packing")
    if docs.shape[1] % 8 != 0:
        raise ValueError("dim must be divisible by 8")
    if not np.all(np.isfinite(docs)):
        raise ValueError("doc_embeddings must contain only finite values")
    if scale_granularity not in {"tensor", "token"}:
        raise ValueError("scale_granularity must be 'tensor' or 'token'")
    token_scale = None
    if scale_granularity == "token":
        if scale is not None:
            raise ValueError("scale cannot be provided when scale_granularity='token'")
        token_scale = np.max(np.abs(docs), axis=1).astype(np.float32) / np.float32(7.0) if docs.shape[0] else \
            np.zeros(0, np.float32)
        token_scale[token_scale == 0.0] = 1.0
        scale_value = 1.0
        values = np.clip(np.rint(docs / token_scale[:, np.newaxis]), -7, 7).astype(np.int8)
    else:
        if scale is None:
            max_abs = float(np.max(np.abs(docs))) if docs.size else 0.0
            scale_value = 1.0 if max_abs == 0.0 else max_abs / 7.0
        else:
            scale_value = float(scale)
            if not np.isfinite(scale_value) or scale_value <= 0.0:
                raise ValueError("scale must be finite and > 0")
        values = np.clip(np.rint(docs / np.float32(scale_value)), -7, 7).astype(np.int8)
    offsets = _normalize_offsets(doc_offsets, docs.shape[0])
    return Int4PackedDocs(data=_pack_nibbles(values), values=np.ascontiguousarray(values), doc_offsets=offsets,
                          dim=int(docs.shape[1]), num_docs=int(offsets.shape[0] - 1), scale=scale_value,
                          device="cpu", token_scale=token_scale)


def _validate_int4_packed(packed: Int4PackedDocs) -> None:
    if not isinstance(packed, Int4PackedDocs):
        raise TypeError("packed must be an Int4PackedDocs instance")
    if packed.device == "cuda" and getattr(packed, "_msb_validated", False):
        return  # resident corpora are immutable once validated; skip the O(N) host checks per call
    if not isinstance(packed.dim, (int, np.integer)) or packed.dim <= 0 or packed.dim % 8 != 0:
        raise ValueError("packed.dim must be positive and divisible by 8")
    if not isinstance(packed.num_docs, (int, np.integer)) or packed.num_docs < 0:
        raise ValueError("packed.num_docs must be a nonnegative integer")
    if packed.values is not None:
        if not isinstance(packed.values, np.ndarray) or packed.values.ndim != 2 or packed.values.shape[1] != packed.dim:
            raise ValueError("packed.values must have shape [num_doc_tokens, dim]")
        if packed.values.dtype != np.int8:
            raise ValueError("packed.values must have dtype int8")
        if np.any(packed.values < -7) or np.any(packed.values > 7):
            raise ValueError("packed.values must be symmetric int4 values in [-7, 7]")
    if packed.device == "cpu":
        if packed.values is None:
            raise ValueError("CPU Int4PackedDocs must include values")
        if (not isinstance(packed.data, np.ndarray) or packed.data.dtype != np.uint8 or packed.data.ndim != 2
                or packed.data.shape != (packed.values.shape[0], packed.dim // 2)):
            raise ValueError("packed.data must have shape [num_doc_tokens, dim / 2]")
    elif packed.device != "cuda":
        raise ValueError("packed.device must be 'cpu' or 'cuda'")
    offsets = packed.doc_offsets
    if not isinstance(offsets, np.ndarray) or offsets.ndim != 1 or offsets.shape[0] != packed.num_docs + 1:
        raise ValueError("packed.doc_offsets must have shape [num_docs + 1]")
    if not np.issubdtype(offsets.dtype, np.integer):
        raise ValueError("packed.doc_offsets must contain integers")
    num_tokens = int(packed.values.shape[0]) if packed.values is not None else int(offsets[-1])
    if int(offsets[0]) != 0 or int(offsets[-1]) != num_tokens:
        raise ValueError("packed.doc_offsets must span all document tokens")
    if np.any(offsets[1:] < offsets[:-1]):
        raise ValueError("packed.doc_offsets must be monotonically nondecreasing")
    try:
        arr = np.asarray(packed.scale)
        if arr.ndim != 0:
            raise ValueError
        scale_value = float(arr)
    except (TypeError, ValueError) as exc:
        raise ValueError("packed.scale must be a finite scalar > 0") from exc
    if not np.isfinite(scale_value) or scale_value <= 0.0:
        raise ValueError("packed.scale must be a finite scalar > 0")
    ts = packed.token_scale
    if ts is not None:
        if not isinstance(ts, np.ndarray) or ts.ndim != 1 or ts.shape[0] != num_tokens:
            raise ValueError("packed.token_scale must have shape [num_doc_tokens]")
        if ts.dtype != np.float32:
            raise ValueError("packed.token_scale must have dtype float32")
        if not np.all(np.isfinite(ts)) or np.any(ts <= 0.0):
            raise ValueError("packed.token_scale values must be finite and > 0")
    if packed.device == "cuda":
        object.__setattr__(packed, "_msb_validated", True)


def _validate_int4_data_matches_values(packed: Int4PackedDocs) -> None:
    """Reject ambiguous host payloads before they cross into device memory."""
    if packed.device != "cpu":
        return
    if not np.array_equal(packed.data, _pack_nibbles(packed.values)):
        raise ValueError("packed.data does not encode packed.values")


def int4_to_device(packed: Int4PackedDocs, device: str = "cuda") -> Int4PackedDocs:
    """Upload to a resident ``CudaInt4PackedDocs`` handle."""
    if device != "cuda":
        raise ValueError("device must be 'cuda'")
    _validate_int4_packed(packed)
    if packed.device == "cuda":
        return packed
    _validate_int4_data_matches_values(packed)
    from maxsim_b200 import _maxsim_cuda

    handle = _maxsim_cuda.CudaInt4PackedDocs(np.ascontiguousarray(packed.data, dtype=np.uint8),
                                             np.ascontiguousarray(packed.doc_offsets, dtype=np.int64), packed.dim,
                                             float(packed.scale))
    stored = None if packed.token_scale is None else packed.token_scale.copy()
    if stored is not None:
        handle.set_token_scale_vector(np.ascontiguousarray(stored, dtype=np.float32))
    return Int4PackedDocs(data=handle, values=None, doc_offsets=packed.doc_offsets.copy(), dim=packed.dim,
                          num_docs=packed.num_docs, scale=packed.scale, device="cuda", token_scale=stored)


def _resident(packed: Int4PackedDocs, device) -> Int4PackedDocs:
    _validate_int4_packed(packed)
    _effective_device(device, packed)
    return packed if packed.device == "cuda" else int4_to_device(packed)


def int4_maxsim(query_tokens, packed: Int4PackedDocs, *, device="auto", reducer="maxsim", query_weights=None,
                temperature: float = 1.0, candidate_indices=None) -> np.ndarray:
    """fp32-query int4 scores of every document (or of candidates), any reducer."""
    resident = _resident(packed, device)
    batches, squeeze, _ = _as_batches(query_tokens, packed.dim)
    reducer_value, weights, temperature_value = _normalize_reducer_options(
        reducer, query_weights, temperature, batch=batches.shape[0], query_tokens=batches.shape[1])
    candidates = _normalize_candidate_indices(candidate_indices, packed.num_docs)
    num_targets = packed.num_docs if candidates is None else candidates.shape[0]
    if num_targets == 0 or batches.shape[0] == 0:
        out = np.empty((batches.shape[0], num_targets), dtype=np.float32)
        return out[0] if squeeze else out
    if batches.shape[1] == 0:
        out = np.zeros((batches.shape[0], num_targets), dtype=np.float32)
        return out[0] if squeeze else out
    handle = resident.data
    if candidates is None and reducer_value == "maxsim":
        out = handle.maxsim_batch(batches)
    elif candidates is None:
        out = handle.score_batch(batches, reducer_value, weights, float(temperature_value))
    else:
        out = handle.score_candidates_batch(batches, candidates, reducer_value, weights, float(temperature_value))
    return out[0] if squeeze else out


def int4_maxsim_int8q(query_tokens, packed: Int4PackedDocs, *, device="auto") -> np.ndarray:
    """Scores with int8-quantised queries x int4 documents (exact integer dots, dim 128)."""
    _validate_int4_packed(packed)
    query = _as_numpy(query_tokens).astype(np.float32, copy=False)
    if query.ndim == 2:
        batches, squeeze = query[np.newaxis], True
    elif query.ndim == 3:
        batches, squeeze = query, False
    else:
        raise ValueError("query_tokens must have shape [query_tokens, dim] or [batch, query_tokens, dim]")
    if batches.shape[2] != packed.dim:
        raise ValueError(f"query dim={batches.shape[2]} does not match packed dim={packed.dim}")
    if batches.shape[0] == 0:
        return np.empty((0, packed.num_docs), dtype=np.float32)
    if batches.shape[1] == 0:
        out = np.zeros((batches.shape[0], packed.num_docs), dtype=np.float32)
        return out[0] if squeeze else out
    resident = _resident(packed, device)
    out = resident.data.maxsim_batch_int8q(np.ascontiguousarray(batches, dtype=np.float32))
    return out[0] if squeeze else out


def topk_int4_maxsim(query_tokens, packed: Int4PackedDocs, k: int, *, device="auto", prefer_int8_query: bool = False,
                     reducer="maxsim", query_weights=None, temperature: float = 1.0):
    """Fused GPU scan + top-k; ``prefer_int8_query`` selects the int8-query scan (MaxSim, dim 128)."""
    if k < 1:
        raise ValueError("k must be >= 1")
    if k > packed.num_docs:
        raise ValueError("k cannot exceed packed.num_docs")
    resident = _resident(packed, device)
    batches, squeeze, _ = _as_batches(query_tokens, packed.dim)
    reducer_value, weights, temperature_value = _normalize_reducer_options(
        reducer, query_weights, temperature, batch=batches.shape[0], query_tokens=batches.shape[1])
    if batches.shape[0] == 0:
        return np.empty((0, k), np.float32), np.empty((0, k), np.int64)
    handle = resident.data
    if reducer_value == "maxsim" and prefer_int8_query and packed.dim == 128:
        scores, ids = handle.topk_batch_int8q(batches, int(k))
    elif reducer_value == "maxsim":
        scores, ids = handle.topk_batch(batches, int(k))
    else:
        from maxsim_b200._maxsim_cuda import _topk_with_options

        scores, ids = _topk_with_options(handle, batches, int(k), reducer_value, weights, temperature_value)
    return (scores[0], ids[0]) if squeeze else (scores, ids)
