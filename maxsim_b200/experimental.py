"""int4 formats (tensor and per-token scale) and their GPU scoring API.

Public surface of the reference's int4 part of ``src/maxsim/experimental.py``
(``Int4PackedDocs``, ``pack_int4_symmetric``, ``int4_to_device``,
``int4_maxsim``, ``int4_maxsim_int8q``, ``topk_int4_maxsim``) and of its
dimension-centroid binary format behind the ``binary_q40`` corpus mode
(``DimCentroidCalibration``, ``fit_dim_centroid_calibration``,
``pack_dim_centroid_signs``, ``transform_query_dim_centroids``,
``dim_centroid_maxsim``, ``topk_dim_centroid_maxsim``).  The ternary
experiments of that module are not part of this package.
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


# ---------------------------------------------------------------------------
# Dimension-centroid sign codes (corpus mode "binary_q40")
# ---------------------------------------------------------------------------
# A token's bit for dimension i says whether x_i >= t_i; the bit decodes to the
# mean of the corpus values on its side of t_i (p_i above, n_i below).  With
# s = 2 * bit - 1, decoded x_i = (p_i + n_i) / 2 + s * (p_i - n_i) / 2, so
#   q . decoded(x) = 0.5 * sum_i q_i (p_i - n_i) s_i + 0.5 * sum_i q_i (p_i + n_i)
# and MaxSim over documents needs only the sign scan of the query scaled by
# (p - n); the second term is a per-query constant added after the scan
# (reference ``src/maxsim/experimental.py:69-146``, ``:612-622``).

@dataclass(frozen=True)
class DimCentroidCalibration:
    """Per-dimension threshold and the two decode values (fp32 ``[dim]`` each)."""

    thresholds: np.ndarray
    negative_centroids: np.ndarray
    positive_centroids: np.ndarray

    @property
    def dim(self) -> int:
        return int(self.thresholds.shape[0])

    @property
    def metadata_bytes(self) -> int:
        return int(self.dim * 3 * 4)


def _side_means(docs: np.ndarray, thresholds: np.ndarray):
    """Mean (float64 accumulation, stored as fp32) of each column at/above and below its threshold;
    an empty side decodes to the threshold itself."""
    negative = np.empty(docs.shape[1], dtype=np.float32)
    positive = np.empty(docs.shape[1], dtype=np.float32)
    for i in range(docs.shape[1]):
        col = docs[:, i]
        above = col >= thresholds[i]
        hi, lo = col[above], col[~above]
        positive[i] = np.float32(np.mean(hi, dtype=np.float64)) if hi.size else np.float32(thresholds[i])
        negative[i] = np.float32(np.mean(lo, dtype=np.float64)) if lo.size else np.float32(thresholds[i])
    return negative, positive


def _thresholds_for(thresholds, dim: int) -> np.ndarray:
    if thresholds is None:
        return np.zeros(dim, dtype=np.float32)
    t = _as_numpy(thresholds).astype(np.float32, copy=False)
    if t.ndim != 1 or t.shape[0] != dim:
        raise ValueError("thresholds must have shape [dim]")
    return np.ascontiguousarray(t, dtype=np.float32)


def fit_dim_centroid_calibration(doc_embeddings, *, thresholds=None, lloyd_iterations: int = 0) -> DimCentroidCalibration:
    """Fit the decode values for given thresholds (default 0), optionally refining the thresholds
    to the midpoints of the decode values (Lloyd iterations, stopping when they move < 1e-6)."""
    docs = _as_numpy(doc_embeddings).astype(np.float32, copy=False)
    if docs.ndim != 2:
        raise ValueError("doc_embeddings must have shape [num_doc_tokens, dim]")
    if docs.shape[1] % 8 != 0:
        raise ValueError("dim must be divisible by 8")
    if lloyd_iterations < 0:
        raise ValueError("lloyd_iterations must be >= 0")
    t = _thresholds_for(thresholds, docs.shape[1])
    negative, positive = _side_means(docs, t)
    for _ in range(lloyd_iterations):
        mid = ((negative + positive) * 0.5).astype(np.float32)
        negative, positive = _side_means(docs, mid)
        converged = np.allclose(mid, t, rtol=0.0, atol=1e-6)
        t = mid
        if converged:
            break
    return DimCentroidCalibration(thresholds=np.ascontiguousarray(t, dtype=np.float32),
                                  negative_centroids=np.ascontiguousarray(negative, dtype=np.float32),
                                  positive_centroids=np.ascontiguousarray(positive, dtype=np.float32))


def _check_calibration(calibration, dim: int | None = None) -> None:
    if not isinstance(calibration, DimCentroidCalibration):
        raise TypeError("calibration must be a DimCentroidCalibration instance")
    if calibration.thresholds.ndim != 1:
        raise ValueError("calibration thresholds must be one-dimensional")
    want = calibration.thresholds.shape[0] if dim is None else int(dim)
    for name, values in (("negative_centroids", calibration.negative_centroids),
                         ("positive_centroids", calibration.positive_centroids)):
        if values.ndim != 1 or values.shape[0] != want:
            raise ValueError(f"calibration {name} must have shape [dim]")
    if calibration.thresholds.shape[0] != want:
        raise ValueError("calibration thresholds must have shape [dim]")


def pack_dim_centroid_signs(doc_embeddings, doc_offsets=None, *, calibration: DimCentroidCalibration | None = None,
                            thresholds=None, lloyd_iterations: int = 0, device: str = "cpu"):
    """Sign bits of ``x - thresholds`` plus the calibration used (fitted when not given)."""
    from maxsim_b200._api import pack_signs

    docs = _as_numpy(doc_embeddings).astype(np.float32, copy=False)
    if calibration is None:
        calibration = fit_dim_centroid_calibration(docs, thresholds=thresholds, lloyd_iterations=lloyd_iterations)
    _check_calibration(calibration, docs.shape[1])
    shifted = docs - calibration.thresholds[np.newaxis, :]
    return pack_signs(shifted, doc_offsets, device=device), calibration


def transform_query_dim_centroids(query_tokens, calibration: DimCentroidCalibration) -> np.ndarray:
    """Query scaled per dimension by (positive - negative) decode values, fp32."""
    _check_calibration(calibration)
    q = _as_numpy(query_tokens).astype(np.float32, copy=False)
    if q.ndim not in (2, 3):
        raise ValueError("query_tokens must have shape [query_tokens, dim] or [batch, query_tokens, dim]")
    if q.shape[-1] != calibration.dim:
        raise ValueError(f"query dim={q.shape[-1]} does not match calibration dim={calibration.dim}")
    return np.ascontiguousarray(q * (calibration.positive_centroids - calibration.negative_centroids),
                                dtype=np.float32)


def _restore_centroid_scores(scores, query_tokens, calibration: DimCentroidCalibration) -> np.ndarray:
    """scan score * 0.5 + 0.5 * sum(q * (positive + negative)) per query (float64 sum, fp32 result)."""
    s = _as_numpy(scores).astype(np.float32, copy=False)
    q = _as_numpy(query_tokens).astype(np.float32, copy=False)
    mid = calibration.positive_centroids + calibration.negative_centroids
    if q.ndim == 2:
        const = np.float32(0.5 * np.sum(q * mid[np.newaxis, :], dtype=np.float64))
        return np.asarray(s * 0.5 + const, dtype=np.float32)
    if q.ndim == 3:
        const = 0.5 * np.sum(q * mid[np.newaxis, np.newaxis, :], axis=(1, 2), dtype=np.float64)
        return np.asarray(s * 0.5 + const[:, np.newaxis].astype(np.float32), dtype=np.float32)
    raise ValueError("query_tokens must have shape [query_tokens, dim] or [batch, query_tokens, dim]")


def dim_centroid_maxsim(query_tokens, packed, calibration: DimCentroidCalibration, *, device="auto",
                        restore_scores: bool = True, candidate_indices=None):
    """MaxSim of every document (or of candidates) against dimension-centroid sign codes (GPU scan)."""
    from maxsim_b200._api import maxsim

    scores = maxsim(transform_query_dim_centroids(query_tokens, calibration), packed, device=device,
                    candidate_indices=candidate_indices)
    return _restore_centroid_scores(scores, query_tokens, calibration) if restore_scores else scores


def topk_dim_centroid_maxsim(query_tokens, packed, calibration: DimCentroidCalibration, k: int, *, device="auto",
                             restore_scores: bool = True):
    """Top-k over dimension-centroid sign codes (scan + top-k on the GPU, ties to the lower id).

    The restore is an increasing affine map per query, so the order of the scan scores is the
    order of the restored scores."""
    from maxsim_b200._api import topk_maxsim

    scores, ids = topk_maxsim(transform_query_dim_centroids(query_tokens, calibration), packed, k, device=device)
    if restore_scores:
        scores = _restore_centroid_scores(scores, query_tokens, calibration)
    return scores, ids
