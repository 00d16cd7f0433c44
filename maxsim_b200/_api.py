"""Binary sign-code format and the generic scoring API.

Public surface of the reference's ``src/maxsim/_api.py`` (``PackedDocs``,
``pack_signs``, ``to_device``, ``score``, ``maxsim``, ``topk_maxsim``) with
the same arguments, validation and error types.  Encoding happens on the host
(offline index build); every score is computed on the GPU by
``libmaxsim_b200.so``.  ``device="auto"`` scores on the GPU, uploading a
host-resident corpus first; ``device="cpu"`` raises ``NotImplementedError``
because this package has no CPU scoring path.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

import numpy as np

Reducer = Literal["maxsim", "weighted_maxsim", "topk2", "topk4", "smoothsim"]
_REDUCERS = frozenset(("maxsim", "weighted_maxsim", "topk2", "topk4", "smoothsim"))
_CPU_SCORING = "maxsim_b200 scores on the GPU only; use device='cuda' or 'auto'"


@dataclass(frozen=True)
class PackedDocs:
    """Sign-bit corpus: ``data`` is uint8 ``[N, dim/8]`` on the host or a CUDA handle."""

    data: object
    doc_offsets: np.ndarray
    dim: int
    num_docs: int
    scale: object = None
    device: Literal["cpu", "cuda"] = "cpu"
    token_scale: object = None


def _as_numpy(value) -> np.ndarray:
    if isinstance(value, np.ndarray):
        return value
    detach = getattr(value, "detach", None)
    if detach is not None:
        return detach().cpu().numpy()
    return np.asarray(value)


def _normalize_offsets(doc_offsets, num_tokens: int) -> np.ndarray:
    if doc_offsets is None:
        return np.arange(num_tokens + 1, dtype=np.int64)
    offsets = _as_numpy(doc_offsets).astype(np.int64, copy=False)
    if offsets.ndim != 1:
        raise ValueError("doc_offsets must be a 1-D array")
    if offsets.shape[0] < 2:
        raise ValueError("doc_offsets must contain at least [0, num_doc_tokens]")
    if int(offsets[0]) != 0:
        raise ValueError("doc_offsets must start at 0")
    if int(offsets[-1]) != num_tokens:
        raise ValueError("doc_offsets must end at num_doc_tokens")
    if np.any(offsets[1:] < offsets[:-1]):
        raise ValueError("doc_offsets must be monotonically nondecreasing")
    return offsets.copy()


def _sign_bits(docs: np.ndarray) -> np.ndarray:
    """Bit i of byte i/8, least significant first, ``x >= 0 -> 1``."""
    n, dim = docs.shape
    bits = (docs >= 0).reshape(n, dim // 8, 8).astype(np.uint8)
    return np.ascontiguousarray(np.packbits(bits, axis=2, bitorder="little").reshape(n, dim // 8))


def _mean_abs(docs: np.ndarray) -> np.ndarray:
    return np.mean(np.abs(docs), axis=1, dtype=np.float64).astype(np.float32)


def _log_levels(scales: np.ndarray, levels: int) -> np.ndarray:
    """Quantise positive scales to ``levels`` log-spaced values."""
    logs = np.log(np.maximum(scales.astype(np.float64), 1e-12))
    lo, hi = float(logs.min()), float(logs.max())
    if hi <= lo:
        return scales.astype(np.float32)
    steps = float(levels - 1)
    codes = np.clip(np.rint((logs - lo) * (steps / (hi - lo))), 0, steps)
    return np.exp(lo + codes * ((hi - lo) / steps)).astype(np.float32)


def _resolve_pack_token_scale(token_scale, docs: np.ndarray):
    if token_scale is None:
        return None
    if isinstance(token_scale, str):
        if token_scale == "mean_abs":
            return _mean_abs(docs)
        if token_scale == "l2":
            return (np.linalg.norm(docs.astype(np.float64), axis=1) / np.sqrt(docs.shape[1])).astype(np.float32)
        if token_scale == "mean_abs_fp16":
            return _mean_abs(docs).astype(np.float16).astype(np.float32)
        if token_scale == "mean_abs_u8":
            return _log_levels(_mean_abs(docs), 256)
        if token_scale == "mean_abs_u4":
            return _log_levels(_mean_abs(docs), 16)
        raise ValueError(
            "token_scale must be None, 'mean_abs', 'mean_abs_fp16', 'mean_abs_u8', 'mean_abs_u4', 'l2', "
            "or a [num_doc_tokens] vector"
        )
    values = np.ascontiguousarray(_as_numpy(token_scale), dtype=np.float32)
    if values.ndim != 1 or values.shape[0] != docs.shape[0]:
        raise ValueError("token_scale vector must have shape [num_doc_tokens]")
    return values


def _doc_mean_abs(docs: np.ndarray, offsets: np.ndarray) -> np.ndarray:
    out = np.zeros(offsets.shape[0] - 1, dtype=np.float32)
    absd = np.abs(docs).astype(np.float32, copy=False)
    for d in range(out.shape[0]):
        s, e = int(offsets[d]), int(offsets[d + 1])
        if s != e:
            out[d] = np.float32(np.mean(absd[s:e], dtype=np.float64))
    return out


def _normalize_explicit_scale(scale, num_docs: int):
    values = _as_numpy(scale)
    if values.ndim == 0:
        return float(values)
    out = np.ascontiguousarray(values, dtype=np.float32)
    if out.ndim != 1 or out.shape[0] != num_docs:
        raise ValueError("scale vector must have shape [num_docs]")
    return out


def pack_signs(doc_embeddings, doc_offsets=None, *, dim=None, scale=None, token_scale=None, device="cpu") -> PackedDocs:
    """Encode embeddings as sign bits with optional document / token scales."""
    if device not in ("cpu", "cuda"):
        raise ValueError("device must be 'cpu' or 'cuda'")
    docs = _as_numpy(doc_embeddings)
    if docs.ndim != 2:
        raise ValueError("doc_embeddings must have shape [num_doc_tokens, dim]")
    actual_dim = int(docs.shape[1])
    if dim is not None and int(dim) != actual_dim:
        raise ValueError(f"dim={dim} does not match doc_embeddings dim={actual_dim}")
    if actual_dim % 8 != 0:
        raise ValueError("dim must be divisible by 8")
    offsets = _normalize_offsets(doc_offsets, docs.shape[0])
    docs = np.asarray(docs)
    packed = _sign_bits(docs) if docs.shape[0] else np.zeros((0, actual_dim // 8), np.uint8)
    if isinstance(scale, str) and scale == "global":
        stored = float(np.mean(np.abs(docs), dtype=np.float64))
    elif isinstance(scale, str) and scale in {"doc", "per_doc"}:
        stored = _doc_mean_abs(docs, offsets)
    elif scale is None:
        stored = None
    else:
        stored = _normalize_explicit_scale(scale, int(offsets.shape[0] - 1))
    result = PackedDocs(
        data=packed,
        doc_offsets=offsets,
        dim=actual_dim,
        num_docs=int(offsets.shape[0] - 1),
        scale=stored,
        device="cpu",
        token_scale=_resolve_pack_token_scale(token_scale, docs),
    )
    return result if device == "cpu" else to_device(result, "cuda")


def _validate_packed(packed: PackedDocs) -> None:
    if not isinstance(packed, PackedDocs):
        raise TypeError("packed must be a PackedDocs instance")
    if packed.dim % 8 != 0:
        raise ValueError("packed.dim must be divisible by 8")
    if packed.scale is not None:
        if isinstance(packed.scale, np.ndarray):
            if packed.scale.ndim != 1 or packed.scale.shape[0] != packed.num_docs:
                raise ValueError("packed.scale vector must have shape [num_docs]")
        else:
            float(packed.scale)
    if packed.token_scale is not None:
        if not isinstance(packed.token_scale, np.ndarray):
            raise ValueError("packed.token_scale must be a [num_doc_tokens] vector or None")
        if packed.token_scale.ndim != 1 or packed.token_scale.shape[0] != int(packed.doc_offsets[-1]):
            raise ValueError("packed.token_scale must have shape [num_doc_tokens]")
    if packed.device == "cuda":
        if not hasattr(packed.data, "maxsim_batch") and not hasattr(packed.data, "topk_batch"):
            raise ValueError("CUDA PackedDocs data must expose maxsim_batch or topk_batch")
        if packed.doc_offsets.ndim != 1 or packed.doc_offsets.shape[0] != packed.num_docs + 1:
            raise ValueError("packed.doc_offsets must have shape [num_docs + 1]")
        return
    if packed.device != "cpu":
        raise ValueError("packed.device must be 'cpu' or 'cuda'")
    if packed.data.ndim != 2 or packed.data.shape[1] != packed.dim // 8:
        raise ValueError("packed.data must have shape [num_doc_tokens, dim / 8]")
    if packed.doc_offsets.ndim != 1 or packed.doc_offsets.shape[0] != packed.num_docs + 1:
        raise ValueError("packed.doc_offsets must have shape [num_docs + 1]")


def to_device(packed: PackedDocs, device: Literal["cpu", "cuda"] = "cuda") -> PackedDocs:
    """Upload a binary corpus to a resident GPU handle (``CudaPackedDocs``)."""
    if device not in ("cpu", "cuda"):
        raise ValueError("device must be 'cpu' or 'cuda'")
    _validate_packed(packed)
    if device == packed.device:
        return packed
    if device == "cpu":
        raise NotImplementedError("copying CUDA PackedDocs back to CPU is not implemented")
    from maxsim_b200 import _maxsim_cuda

    offsets = np.ascontiguousarray(packed.doc_offsets, dtype=np.int64)
    handle = _maxsim_cuda.CudaPackedDocs(np.ascontiguousarray(packed.data, dtype=np.uint8), offsets, packed.dim)
    scale = packed.scale.copy() if isinstance(packed.scale, np.ndarray) else packed.scale
    if isinstance(scale, np.ndarray):
        handle.set_scale_vector(np.ascontiguousarray(scale, dtype=np.float32))
    token_scale = packed.token_scale.copy() if isinstance(packed.token_scale, np.ndarray) else packed.token_scale
    if isinstance(token_scale, np.ndarray):
        handle.set_token_scale_vector(np.ascontiguousarray(token_scale, dtype=np.float32))
    return PackedDocs(data=handle, doc_offsets=offsets.copy(), dim=packed.dim, num_docs=packed.num_docs,
                      scale=scale, device="cuda", token_scale=token_scale)


def _normalize_reducer_options(reducer, query_weights, temperature, *, batch: int, query_tokens: int):
    if not isinstance(reducer, str) or reducer not in _REDUCERS:
        raise ValueError(f"reducer must be one of: {', '.join(sorted(_REDUCERS))}")
    try:
        temperature_value = float(temperature)
    except (TypeError, ValueError) as exc:
        raise ValueError("temperature must be a finite value greater than 0") from exc
    if not np.isfinite(temperature_value) or temperature_value <= 0.0:
        raise ValueError("temperature must be a finite value greater than 0")
    if reducer != "weighted_maxsim":
        if query_weights is not None:
            raise ValueError("query_weights is only supported with reducer='weighted_maxsim'")
        return reducer, None, temperature_value
    if query_weights is None:
        raise ValueError("query_weights is required with reducer='weighted_maxsim'")
    weights = _as_numpy(query_weights).astype(np.float32, copy=False)
    if weights.ndim == 1:
        if weights.shape[0] != query_tokens:
            raise ValueError("query_weights must have shape [query_tokens] or [batch, query_tokens]")
        weights = np.broadcast_to(weights[np.newaxis, :], (batch, query_tokens))
    elif weights.ndim == 2:
        if weights.shape != (batch, query_tokens):
            raise ValueError("query_weights must have shape [query_tokens] or [batch, query_tokens]")
    else:
        raise ValueError("query_weights must have shape [query_tokens] or [batch, query_tokens]")
    if not np.all(np.isfinite(weights)):
        raise ValueError("query_weights must contain only finite values")
    return reducer, np.ascontiguousarray(weights, dtype=np.float32), temperature_value


def _normalize_candidate_indices(candidate_indices, num_docs: int):
    if candidate_indices is None:
        return None
    values = _as_numpy(candidate_indices)
    if values.ndim != 1 or not np.issubdtype(values.dtype, np.integer):
        raise ValueError("candidate_indices must be a one-dimensional integer array")
    out = np.ascontiguousarray(values, dtype=np.int64)
    if np.any(out < 0) or np.any(out >= num_docs):
        raise ValueError("candidate_indices must be between 0 and packed.num_docs - 1")
    return out


def _as_batches(query_tokens, dim: int):
    query = _as_numpy(query_tokens)
    if query.ndim == 2:
        batches, squeeze = query[np.newaxis, :, :], True
    elif query.ndim == 3:
        batches, squeeze = query, False
    else:
        raise ValueError("query_tokens must have shape [query_tokens, dim] or [batch, query_tokens, dim]")
    if batches.shape[2] != dim:
        raise ValueError(f"query dim={batches.shape[2]} does not match packed dim={dim}")
    return np.ascontiguousarray(batches, dtype=np.float32), squeeze, query


def _resolve_scale(scale, packed: PackedDocs):
    if scale is None:
        return 1.0 if packed.scale is None else packed.scale
    if isinstance(scale, str) and scale == "global":
        if packed.scale is None:
            raise ValueError("scale='global' requires a PackedDocs object with stored scale")
        if isinstance(packed.scale, np.ndarray):
            raise ValueError("scale='global' requires a scalar stored scale")
        return float(packed.scale)
    if isinstance(scale, str) and scale in {"doc", "per_doc"}:
        if not isinstance(packed.scale, np.ndarray):
            raise ValueError("scale='doc' requires a PackedDocs object with stored per-document scale")
        return packed.scale
    if isinstance(scale, str):
        raise ValueError("scale must be None, 'global', 'doc', a scalar, or a [num_docs] vector")
    return _normalize_explicit_scale(scale, packed.num_docs)


def _effective_device(device, packed) -> str:
    if device not in ("auto", "cpu", "cuda"):
        raise ValueError("device must be 'auto', 'cpu', or 'cuda'")
    if device == "cpu":
        raise NotImplementedError(_CPU_SCORING)
    return "cuda"


def _binary_handle_and_scale(packed: PackedDocs, resolved_scale):
    """Resident handle plus how to apply the resolved document scale."""
    resident = packed if packed.device == "cuda" else to_device(packed, "cuda")
    handle = resident.data
    use_vector = (isinstance(resolved_scale, np.ndarray) and resolved_scale is packed.scale
                  and bool(getattr(handle, "has_scale_vector", False)))
    override = None
    if isinstance(resolved_scale, np.ndarray) and not use_vector:
        override = np.ascontiguousarray(resolved_scale, dtype=np.float32)
    scalar = 1.0 if isinstance(resolved_scale, np.ndarray) else float(resolved_scale)
    return resident, handle, scalar, use_vector, override


def _score_binary(query_tokens, packed, *, scale, device, reducer, query_weights, temperature, candidate_indices):
    _effective_device(device, packed)
    _validate_packed(packed)
    batches, squeeze, _ = _as_batches(query_tokens, packed.dim)
    reducer_value, weights, temperature_value = _normalize_reducer_options(
        reducer, query_weights, temperature, batch=batches.shape[0], query_tokens=batches.shape[1])
    candidates = _normalize_candidate_indices(candidate_indices, packed.num_docs)
    resolved = _resolve_scale(scale, packed)
    use_token = isinstance(packed.token_scale, np.ndarray)
    num_targets = packed.num_docs if candidates is None else candidates.shape[0]
    if num_targets == 0 or batches.shape[0] == 0:
        out = np.empty((batches.shape[0], num_targets), dtype=np.float32)
        return out[0] if squeeze else out
    if batches.shape[1] == 0:
        out = np.zeros((batches.shape[0], num_targets), dtype=np.float32)
        return out[0] if squeeze else out
    _, handle, scalar, use_vector, override = _binary_handle_and_scale(packed, resolved)
    args = (reducer_value, weights, float(temperature_value), scalar, use_vector, use_token, override)
    if candidates is None:
        out = handle.score_batch(batches, *args)
    else:
        out = handle.score_candidates_batch(batches, candidates, *args)
    return out[0] if squeeze else out


def score(query_tokens, packed, *, reducer: Reducer = "maxsim", query_weights=None, temperature: float = 1.0,
          candidate_indices=None, scale=None, device="auto"):
    """Score binary or int4 corpora with a selected reducer (GPU)."""
    if isinstance(packed, PackedDocs):
        return _score_binary(query_tokens, packed, scale=scale, device=device, reducer=reducer,
                             query_weights=query_weights, temperature=temperature,
                             candidate_indices=candidate_indices)
    from maxsim_b200.experimental import Int4PackedDocs, int4_maxsim

    if isinstance(packed, Int4PackedDocs):
        if scale is not None:
            raise ValueError("scale is stored by Int4PackedDocs and cannot be overridden")
        return int4_maxsim(query_tokens, packed, device=device, reducer=reducer, query_weights=query_weights,
                           temperature=temperature, candidate_indices=candidate_indices)
    raise TypeError("packed must be a PackedDocs or Int4PackedDocs instance")


def maxsim(query_tokens, packed: PackedDocs, *, scale=None, device="auto", reducer: Reducer = "maxsim",
           query_weights=None, temperature: float = 1.0, candidate_indices=None):
    """Binary MaxSim (or another reducer) of every document, or of candidates."""
    return _score_binary(query_tokens, packed, scale=scale, device=device, reducer=reducer,
                         query_weights=query_weights, temperature=temperature, candidate_indices=candidate_indices)


def topk_maxsim(query_tokens, packed: PackedDocs, k: int, *, scale=None, device="auto", reducer: Reducer = "maxsim",
                query_weights=None, temperature: float = 1.0):
    """Fused GPU scan + top-k (score descending, ties to the lower document id)."""
    if k < 1:
        raise ValueError("k must be >= 1")
    if k > packed.num_docs:
        raise ValueError("k cannot exceed packed.num_docs")
    _validate_packed(packed)
    _effective_device(device, packed)
    batches, squeeze, raw = _as_batches(query_tokens, packed.dim)
    reducer_value, weights, temperature_value = _normalize_reducer_options(
        reducer, query_weights, temperature, batch=batches.shape[0], query_tokens=batches.shape[1])
    if batches.shape[0] == 0:
        return np.empty((0, k), np.float32), np.empty((0, k), np.int64)
    resolved = _resolve_scale(scale, packed)
    use_token = isinstance(packed.token_scale, np.ndarray)
    _, handle, scalar, use_vector, override = _binary_handle_and_scale(packed, resolved)
    if reducer_value == "maxsim" and override is None:
        scores, ids = handle.topk_batch(batches, int(k), scalar, use_vector, use_token)
    else:
        from maxsim_b200._maxsim_cuda import _topk_with_options

        scores, ids = _topk_with_options(handle, batches, int(k), reducer_value, weights, temperature_value,
                                         scalar, use_vector, use_token, override)
    return (scores[0], ids[0]) if squeeze else (scores, ids)
