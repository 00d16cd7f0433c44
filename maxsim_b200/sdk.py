"""Public SDK: ``Index`` (= ``Corpus``), ``Reranker``, ``SearchResult``.

Same surface as the reference's ``src/maxsim/sdk.py``: corpus modes and named
presets, ``Index.from_embeddings`` / ``save`` / ``load`` with the reference's
npz layout (schema 2, readable schema 1), ``memory_report``,
``Reranker.load(path, device="cuda", int4_query=...)``, ``search`` (with
``rescore_candidates`` for ``int4_residual``) and ``rerank``.

All scoring runs on the GPU through ``libmaxsim_b200.so``; ``device="cpu"``
raises ``NotImplementedError``.  ``pooled_binary`` corpora are built by Ward
pooling of each document's tokens; ``binary_q40`` corpora carry a
dimension-centroid calibration (40th-percentile thresholds) and are scored by
the sign scan on the calibrated query.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Literal

import numpy as np

from maxsim_b200._api import PackedDocs, _as_numpy, maxsim, pack_signs, to_device, topk_maxsim, _CPU_SCORING
from maxsim_b200.cascade import (
    ResidualInt4PackedDocs,
    _stable_topk,
    _validate_residual_packed,
    cascade_topk,
    pack_residual_int4,
    residual_int4_to_device,
    residual_score,
)
from maxsim_b200.experimental import (
    DimCentroidCalibration,
    Int4PackedDocs,
    dim_centroid_maxsim,
    fit_dim_centroid_calibration,
    pack_dim_centroid_signs,
    topk_dim_centroid_maxsim,
    _validate_int4_data_matches_values,
    _validate_int4_packed,
    int4_maxsim,
    int4_to_device,
    pack_int4_symmetric,
    topk_int4_maxsim,
)

CorpusMode = Literal["binary", "binary_token_scale", "binary_token_scale_u8", "binary_token_scale_u4",
                     "pooled_binary", "binary_q40", "int4", "int4_per_token", "int4_residual"]

MODE_PRESETS = {
    "balanced": "binary_token_scale",
    "max_quality": "int4_per_token",
    "max_compression": "pooled_binary",
    "compact": "binary_token_scale_u4",
    "max_speed": "binary",
}
_BINARY_MODES = frozenset({"binary", "binary_token_scale", "binary_token_scale_u8", "binary_token_scale_u4",
                           "pooled_binary", "binary_q40"})
_INT4_MODES = frozenset({"int4", "int4_per_token"})
_ALL_MODES = _BINARY_MODES | _INT4_MODES | {"int4_residual"}
_MODE_ERROR = ("mode must be 'auto', one of 'binary', 'binary_token_scale', 'binary_token_scale_u8', "
               "'binary_token_scale_u4', 'pooled_binary', 'binary_q40', 'int4', 'int4_per_token', 'int4_residual', "
               f"or a preset in {sorted(MODE_PRESETS)}")


def resolve_auto_mode(num_docs: int, embeddings: np.ndarray | None = None) -> str:
    """``mode="auto"`` is the per-token int4 preset."""
    del num_docs, embeddings
    return "int4_per_token"


@dataclass(frozen=True)
class CorpusMemoryReport:
    encoded_bytes: int
    host_array_bytes: int
    device_index_bytes: int
    device_workspace_bytes: int | None
    serialized_bytes: int | None


@dataclass(frozen=True)
class SearchResult:
    doc_id: str
    score: float
    rank: int


def _pool_doc_tokens(docs: np.ndarray, offsets: np.ndarray, pool_factor: int):
    """Pool each document's tokens into ceil(n / pool_factor) clusters (reference
    src/maxsim/pooling.py:18-62): Ward linkage on the L2-normalised tokens, at most that
    many clusters, each replaced by the float64-accumulated mean of its raw tokens, in
    cluster-label order.  Documents already at or below the target keep their tokens."""
    if pool_factor < 1:
        raise ValueError("factor must be >= 1")
    if pool_factor == 1:
        return docs.copy(), offsets.copy()
    from scipy.cluster.hierarchy import fcluster, linkage

    pieces, lengths = [], []
    for d in range(offsets.shape[0] - 1):
        tokens = docs[int(offsets[d]):int(offsets[d + 1])]
        n = tokens.shape[0]
        target = max(1, -(-n // pool_factor))
        if n == 0 or n <= target:
            pieces.append(tokens.astype(np.float32, copy=True))
            lengths.append(n)
            continue
        unit = tokens / np.maximum(np.linalg.norm(tokens, axis=1, keepdims=True), 1e-12)
        labels = fcluster(linkage(unit, method="ward"), t=target, criterion="maxclust")
        count = int(labels.max())
        means = np.empty((count, tokens.shape[1]), dtype=np.float32)
        for c in range(count):
            means[c] = tokens[labels == c + 1].mean(axis=0, dtype=np.float64)
        pieces.append(means)
        lengths.append(count)
    out_offsets = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    out = np.concatenate(pieces, axis=0) if pieces else np.zeros((0, docs.shape[1]), np.float32)
    return np.ascontiguousarray(out, dtype=np.float32), out_offsets


@dataclass(frozen=True)
class Corpus:
    doc_ids: tuple[str, ...]
    mode: str
    packed: PackedDocs | None = None
    int4_packed: object | None = None
    calibration: object | None = None
    metadata: dict[str, Any] | None = None
    _source_path: Path | None = field(default=None, repr=False, compare=False)

    @classmethod
    def from_embeddings(cls, doc_ids, embeddings, offsets, *, mode: str = "auto", pool_factor: int | None = None,
                        metadata: dict[str, Any] | None = None) -> "Corpus":
        requested = mode
        ids = _normalize_doc_ids(doc_ids)
        docs = _as_numpy(embeddings).astype(np.float32, copy=False)
        mode = resolve_auto_mode(len(ids), docs) if mode == "auto" else MODE_PRESETS.get(mode, mode)
        offs = _normalize_sdk_offsets(offsets, docs.shape[0] if docs.ndim else 0)
        _validate_corpus_inputs(ids, docs, offs, mode)
        meta = {} if metadata is None else dict(metadata)
        if mode == "pooled_binary":
            factor = 3 if requested == "max_compression" and pool_factor is None else pool_factor
            factor = 2 if factor is None else factor
            if isinstance(factor, bool) or not isinstance(factor, (int, np.integer)) or int(factor) < 1:
                raise ValueError("pool_factor must be an integer >= 1")
            original = int(docs.shape[0])
            docs, offs = _pool_doc_tokens(docs, offs, int(factor))
            meta.update({"pool_factor": int(factor), "original_tokens": original, "pooled_tokens": int(docs.shape[0])})
            return cls(doc_ids=ids, mode=mode, packed=pack_signs(docs, offs), metadata=meta)
        if mode == "binary":
            return cls(doc_ids=ids, mode=mode, packed=pack_signs(docs, offs), metadata=meta)
        if mode in ("binary_token_scale", "binary_token_scale_u8", "binary_token_scale_u4"):
            kind = {"binary_token_scale": "mean_abs_fp16", "binary_token_scale_u8": "mean_abs_u8",
                    "binary_token_scale_u4": "mean_abs_u4"}[mode]
            return cls(doc_ids=ids, mode=mode, packed=pack_signs(docs, offs, token_scale=kind), metadata=meta)
        if mode == "binary_q40":
            # per-dimension 40th-percentile thresholds of the corpus (reference src/maxsim/sdk.py:164-174)
            thresholds = np.percentile(docs, 40.0, axis=0).astype(np.float32)
            calibration = fit_dim_centroid_calibration(docs, thresholds=thresholds)
            packed, calibration = pack_dim_centroid_signs(docs, offs, calibration=calibration)
            return cls(doc_ids=ids, mode=mode, packed=packed, calibration=calibration, metadata=meta)
        if mode == "int4":
            return cls(doc_ids=ids, mode=mode, int4_packed=pack_int4_symmetric(docs, offs), metadata=meta)
        if mode == "int4_per_token":
            return cls(doc_ids=ids, mode=mode,
                       int4_packed=pack_int4_symmetric(docs, offs, scale_granularity="token"), metadata=meta)
        if mode == "int4_residual":
            return cls(doc_ids=ids, mode=mode, int4_packed=pack_residual_int4(docs, offs), metadata=meta)
        raise ValueError(_MODE_ERROR)

    # -- persistence (npz schema 2) ----------------------------------------
    def save(self, path, *, compress: bool = True) -> None:
        """Reference ``Corpus.save`` (src/maxsim/sdk.py:203-250): one ``.npz``, schema 2.
        ``compress=False`` stores the members uncompressed (``np.savez``); int4 codes hardly compress,
        and stored members stream to the GPU at file-read speed (``maxsim_b200.loader``)."""
        _validate_corpus(self)
        out = Path(path)
        out.parent.mkdir(parents=True, exist_ok=True)
        arrays: dict[str, object] = {
            "schema_version": np.array(2, dtype=np.int64),
            "format": np.array("maxsim_corpus"),
            "mode": np.array(self.mode),
            "doc_ids": np.asarray(self.doc_ids),
            "metadata_json": np.array(json.dumps({} if self.metadata is None else self.metadata, sort_keys=True)),
        }
        if self.packed is not None:
            if self.packed.device != "cpu":
                raise ValueError("Corpus.save requires CPU packed docs")
            kind, values = _encode_scale(self.packed.scale)
            arrays.update({
                "packed_data": np.ascontiguousarray(self.packed.data, dtype=np.uint8),
                "doc_offsets": np.ascontiguousarray(self.packed.doc_offsets, dtype=np.int64),
                "dim": np.array(self.packed.dim, dtype=np.int64),
                "scale_kind": np.array(kind),
                "scale_values": values,
            })
            ts = self.packed.token_scale
            if ts is not None:
                if self.mode == "binary_token_scale_u8":
                    codes, params = _encode_log_codes(ts, 256)
                    arrays["token_scale_u8_codes"] = codes
                    arrays["token_scale_u8_params"] = params
                elif self.mode == "binary_token_scale_u4":
                    codes, params = _encode_log_codes(ts, 16)
                    padded = np.concatenate([codes, np.zeros(len(codes) % 2, dtype=np.uint8)])
                    arrays["token_scale_u4_codes"] = (padded[0::2] | (padded[1::2] << 4)).astype(np.uint8)
                    arrays["token_scale_u4_params"] = params
                    arrays["token_scale_u4_count"] = np.array(len(codes), dtype=np.int64)
                else:
                    arrays["token_scale_fp16"] = np.ascontiguousarray(ts, dtype=np.float16)
            if self.calibration is not None:
                arrays.update({
                    "centroid_thresholds": np.ascontiguousarray(self.calibration.thresholds, dtype=np.float32),
                    "centroid_negative": np.ascontiguousarray(self.calibration.negative_centroids, dtype=np.float32),
                    "centroid_positive": np.ascontiguousarray(self.calibration.positive_centroids, dtype=np.float32),
                })
        elif self.int4_packed is not None and self.mode == "int4_residual":
            p = self.int4_packed
            if p.device != "cpu":
                raise ValueError("Corpus.save requires CPU residual int4 packed docs")
            arrays.update({
                "int4_data": np.ascontiguousarray(p.prefix_data, dtype=np.uint8),
                "doc_offsets": np.ascontiguousarray(p.doc_offsets, dtype=np.int64),
                "dim": np.array(p.dim, dtype=np.int64),
                "int4_scale": np.array(p.prefix_scale, dtype=np.float32),
                "int4_token_scale": np.ascontiguousarray(p.prefix_token_scale, dtype=np.float32),
                "residual_int4_data": np.ascontiguousarray(p.residual_data, dtype=np.uint8),
                "residual_int4_scale": np.array(p.residual_scale, dtype=np.float32),
                "residual_int4_token_scale": np.ascontiguousarray(p.residual_token_scale, dtype=np.float32),
            })
        elif self.int4_packed is not None:
            p = self.int4_packed
            if p.device != "cpu":
                raise ValueError("Corpus.save requires CPU int4 packed docs")
            arrays.update({
                "int4_data": np.ascontiguousarray(p.data, dtype=np.uint8),
                "doc_offsets": np.ascontiguousarray(p.doc_offsets, dtype=np.int64),
                "dim": np.array(p.dim, dtype=np.int64),
                "int4_scale": np.array(p.scale, dtype=np.float32),
            })
            if p.token_scale is not None:
                arrays["int4_token_scale"] = np.ascontiguousarray(p.token_scale, dtype=np.float32)
        else:
            raise ValueError("corpus has no packed payload")
        with out.open("wb") as handle:
            (np.savez_compressed if compress else np.savez)(handle, **arrays)
        object.__setattr__(self, "_source_path", out.resolve())

    @classmethod
    def load(cls, path) -> "Corpus":
        source = Path(path).resolve()
        with np.load(source, allow_pickle=False) as data:
            if int(np.asarray(data["schema_version"]).item()) not in {1, 2}:
                raise ValueError("unsupported corpus schema_version")
            if str(np.asarray(data["format"]).item()) != "maxsim_corpus":
                raise ValueError("unsupported corpus format")
            mode = str(np.asarray(data["mode"]).item())
            ids = tuple(str(v) for v in np.asarray(data["doc_ids"]))
            metadata = json.loads(str(np.asarray(data["metadata_json"]).item()))
            raw_offsets = np.asarray(data["doc_offsets"])
            if not np.issubdtype(raw_offsets.dtype, np.integer):
                raise ValueError("serialized doc_offsets must contain integers")
            offsets = np.ascontiguousarray(raw_offsets, dtype=np.int64)
            dim = int(np.asarray(data["dim"]).item())
            calibration = None
            if mode == "binary_q40":
                calibration = DimCentroidCalibration(
                    thresholds=np.ascontiguousarray(data["centroid_thresholds"], dtype=np.float32),
                    negative_centroids=np.ascontiguousarray(data["centroid_negative"], dtype=np.float32),
                    positive_centroids=np.ascontiguousarray(data["centroid_positive"], dtype=np.float32))
            if mode in _BINARY_MODES:
                token_scale = None
                if "token_scale_fp16" in data:
                    token_scale = np.ascontiguousarray(data["token_scale_fp16"]).astype(np.float32)
                elif "token_scale_u8_codes" in data:
                    token_scale = _decode_log_codes(np.asarray(data["token_scale_u8_codes"]),
                                                    np.asarray(data["token_scale_u8_params"]), 256)
                elif "token_scale_u4_codes" in data:
                    packed_codes = np.asarray(data["token_scale_u4_codes"])
                    count = int(np.asarray(data["token_scale_u4_count"]).item())
                    codes = np.empty(packed_codes.shape[0] * 2, dtype=np.uint8)
                    codes[0::2] = packed_codes & 0x0F
                    codes[1::2] = packed_codes >> 4
                    token_scale = _decode_log_codes(codes[:count], np.asarray(data["token_scale_u4_params"]), 16)
                corpus = cls(doc_ids=ids, mode=mode, packed=PackedDocs(
                    data=_load_u8(data, "packed_data"), doc_offsets=offsets, dim=dim, num_docs=len(ids),
                    scale=_decode_scale(str(np.asarray(data["scale_kind"]).item()), np.asarray(data["scale_values"])),
                    device="cpu", token_scale=token_scale), calibration=calibration, metadata=metadata,
                    _source_path=source)
                _validate_corpus(corpus)
                return corpus
            if mode == "int4_residual":
                int4_data = _load_u8(data, "int4_data")
                residual_data = _load_u8(data, "residual_int4_data")
                _validate_serialized_offsets(offsets, len(ids), int4_data, dim, bytes_per_token=dim // 2)
                _validate_serialized_offsets(offsets, len(ids), residual_data, dim, bytes_per_token=dim // 2)
                packed = ResidualInt4PackedDocs(
                    prefix_data=int4_data, prefix_values=_unpack_signed_int4(int4_data, dim),
                    prefix_scale=float(np.asarray(data["int4_scale"]).item()),
                    prefix_token_scale=_load_f32(data, "int4_token_scale"),
                    residual_data=residual_data, residual_values=_unpack_signed_int4(residual_data, dim),
                    residual_scale=float(np.asarray(data["residual_int4_scale"]).item()),
                    residual_token_scale=_load_f32(data, "residual_int4_token_scale"),
                    doc_offsets=offsets, dim=dim, num_docs=len(ids), device="cpu")
                corpus = cls(doc_ids=ids, mode=mode, int4_packed=packed, metadata=metadata, _source_path=source)
                _validate_corpus(corpus)
                return corpus
            if mode in _INT4_MODES:
                int4_data = _load_u8(data, "int4_data")
                token_scale = _load_f32(data, "int4_token_scale") if "int4_token_scale" in data else None
                _validate_serialized_offsets(offsets, len(ids), int4_data, dim, bytes_per_token=dim // 2)
                corpus = cls(doc_ids=ids, mode=mode, int4_packed=Int4PackedDocs(
                    data=int4_data, values=_unpack_signed_int4(int4_data, dim), doc_offsets=offsets, dim=dim,
                    num_docs=len(ids), scale=float(np.asarray(data["int4_scale"]).item()), device="cpu",
                    token_scale=token_scale), metadata=metadata, _source_path=source)
                _validate_corpus(corpus)
                return corpus
            raise ValueError("unsupported corpus mode")

    @property
    def num_docs(self) -> int:
        return len(self.doc_ids)

    @property
    def dim(self) -> int:
        if self.packed is not None:
            return int(self.packed.dim)
        if self.int4_packed is not None:
            return int(self.int4_packed.dim)
        raise ValueError("corpus has no packed payload")

    @property
    def encoded_bytes(self) -> int:
        if self.packed is not None:
            extra = 0 if self.calibration is None else int(self.calibration.metadata_bytes)
            if isinstance(self.packed.scale, np.ndarray):
                extra += int(self.packed.scale.astype(np.float32, copy=False).nbytes)
            elif self.packed.scale is not None:
                extra += 4
            if self.packed.token_scale is not None:
                count = int(self.packed.token_scale.shape[0])
                if self.mode == "binary_token_scale_u8":
                    extra += count + 16
                elif self.mode == "binary_token_scale_u4":
                    extra += (count + 1) // 2 + 16
                else:
                    extra += count * 2
            if isinstance(self.packed.data, np.ndarray):
                return int(self.packed.data.size + extra)
            return int(self.packed.doc_offsets[-1] * (self.packed.dim // 8) + extra)
        if self.int4_packed is not None:
            return int(self.int4_packed.storage_bytes)
        return 0

    @property
    def storage_bytes(self) -> int:
        return self.encoded_bytes

    def memory_report(self, serialized_path=None) -> CorpusMemoryReport:
        _validate_corpus(self)
        src = self._source_path if serialized_path is None else Path(serialized_path)
        return CorpusMemoryReport(
            encoded_bytes=self.encoded_bytes,
            host_array_bytes=_host_array_bytes(self),
            device_index_bytes=_device_index_bytes(self),
            device_workspace_bytes=_device_workspace_bytes(self),
            serialized_bytes=None if src is None else int(src.stat().st_size),
        )


class Reranker:
    """GPU search / rerank over a corpus resident in device memory."""

    def __init__(self, corpus: Corpus, *, device: Literal["cpu", "cuda"] = "cuda",
                 int4_query: Literal["fp32", "int8"] = "fp32"):
        if device not in {"cpu", "cuda"}:
            raise ValueError("device must be 'cpu' or 'cuda'")
        if int4_query not in {"fp32", "int8"}:
            raise ValueError("int4_query must be 'fp32' or 'int8'")
        if device == "cpu":
            raise NotImplementedError(_CPU_SCORING)
        self.corpus = _move_corpus(corpus, device)
        self.device = device
        self.int4_query = int4_query
        self._doc_index = {doc_id: i for i, doc_id in enumerate(self.corpus.doc_ids)}

    @classmethod
    def _from_resident(cls, corpus: Corpus, *, int4_query: Literal["fp32", "int8"] = "fp32") -> "Reranker":
        """Wrap a corpus whose payload the streaming loader already placed and checked on the device."""
        if int4_query not in {"fp32", "int8"}:
            raise ValueError("int4_query must be 'fp32' or 'int8'")
        self = cls.__new__(cls)
        self.corpus = corpus
        self.device = "cuda"
        self.int4_query = int4_query
        self._doc_index = {doc_id: i for i, doc_id in enumerate(corpus.doc_ids)}
        return self

    @classmethod
    def from_corpus(cls, corpus: Corpus, *, device: Literal["cpu", "cuda"] = "cuda",
                    int4_query: Literal["fp32", "int8"] = "fp32") -> "Reranker":
        return cls(corpus, device=device, int4_query=int4_query)

    @classmethod
    def load(cls, path, *, device: Literal["cpu", "cuda"] = "cuda",
             int4_query: Literal["fp32", "int8"] = "fp32") -> "Reranker":
        """Reference ``Reranker.load`` (src/maxsim/sdk.py:393-396).  On CUDA the int4 family streams
        from the file into device memory (``maxsim_b200.loader``); the device arrays are the same."""
        if device == "cuda" and int4_query in {"fp32", "int8"}:
            from maxsim_b200.loader import load_reranker

            return load_reranker(path, int4_query=int4_query)
        return cls.from_corpus(Corpus.load(path), device=device, int4_query=int4_query)

    def search_arrays(self, query_embeddings, *, k: int = 10, rescore_candidates: int | None = None,
                      reducer: str = "maxsim", query_weights=None, temperature: float = 1.0):
        """Like :meth:`search` but returns ``(scores, doc indices)`` arrays."""
        _validate_k(k, self.corpus.num_docs)
        k = min(k, self.corpus.num_docs)
        mode = self.corpus.mode
        if rescore_candidates is not None and mode != "int4_residual":
            raise ValueError("rescore_candidates requires corpus mode='int4_residual'")
        kw = dict(reducer=reducer, query_weights=query_weights, temperature=temperature)
        if mode == "binary_q40":
            _require_maxsim_reducer(mode, reducer, query_weights, temperature)
            return topk_dim_centroid_maxsim(query_embeddings, self.corpus.packed, self.corpus.calibration, k,
                                            device="auto")
        if mode in _BINARY_MODES:
            return topk_maxsim(query_embeddings, self.corpus.packed, k, device="auto", **kw)
        if mode == "int4_residual":
            if rescore_candidates is None:
                return _stable_topk(residual_score(query_embeddings, self.corpus.int4_packed, device="auto", **kw), k)
            return cascade_topk(query_embeddings, self.corpus.int4_packed, k, candidates=rescore_candidates,
                                device="auto", **kw)
        if mode in _INT4_MODES:
            return topk_int4_maxsim(query_embeddings, self.corpus.int4_packed, k, device="auto",
                                    prefer_int8_query=self.int4_query == "int8", **kw)
        raise ValueError(f"unsupported corpus mode: {mode}")

    def search(self, query_embeddings, *, k: int = 10, rescore_candidates: int | None = None, reducer: str = "maxsim",
               query_weights=None, temperature: float = 1.0):
        scores, indices = self.search_arrays(query_embeddings, k=k, rescore_candidates=rescore_candidates,
                                             reducer=reducer, query_weights=query_weights, temperature=temperature)
        return _format_topk_results(scores, indices, self.corpus.doc_ids)

    def rerank(self, query_embeddings, candidate_ids, *, k: int = 10, reducer: str = "maxsim", query_weights=None,
               temperature: float = 1.0):
        candidates = _dedupe_candidate_ids(candidate_ids)
        idx = self._candidate_indices(candidates)
        if not candidates:
            return []
        scores = self._score_candidates(query_embeddings, idx, reducer=reducer, query_weights=query_weights,
                                        temperature=temperature)
        return _format_candidate_results(scores, np.arange(len(candidates), dtype=np.int64), candidates,
                                         min(k, len(candidates)))

    def _score_candidates(self, query_embeddings, candidate_indices, *, reducer, query_weights, temperature):
        kw = dict(device="auto", reducer=reducer, query_weights=query_weights, temperature=temperature,
                  candidate_indices=candidate_indices)
        mode = self.corpus.mode
        if mode == "binary_q40":
            _require_maxsim_reducer(mode, reducer, query_weights, temperature)
            return dim_centroid_maxsim(query_embeddings, self.corpus.packed, self.corpus.calibration, device="auto",
                                       candidate_indices=candidate_indices)
        if mode in _BINARY_MODES:
            return maxsim(query_embeddings, self.corpus.packed, **kw)
        if mode in _INT4_MODES:
            return int4_maxsim(query_embeddings, self.corpus.int4_packed, **kw)
        if mode == "int4_residual":
            return residual_score(query_embeddings, self.corpus.int4_packed, **kw)
        raise ValueError(f"unsupported corpus mode: {mode}")

    def _candidate_indices(self, candidate_ids):
        out = []
        for doc_id in candidate_ids:
            try:
                out.append(self._doc_index[doc_id])
            except KeyError as exc:
                raise KeyError(doc_id) from exc
        return np.asarray(out, dtype=np.int64)


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def _normalize_doc_ids(doc_ids) -> tuple[str, ...]:
    values = tuple(str(d) for d in doc_ids)
    if not values:
        raise ValueError("doc_ids must contain at least one id")
    if len(set(values)) != len(values):
        raise ValueError("doc_ids must be unique")
    return values


def _normalize_sdk_offsets(offsets, num_tokens: int) -> np.ndarray:
    raw = _as_numpy(offsets)
    if not np.issubdtype(raw.dtype, np.integer):
        raise ValueError("offsets must contain integers")
    values = raw.astype(np.int64, copy=False)
    if values.ndim != 1 or values.shape[0] < 2:
        raise ValueError("offsets must have shape [num_docs + 1]")
    if int(values[0]) != 0 or int(values[-1]) != num_tokens:
        raise ValueError("offsets must span embeddings")
    if np.any(values[1:] < values[:-1]):
        raise ValueError("offsets must be monotonically nondecreasing")
    return values.copy()


def _validate_corpus_inputs(doc_ids, docs, offsets, mode) -> None:
    if docs.ndim != 2:
        raise ValueError("embeddings must have shape [total_doc_tokens, dim]")
    if docs.shape[1] % 8 != 0:
        raise ValueError("embedding dim must be divisible by 8")
    if offsets.shape[0] != len(doc_ids) + 1:
        raise ValueError("offsets must have one more entry than doc_ids")
    if mode not in _ALL_MODES:
        raise ValueError(_MODE_ERROR)


def _validate_offset_values(offsets, num_docs: int, num_tokens: int) -> None:
    if not isinstance(offsets, np.ndarray) or not np.issubdtype(offsets.dtype, np.integer):
        raise ValueError("doc_offsets must be an integer NumPy array")
    if offsets.ndim != 1 or offsets.shape[0] != num_docs + 1:
        raise ValueError("doc_offsets must have shape [num_docs + 1]")
    if int(offsets[0]) != 0:
        raise ValueError("doc_offsets must start at 0")
    if np.any(offsets[1:] < offsets[:-1]):
        raise ValueError("doc_offsets must be monotonically nondecreasing")
    if int(offsets[-1]) != num_tokens:
        raise ValueError("doc_offsets must end at num_doc_tokens")


def _validate_token_scale(scale, num_tokens, name, *, allow_zero=True):
    if scale is None:
        return
    if not isinstance(scale, np.ndarray) or scale.ndim != 1 or scale.shape[0] != num_tokens:
        raise ValueError(f"{name} must have shape [num_doc_tokens]")
    if not np.issubdtype(scale.dtype, np.number):
        raise ValueError(f"{name} must contain numeric values")
    bad = scale < 0.0 if allow_zero else scale <= 0.0
    if not np.all(np.isfinite(scale)) or np.any(bad):
        raise ValueError(f"{name} must contain finite values {'nonnegative' if allow_zero else '> 0'}")


def _read_size(value, *names):
    for name in names:
        try:
            result = getattr(value, name)
        except (AttributeError, TypeError):
            continue
        if callable(result):
            result = result()
        result = int(result)
        if result < 0:
            raise ValueError(f"{name} must be nonnegative")
        return result
    return None


def _validate_corpus(corpus: Corpus) -> None:
    if not isinstance(corpus, Corpus):
        raise TypeError("corpus must be a Corpus instance")
    if not corpus.doc_ids:
        raise ValueError("corpus.doc_ids must contain at least one id")
    if any(not isinstance(d, str) for d in corpus.doc_ids):
        raise ValueError("corpus.doc_ids must contain strings")
    if len(set(corpus.doc_ids)) != len(corpus.doc_ids):
        raise ValueError("corpus.doc_ids must be unique")
    if corpus.metadata is not None and not isinstance(corpus.metadata, dict):
        raise ValueError("corpus.metadata must be a dictionary or None")
    if corpus.mode in _BINARY_MODES:
        p = corpus.packed
        if p is None or corpus.int4_packed is not None:
            raise ValueError(f"mode {corpus.mode!r} requires exactly one binary packed payload")
        if not isinstance(p, PackedDocs):
            raise ValueError("corpus.packed must be a PackedDocs instance")
        if p.dim <= 0 or p.dim % 8 != 0:
            raise ValueError("packed.dim must be positive and divisible by 8")
        if p.num_docs != len(corpus.doc_ids):
            raise ValueError("packed.num_docs must match corpus.doc_ids")
        if p.device == "cpu":
            if not isinstance(p.data, np.ndarray) or p.data.dtype != np.uint8:
                raise ValueError("CPU packed.data must be a uint8 NumPy array")
            if p.data.ndim != 2 or p.data.shape[1] != p.dim // 8:
                raise ValueError("packed.data must have shape [num_doc_tokens, dim / 8]")
            num_tokens = int(p.data.shape[0])
        else:
            size = _read_size(p.data, "packed_size")
            num_tokens = int(p.doc_offsets[-1]) if size is None else size // (p.dim // 8)
        _validate_offset_values(p.doc_offsets, len(corpus.doc_ids), num_tokens)
        needs = corpus.mode in {"binary_token_scale", "binary_token_scale_u8", "binary_token_scale_u4"}
        if needs != (p.token_scale is not None):
            raise ValueError(f"mode {corpus.mode!r} {'requires' if needs else 'does not accept'} binary token scales")
        _validate_token_scale(p.token_scale, num_tokens, "packed.token_scale")
        if corpus.mode == "binary_q40":
            if corpus.calibration is None:
                raise ValueError("binary_q40 mode requires centroid calibration")
            _validate_calibration_values(corpus.calibration, p.dim)
        elif corpus.calibration is not None:
            raise ValueError("centroid calibration is only valid for binary_q40 mode")
        return
    if corpus.calibration is not None and corpus.mode in _INT4_MODES:
        raise ValueError("centroid calibration is not valid for int4 modes")
    if corpus.calibration is not None and corpus.mode == "int4_residual":
        raise ValueError("centroid calibration is not valid for int4_residual")
    if corpus.mode in _INT4_MODES:
        p = corpus.int4_packed
        if p is None or corpus.packed is not None:
            raise ValueError(f"mode {corpus.mode!r} requires exactly one int4 packed payload")
        if not isinstance(p, Int4PackedDocs):
            raise ValueError("corpus.int4_packed must be an Int4PackedDocs instance")
        _validate_int4_packed(p)
        if p.num_docs != len(corpus.doc_ids):
            raise ValueError("int4_packed.num_docs must match corpus.doc_ids")
        if p.device == "cpu":
            _validate_int4_data_matches_values(p)
        needs = corpus.mode == "int4_per_token"
        if needs != (p.token_scale is not None):
            raise ValueError(f"mode {corpus.mode!r} {'requires' if needs else 'does not accept'} int4 token scales")
        return
    if corpus.mode == "int4_residual":
        if corpus.int4_packed is None or corpus.packed is not None:
            raise ValueError("mode 'int4_residual' requires exactly one residual int4 payload")
        _validate_residual_packed(corpus.int4_packed, verify_packed_values=True)
        if corpus.int4_packed.num_docs != len(corpus.doc_ids):
            raise ValueError("residual int4 num_docs must match corpus.doc_ids")
        return
    raise ValueError(f"unsupported corpus mode: {corpus.mode}")


def _validate_calibration_values(calibration, dim: int) -> None:
    """Shape and finiteness of a binary_q40 calibration (reference src/maxsim/sdk.py:897-903)."""
    for name in ("thresholds", "negative_centroids", "positive_centroids"):
        values = getattr(calibration, name, None)
        if not isinstance(values, np.ndarray) or values.ndim != 1 or values.shape[0] != dim:
            raise ValueError(f"calibration.{name} must have shape [dim]")
        if not np.all(np.isfinite(values)):
            raise ValueError(f"calibration.{name} must contain finite values")


def _require_maxsim_reducer(mode: str, reducer, query_weights, temperature) -> None:
    """Corpus modes scored by a transformed query support plain MaxSim only (reference sdk.py:1103-1113)."""
    if reducer != "maxsim":
        raise ValueError(f"corpus mode '{mode}' currently supports only reducer='maxsim'")
    if query_weights is not None:
        raise ValueError("query_weights is only supported with reducer='weighted_maxsim'")
    try:
        t = float(temperature)
    except (TypeError, ValueError) as exc:
        raise ValueError("temperature must be a finite value greater than 0") from exc
    if not np.isfinite(t) or t <= 0.0:
        raise ValueError("temperature must be a finite value greater than 0")


def _validate_serialized_offsets(offsets, num_docs, data, dim, *, bytes_per_token):
    if dim <= 0 or dim % 8 != 0:
        raise ValueError("serialized dim must be positive and divisible by 8")
    if data.ndim != 2 or data.shape[1] != bytes_per_token:
        raise ValueError("serialized packed data shape does not match dim")
    _validate_offset_values(offsets, num_docs, int(data.shape[0]))


def _load_u8(data, name):
    values = np.asarray(data[name])
    if values.dtype != np.uint8:
        raise ValueError(f"serialized {name} must have dtype uint8")
    return np.ascontiguousarray(values, dtype=np.uint8)


def _load_f32(data, name):
    values = np.asarray(data[name])
    if values.dtype != np.float32:
        raise ValueError(f"serialized {name} must have dtype float32")
    return np.ascontiguousarray(values, dtype=np.float32)


def _host_array_bytes(corpus: Corpus) -> int:
    arrays = []
    if corpus.packed is not None:
        p = corpus.packed
        for a in (p.data, p.doc_offsets, p.scale, p.token_scale):
            if isinstance(a, np.ndarray):
                arrays.append(a)
    if corpus.calibration is not None:
        for name in ("thresholds", "negative_centroids", "positive_centroids"):
            a = getattr(corpus.calibration, name, None)
            if isinstance(a, np.ndarray):
                arrays.append(a)
    if corpus.int4_packed is not None:
        names = (("prefix_data", "prefix_values", "prefix_token_scale", "residual_data", "residual_values",
                  "residual_token_scale", "doc_offsets") if corpus.mode == "int4_residual"
                 else ("data", "values", "doc_offsets", "token_scale"))
        for name in names:
            a = getattr(corpus.int4_packed, name, None)
            if isinstance(a, np.ndarray):
                arrays.append(a)
    return int(sum(a.nbytes for a in arrays))


def _device_index_bytes(corpus: Corpus) -> int:
    payload = corpus.packed if corpus.packed is not None else corpus.int4_packed
    if payload is None or getattr(payload, "device", "cpu") != "cuda":
        return 0
    handle = payload.prefix_data if corpus.mode == "int4_residual" else payload.data
    explicit = _read_size(handle, "device_index_bytes", "index_bytes", "resident_bytes")
    return 0 if explicit is None else explicit


def _device_workspace_bytes(corpus: Corpus):
    payload = corpus.packed if corpus.packed is not None else corpus.int4_packed
    if payload is None or getattr(payload, "device", "cpu") != "cuda":
        return 0
    handle = payload.prefix_data if corpus.mode == "int4_residual" else payload.data
    return _read_size(handle, "device_workspace_bytes", "workspace_bytes")


def _move_corpus(corpus: Corpus, device: str) -> Corpus:
    _validate_corpus(corpus)
    kw = dict(doc_ids=corpus.doc_ids, mode=corpus.mode, calibration=corpus.calibration, metadata=corpus.metadata,
              _source_path=corpus._source_path)
    if corpus.packed is not None:
        return Corpus(packed=to_device(corpus.packed, "cuda"), int4_packed=corpus.int4_packed, **kw)
    if corpus.mode == "int4_residual":
        return Corpus(packed=None, int4_packed=residual_int4_to_device(corpus.int4_packed), **kw)
    if corpus.int4_packed is not None:
        return Corpus(packed=None, int4_packed=int4_to_device(corpus.int4_packed), **kw)
    return corpus


def _encode_scale(scale):
    if scale is None:
        return "none", np.empty((0,), dtype=np.float32)
    if isinstance(scale, np.ndarray):
        return "vector", np.ascontiguousarray(scale, dtype=np.float32)
    return "scalar", np.array([float(scale)], dtype=np.float32)


def _decode_scale(kind, values):
    if kind == "none":
        return None
    if kind == "scalar":
        return float(values.reshape(-1)[0])
    if kind == "vector":
        return np.ascontiguousarray(values, dtype=np.float32)
    raise ValueError(f"unknown scale kind: {kind}")


def _encode_log_codes(values, levels):
    logs = np.log(np.maximum(values.astype(np.float64), 1e-12))
    lo, hi = float(logs.min()), float(logs.max())
    if hi <= lo:
        return np.zeros(values.shape[0], dtype=np.uint8), np.array([lo, lo], dtype=np.float64)
    steps = float(levels - 1)
    codes = np.clip(np.rint((logs - lo) * (steps / (hi - lo))), 0, steps).astype(np.uint8)
    return codes, np.array([lo, hi], dtype=np.float64)


def _decode_log_codes(codes, params, levels):
    lo, hi = float(params[0]), float(params[1])
    if hi <= lo:
        return np.full(codes.shape[0], np.exp(lo), dtype=np.float32)
    return np.exp(lo + codes.astype(np.float64) * ((hi - lo) / float(levels - 1))).astype(np.float32)


def _unpack_signed_int4(data, dim):
    low = (data & 0x0F).astype(np.int8)
    high = ((data >> 4) & 0x0F).astype(np.int8)
    out = np.empty((data.shape[0], dim), dtype=np.int8)
    out[:, 0::2] = np.where(low >= 8, low - 16, low)
    out[:, 1::2] = np.where(high >= 8, high - 16, high)
    return out


def _validate_k(k, max_count):
    if k < 1:
        raise ValueError("k must be >= 1")
    if max_count < 1:
        raise ValueError("corpus must contain at least one document")


def _dedupe_candidate_ids(candidate_ids):
    seen, out = set(), []
    for c in candidate_ids:
        v = str(c)
        if v not in seen:
            seen.add(v)
            out.append(v)
    return tuple(out)


def _format_topk_results(scores, indices, doc_ids):
    s = np.asarray(scores, dtype=np.float32)
    i = np.asarray(indices, dtype=np.int64)
    if s.ndim == 1:
        return _format_row(s, i, doc_ids)
    return [_format_row(rs, ri, doc_ids) for rs, ri in zip(s, i)]


def _format_row(scores, indices, doc_ids):
    return [SearchResult(doc_id=doc_ids[int(d)], score=float(v), rank=r)
            for r, (v, d) in enumerate(zip(scores, indices), start=1)]


def _format_candidate_results(scores, positions, candidate_ids, k):
    s = np.asarray(scores, dtype=np.float32)
    if s.ndim == 1:
        return _format_candidate_row(s, positions, candidate_ids, k)
    return [_format_candidate_row(row, positions, candidate_ids, k) for row in s]


def _format_candidate_row(scores, positions, candidate_ids, k):
    cand = scores[positions]
    order = np.lexsort((np.arange(cand.shape[0], dtype=np.int64), -cand))[:k]
    return [SearchResult(doc_id=candidate_ids[int(p)], score=float(cand[int(p)]), rank=r)
            for r, p in enumerate(order, start=1)]


Index = Corpus
