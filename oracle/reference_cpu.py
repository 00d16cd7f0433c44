"""NumPy restatement of the reference maxsim scoring path (CPU oracle).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.  The product package
never imports this module.

Every function cites the reference file and line it restates (paths are
relative to the reference project root, ``src/maxsim/...`` for Python and
``cpp/maxsim/...`` for C++/CUDA).  Floating-point dot products of fp32-query
paths are evaluated in float64 here, i.e. closer to the exact value than
either reference implementation; parity with them is therefore a tolerance
check.  Integer (int8-query) paths are restated bit-exactly, including the
CUDA kernel's fp32 rounding steps, so those checks are exact.
"""

from __future__ import annotations

import numpy as np

REDUCERS = ("maxsim", "weighted_maxsim", "topk2", "topk4", "smoothsim")

# ---------------------------------------------------------------------------
# Formats
# ---------------------------------------------------------------------------


def pack_signs(docs: np.ndarray) -> np.ndarray:
    """Sign bits, bit ``i`` of byte ``i // 8`` (LSB first), ``x >= 0 -> 1``.

    Restates ``src/maxsim/_api.py:49-54``.
    """
    docs = np.asarray(docs, dtype=np.float32)
    bits = (docs >= 0).astype(np.uint8)
    n, dim = bits.shape
    bits = bits.reshape(n, dim // 8, 8)
    weights = (1 << np.arange(8, dtype=np.uint8)).astype(np.uint8)
    return np.ascontiguousarray((bits * weights).sum(axis=2).astype(np.uint8))


def unpack_signs(packed: np.ndarray, dim: int) -> np.ndarray:
    """Packed sign bits back to +-1.0 float32 (``src/maxsim/_api.py:632-637``)."""
    packed = np.asarray(packed, dtype=np.uint8)
    bits = np.unpackbits(packed, axis=1, bitorder="little")[:, :dim]
    return np.where(bits == 1, 1.0, -1.0).astype(np.float32)


def mean_abs_token_scale(docs: np.ndarray) -> np.ndarray:
    """Per-token mean |x| in float64, cast to float32 (``src/maxsim/_api.py:84-85``)."""
    return np.mean(np.abs(np.asarray(docs, dtype=np.float32)), axis=1, dtype=np.float64).astype(np.float32)


def log_quantized_scales(scales: np.ndarray, levels: int) -> np.ndarray:
    """Log-spaced scale quantisation (``src/maxsim/_api.py:106-116``)."""
    logs = np.log(np.maximum(scales.astype(np.float64), 1e-12))
    lo, hi = float(logs.min()), float(logs.max())
    if hi <= lo:
        return scales.astype(np.float32)
    steps = float(levels - 1)
    codes = np.clip(np.rint((logs - lo) * (steps / (hi - lo))), 0, steps)
    return np.exp(lo + codes * ((hi - lo) / steps)).astype(np.float32)


def token_scale(docs: np.ndarray, kind: str) -> np.ndarray:
    """Binary token-scale variants (``src/maxsim/_api.py:80-103``)."""
    if kind == "mean_abs":
        return mean_abs_token_scale(docs)
    if kind == "l2":
        d = np.asarray(docs, dtype=np.float64)
        return (np.linalg.norm(d, axis=1) / np.sqrt(d.shape[1])).astype(np.float32)
    if kind == "mean_abs_fp16":
        return mean_abs_token_scale(docs).astype(np.float16).astype(np.float32)
    if kind == "mean_abs_u8":
        return log_quantized_scales(mean_abs_token_scale(docs), 256)
    if kind == "mean_abs_u4":
        return log_quantized_scales(mean_abs_token_scale(docs), 16)
    raise ValueError(kind)


def encode_log_codes(values: np.ndarray, levels: int):
    """npz log-code encoder (``src/maxsim/sdk.py:1066-1074``)."""
    logs = np.log(np.maximum(values.astype(np.float64), 1e-12))
    lo, hi = float(logs.min()), float(logs.max())
    if hi <= lo:
        return np.zeros(values.shape[0], dtype=np.uint8), np.array([lo, lo], dtype=np.float64)
    steps = float(levels - 1)
    codes = np.clip(np.rint((logs - lo) * (steps / (hi - lo))), 0, steps).astype(np.uint8)
    return codes, np.array([lo, hi], dtype=np.float64)


def decode_log_codes(codes: np.ndarray, params: np.ndarray, levels: int) -> np.ndarray:
    """npz log-code decoder (``src/maxsim/sdk.py:1077-1082``)."""
    lo, hi = float(params[0]), float(params[1])
    if hi <= lo:
        return np.full(codes.shape[0], np.exp(lo), dtype=np.float32)
    return np.exp(lo + codes.astype(np.float64) * ((hi - lo) / float(levels - 1))).astype(np.float32)


def pack_nibbles(values: np.ndarray) -> np.ndarray:
    """Even dim in the low nibble, odd dim in the high nibble (``src/maxsim/experimental.py:604-609``)."""
    v = np.asarray(values).astype(np.int16)
    low = (v[:, 0::2] & 0x0F).astype(np.uint8)
    high = (v[:, 1::2] & 0x0F).astype(np.uint8)
    return np.ascontiguousarray(low | (high << 4))


def unpack_nibbles(data: np.ndarray, dim: int) -> np.ndarray:
    """Signed nibble decode (``src/maxsim/sdk.py:1085-1093``)."""
    data = np.asarray(data, dtype=np.uint8)
    low = (data & 0x0F).astype(np.int16)
    high = (data >> 4).astype(np.int16)
    low = np.where(low >= 8, low - 16, low)
    high = np.where(high >= 8, high - 16, high)
    out = np.empty((data.shape[0], dim), dtype=np.int8)
    out[:, 0::2] = low
    out[:, 1::2] = high
    return out


def pack_int4(docs: np.ndarray, granularity: str = "tensor"):
    """Symmetric int4 codes in [-7, 7].

    Restates ``src/maxsim/experimental.py:239-257``: per-token scale
    ``max|x_t| / 7`` (float32, zero -> 1) or tensor scale ``max|X| / 7``
    (float64 then used as float32), codes ``clip(rint(x / s), -7, 7)``.
    Returns ``(data, values, scale, token_scale)``.
    """
    docs = np.asarray(docs, dtype=np.float32)
    if granularity == "token":
        ts = np.max(np.abs(docs), axis=1).astype(np.float32) / np.float32(7.0)
        ts[ts == 0.0] = 1.0
        values = np.clip(np.rint(docs / ts[:, None]), -7, 7).astype(np.int8)
        scale = 1.0
    else:
        max_abs = float(np.max(np.abs(docs))) if docs.size else 0.0
        scale = 1.0 if max_abs == 0.0 else max_abs / 7.0
        values = np.clip(np.rint(docs / np.float32(scale)), -7, 7).astype(np.int8)
        ts = None
    return pack_nibbles(values), values, float(scale), ts


def reconstruct_int4(values, scale, token_scale):
    """``values * scale * token_scale`` (``src/maxsim/cascade.py:483-494``)."""
    out = values.astype(np.float32) * np.float32(scale)
    if token_scale is not None:
        out = out * token_scale[:, None]
    return out


def pack_residual_int4(docs: np.ndarray):
    """Per-token int4 prefix plus per-token int4 of the residual (``src/maxsim/cascade.py:60-93``)."""
    docs = np.asarray(docs, dtype=np.float32)
    p_data, p_values, p_scale, p_ts = pack_int4(docs, "token")
    residual = np.asarray(docs - reconstruct_int4(p_values, p_scale, p_ts), dtype=np.float32)
    r_data, r_values, r_scale, r_ts = pack_int4(residual, "token")
    return dict(
        prefix_data=p_data, prefix_values=p_values, prefix_scale=p_scale, prefix_token_scale=p_ts,
        residual_data=r_data, residual_values=r_values, residual_scale=r_scale, residual_token_scale=r_ts,
    )


# ---------------------------------------------------------------------------
# Query quantisation (CUDA kernel formula)
# ---------------------------------------------------------------------------


def quantize_query_int8(query: np.ndarray):
    """Per-row symmetric int8 query quantisation, kernel formula.

    Restates ``cpp/maxsim/cuda_extension.cu:1467-1491``: ``s = max|x| / 127``
    (1 when the row is all zero), ``inv = 1.0f / s`` (IEEE), code
    ``clamp(rint_half_even(x * inv), -127, 127)``.  Every step is an fp32
    operation, reproduced here with float32 NumPy arithmetic.
    Returns ``(codes int8 [..., dim], scales float32 [...])``.
    """
    q = np.asarray(query, dtype=np.float32)
    max_abs = np.max(np.abs(q), axis=-1)
    scale = np.where(max_abs == np.float32(0.0), np.float32(1.0), max_abs / np.float32(127.0)).astype(np.float32)
    inv = (np.float32(1.0) / scale).astype(np.float32)
    prod = (q * inv[..., None]).astype(np.float32)
    codes = np.clip(np.rint(prod), -127, 127).astype(np.int8)
    return codes, scale


# ---------------------------------------------------------------------------
# Reducers and top-k
# ---------------------------------------------------------------------------


def reduce_similarities(sims: np.ndarray, reducer: str, weights=None, temperature: float = 1.0) -> float:
    """Per-query-token reduction summed over query tokens.

    Restates ``src/maxsim/_api.py:558-585`` (evaluated in float64).
    ``sims`` is ``[query_tokens, doc_tokens]``.
    """
    if sims.shape[0] == 0 or sims.shape[1] == 0:
        return 0.0
    v = np.asarray(sims, dtype=np.float64)
    if reducer == "maxsim":
        return float(v.max(axis=1).sum())
    if reducer == "weighted_maxsim":
        return float((v.max(axis=1) * np.asarray(weights, dtype=np.float64)).sum())
    if reducer in ("topk2", "topk4"):
        want = 2 if reducer == "topk2" else 4
        count = min(want, v.shape[1])
        top = np.sort(v, axis=1)[:, -count:]
        return float(top.mean(axis=1).sum())
    if reducer == "smoothsim":
        tau = float(temperature)
        m = v.max(axis=1)
        return float((m + tau * np.log(np.exp((v - m[:, None]) / tau).sum(axis=1))).sum())
    raise ValueError(reducer)


def topk_indices(scores: np.ndarray, k: int, tie_ids=None) -> np.ndarray:
    """Score descending, ties to the lower id.

    Restates ``src/maxsim/_api.py:732-735`` and, with ``tie_ids``,
    ``src/maxsim/cascade.py:436-453``.
    """
    scores = np.asarray(scores, dtype=np.float32)
    ids = np.arange(scores.shape[0], dtype=np.int64) if tie_ids is None else np.asarray(tie_ids, dtype=np.int64)
    order = np.lexsort((ids, -scores))
    return np.ascontiguousarray(order[:k].astype(np.int64))


def topk_rows(scores: np.ndarray, k: int):
    """Row-wise :func:`topk_indices` returning ``(scores, indices)``."""
    scores = np.asarray(scores, dtype=np.float32)
    if scores.ndim == 1:
        idx = topk_indices(scores, k)
        return scores[idx], idx
    idx = np.stack([topk_indices(row, k) for row in scores]) if scores.shape[0] else np.empty((0, k), np.int64)
    return np.take_along_axis(scores, idx, axis=1), idx


# ---------------------------------------------------------------------------
# Scoring
# ---------------------------------------------------------------------------


def _targets(offsets, candidates):
    n_docs = int(len(offsets) - 1)
    return np.arange(n_docs, dtype=np.int64) if candidates is None else np.asarray(candidates, dtype=np.int64)


def _as_batches(query):
    q = np.asarray(query, dtype=np.float32)
    return (q[None], True) if q.ndim == 2 else (q, False)


def _weights_for(weights, b, qtok):
    if weights is None:
        return None
    w = np.asarray(weights, dtype=np.float32)
    if w.ndim == 1:
        return w
    return w[b] if w.shape[0] > 1 else w[0]


def score_dense(query, doc_vectors, offsets, *, reducer="maxsim", weights=None, temperature=1.0,
                candidates=None, token_scale=None, doc_scale=None, scale_before_reduction_for_smooth=True):
    """Generic reducer scoring of reconstructed document vectors.

    This is the shared shape of ``src/maxsim/experimental.py:403-420`` (int4),
    ``src/maxsim/_api.py:396-422`` (binary) and
    ``src/maxsim/cascade.py:272-291`` (residual): per document,
    ``sims = q @ doc.T`` (times per-token scales), reduce, then apply the
    document scale -- before the reduction for SmoothSim, after it otherwise.
    """
    batches, squeeze = _as_batches(query)
    targets = _targets(offsets, candidates)
    out = np.zeros((batches.shape[0], targets.shape[0]), dtype=np.float64)
    docs64 = np.asarray(doc_vectors, dtype=np.float64)
    for b, qm in enumerate(batches.astype(np.float64)):
        wb = _weights_for(weights, b, qm.shape[0])
        for j, d in enumerate(targets):
            s, e = int(offsets[d]), int(offsets[d + 1])
            if s == e or qm.shape[0] == 0:
                out[b, j] = 0.0
                continue
            sims = qm @ docs64[s:e].T
            if token_scale is not None:
                sims = sims * np.asarray(token_scale[s:e], dtype=np.float64)[None, :]
            ds = 1.0 if doc_scale is None else (float(doc_scale[d]) if np.ndim(doc_scale) else float(doc_scale))
            if reducer == "smoothsim" and scale_before_reduction_for_smooth:
                out[b, j] = reduce_similarities(sims * ds, reducer, wb, temperature)
            else:
                out[b, j] = reduce_similarities(sims, reducer, wb, temperature) * ds
    out = out.astype(np.float32)
    return out[0] if squeeze else out


def score_int4_fp32(query, values, offsets, *, scale=1.0, token_scale=None, **kw):
    """fp32-query int4 scoring (``src/maxsim/experimental.py:403-420``;
    CUDA semantics ``cpp/maxsim/cuda_extension.cu:1268-1323`` and ``:682-844``)."""
    return score_dense(query, np.asarray(values, dtype=np.float32), offsets, token_scale=token_scale,
                       doc_scale=float(scale), **kw)


def score_binary_fp32(query, packed, dim, offsets, *, token_scale=None, doc_scale=1.0, **kw):
    """fp32-query binary scoring (``src/maxsim/_api.py:396-422``)."""
    return score_dense(query, unpack_signs(packed, dim), offsets, token_scale=token_scale,
                       doc_scale=doc_scale, **kw)


def score_residual(query, res: dict, offsets, **kw):
    """Fused residual scoring ``dot(q,p)*ps*pts + dot(q,r)*rs*rts`` then reduce.

    Restates ``src/maxsim/cascade.py:272-291`` / ``:469-480`` and the CUDA
    kernel ``cpp/maxsim/cuda_extension.cu:1087-1101``.
    """
    p = res["prefix_values"].astype(np.float64) * float(np.float32(res["prefix_scale"])) * \
        res["prefix_token_scale"].astype(np.float64)[:, None]
    r = res["residual_values"].astype(np.float64) * float(np.float32(res["residual_scale"])) * \
        res["residual_token_scale"].astype(np.float64)[:, None]
    return score_dense(query, p + r, offsets, **kw)


def _int8q_epilogue(dots_int, row_scales, token_scale, doc_scale_value):
    """fp32 epilogue of the int8-query kernels, bit-exact.

    ``cpp/maxsim/cuda_extension.cu:1602-1625``: per token ``float(dot) * s_t``
    (fp32 RN), maximum over tokens, ``doc += best * qscale`` accumulated in
    fp32 in query-token order, finally ``* scale``.
    Tensor-scale variant (``:1539-1562``) takes the integer maximum first,
    which yields the same value because ``float()`` is exact below 2**24.
    """
    vals = dots_int.astype(np.float32)
    if token_scale is not None:
        vals = (vals * token_scale[None, :].astype(np.float32)).astype(np.float32)
    best = vals.max(axis=1).astype(np.float32)
    acc = np.float32(0.0)
    for r in range(best.shape[0]):
        acc = np.float32(acc + np.float32(best[r] * row_scales[r]))
    return np.float32(acc * np.float32(doc_scale_value))


def score_int4_int8q(query, values, offsets, *, scale=1.0, token_scale=None, candidates=None):
    """int8-query x int4 scoring with exact integer dots.

    Restates ``cpp/maxsim/cuda_extension.cu:1455-1627`` (quantise, exact
    int32 dot, scale-before-max for per-token scales).  Empty documents and
    empty query rows give 0.
    """
    batches, squeeze = _as_batches(query)
    targets = _targets(offsets, candidates)
    vals64 = np.asarray(values, dtype=np.int64)
    out = np.zeros((batches.shape[0], targets.shape[0]), dtype=np.float32)
    for b, qm in enumerate(batches):
        if qm.shape[0] == 0:
            continue
        codes, qs = quantize_query_int8(qm)
        c64 = codes.astype(np.int64)
        for j, d in enumerate(targets):
            s, e = int(offsets[d]), int(offsets[d + 1])
            if s == e:
                continue
            dots = c64 @ vals64[s:e].T
            out[b, j] = _int8q_epilogue(dots, qs, None if token_scale is None else token_scale[s:e], scale)
    return out[0] if squeeze else out


def score_binary_int8q(query, packed, offsets, *, token_scale=None, doc_scale=1.0, candidates=None):
    """int8-query x binary scoring, exact ``2*dot01 - qsum`` = sum of +-q.

    Restates ``cpp/maxsim/cuda_extension.cu:1328-1449``; the quantiser there
    (``:1341-1362``) uses the same formula as the int4 path.
    """
    batches, squeeze = _as_batches(query)
    dim = batches.shape[-1]
    signs = unpack_signs(packed, dim).astype(np.int64)
    targets = _targets(offsets, candidates)
    out = np.zeros((batches.shape[0], targets.shape[0]), dtype=np.float32)
    for b, qm in enumerate(batches):
        if qm.shape[0] == 0:
            continue
        codes, qs = quantize_query_int8(qm)
        c64 = codes.astype(np.int64)
        for j, d in enumerate(targets):
            s, e = int(offsets[d]), int(offsets[d + 1])
            if s == e:
                continue
            dots = c64 @ signs[s:e].T
            ds = float(doc_scale[d]) if np.ndim(doc_scale) else float(doc_scale)
            out[b, j] = _int8q_epilogue(dots, qs, None if token_scale is None else token_scale[s:e], ds)
    return out[0] if squeeze else out


def exact_int_dots(query_codes: np.ndarray, values: np.ndarray) -> np.ndarray:
    """Exact int64 ``codes @ values.T`` -- the integer dot that GPU paths must reproduce."""
    return np.asarray(query_codes, dtype=np.int64) @ np.asarray(values, dtype=np.int64).T


# ---------------------------------------------------------------------------
# Cascade
# ---------------------------------------------------------------------------


def cascade_topk(query, res: dict, offsets, k: int, candidates: int, *, reducer="maxsim", weights=None,
                 temperature=1.0):
    """Prefix scan -> stable top-M -> fused residual rescoring -> top-k.

    Restates ``src/maxsim/cascade.py:294-417``: the coarse pass scores the
    per-token int4 prefix with the same reducer, the per-row top-``M`` uses
    lower-id ties, the candidates are rescored with the fused two-stream
    similarity and the final order breaks ties by candidate document id.
    """
    batches, squeeze = _as_batches(query)
    n_docs = int(len(offsets) - 1)
    out_s, out_i = [], []
    for b, qm in enumerate(batches):
        wb = None if weights is None else _weights_for(weights, b, qm.shape[0])
        if candidates == n_docs:
            fine = score_residual(qm, res, offsets, reducer=reducer, weights=wb, temperature=temperature)
            idx = topk_indices(fine, k)
            out_s.append(fine[idx])
            out_i.append(idx)
            continue
        coarse = score_int4_fp32(qm, res["prefix_values"], offsets, scale=res["prefix_scale"],
                                 token_scale=res["prefix_token_scale"], reducer=reducer, weights=wb,
                                 temperature=temperature)
        cand = topk_indices(coarse, candidates)
        fine = score_residual(qm, res, offsets, reducer=reducer, weights=wb, temperature=temperature,
                              candidates=cand)
        order = topk_indices(fine, k, tie_ids=cand)
        out_s.append(fine[order])
        out_i.append(cand[order])
    s, i = np.stack(out_s), np.stack(out_i)
    return (s[0], i[0]) if squeeze else (s, i)


# ---------------------------------------------------------------------------
# Binary-prefix residual cascade (parity unpinned: the reference has no such
# format; this follows the benchmark description of the binary-prefix cascade,
# with the per-token mean |x| of ``src/maxsim/_api.py:84-85`` as the sign
# reconstruction scale and the per-token int4 of ``experimental.py:240-246``
# for the residual, fused like ``cascade.py:469-480``)
# ---------------------------------------------------------------------------

def pack_binary_residual(docs: np.ndarray) -> dict:
    """Sign bits + per-token mean |x|; residual x - mean|x| * sign(x) as per-token int4."""
    x = np.asarray(docs, dtype=np.float32)
    ps = mean_abs_token_scale(x)
    signs = np.where(x >= 0, np.float32(1.0), np.float32(-1.0))
    residual = (x - ps[:, None] * signs).astype(np.float32)
    rdata, rvals, _, rts = pack_int4(residual, "token")
    return dict(bits=pack_signs(x), prefix_token_scale=ps, residual_data=rdata, residual_values=rvals,
                residual_token_scale=rts)


def score_binary_residual(query, res: dict, offsets, **kw):
    """Fused similarity sign(x).q * ps + r.q * rts, then the reducer (float64 reference)."""
    dim = res["bits"].shape[1] * 8
    p = unpack_signs(res["bits"], dim).astype(np.float64) * res["prefix_token_scale"].astype(np.float64)[:, None]
    r = res["residual_values"].astype(np.float64) * res["residual_token_scale"].astype(np.float64)[:, None]
    return score_dense(query, p + r, offsets, **kw)


def binary_cascade_topk(query, res: dict, offsets, k: int, candidates: int, *, reducer="maxsim", weights=None,
                        temperature=1.0):
    """Sign-prefix scan (scaled by ps) -> stable top-M -> fused rescoring -> top-k (ties by candidate id)."""
    batches, squeeze = _as_batches(query)
    n_docs = int(len(offsets) - 1)
    dim = res["bits"].shape[1] * 8
    out_s, out_i = [], []
    for b, qm in enumerate(batches):
        wb = None if weights is None else _weights_for(weights, b, qm.shape[0])
        kw = dict(reducer=reducer, weights=wb, temperature=temperature)
        if candidates == n_docs:
            fine = score_binary_residual(qm, res, offsets, **kw)
            idx = topk_indices(fine, k)
            out_s.append(fine[idx])
            out_i.append(idx)
            continue
        coarse = score_binary_fp32(qm, res["bits"], dim, offsets, token_scale=res["prefix_token_scale"], **kw)
        cand = topk_indices(coarse, candidates)
        fine = score_binary_residual(qm, res, offsets, candidates=cand, **kw)
        order = topk_indices(fine, k, tie_ids=cand)
        out_s.append(fine[order])
        out_i.append(cand[order])
    s, i = np.stack(out_s), np.stack(out_i)
    return (s[0], i[0]) if squeeze else (s, i)


# ---------------------------------------------------------------------------
# Synthetic corpora shaped like the benchmark configurations
# ---------------------------------------------------------------------------


def clustered_corpus(num_docs: int, min_len: int, max_len: int, dim: int = 128, noise: float = 0.3,
                     seed: int = 0):
    """Per-doc Gaussian centroid + N(0, noise^2) noise, L2-normalised fp32."""
    rng = np.random.default_rng(seed)
    lengths = rng.integers(min_len, max_len + 1, size=num_docs)
    offsets = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    centroids = rng.standard_normal((num_docs, dim)).astype(np.float32)
    centroids /= np.linalg.norm(centroids, axis=1, keepdims=True)
    docs = np.repeat(centroids, lengths, axis=0) + noise * rng.standard_normal((int(offsets[-1]), dim)).astype(np.float32)
    docs /= np.linalg.norm(docs, axis=1, keepdims=True)
    return docs.astype(np.float32), offsets


def clustered_queries(docs, offsets, batch: int, qtok: int, noise: float = 0.3, seed: int = 1):
    """Query tokens sampled from random target docs plus noise, L2-normalised."""
    rng = np.random.default_rng(seed)
    n_docs = len(offsets) - 1
    out = np.empty((batch, qtok, docs.shape[1]), dtype=np.float32)
    for b in range(batch):
        d = int(rng.integers(0, n_docs))
        s, e = int(offsets[d]), int(offsets[d + 1])
        if e == s:
            out[b] = rng.standard_normal((qtok, docs.shape[1]))
        else:
            out[b] = docs[rng.integers(s, e, size=qtok)] + noise * rng.standard_normal((qtok, docs.shape[1]))
    out /= np.maximum(np.linalg.norm(out, axis=2, keepdims=True), 1e-12)
    return out.astype(np.float32)
