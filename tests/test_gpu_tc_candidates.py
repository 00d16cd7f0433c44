"""Short candidate lists on the tensor cores: each listed document a work unit of the full scan's kernel.

Lists naming fewer than one document in sixteen are scanned as work units built from the list on the
device (one per listed document and query-tile pair; an empty document scores 0) into a [B, D] scratch
and gathered; per-row lists (the residual cascade's rescoring) give each document to its row's tile
pair.  Scores must equal the full tensor-core scan's at the same positions bit for bit (same kernel, same
arithmetic), the C oracle for int8 queries, and the SIMT engine within 1e-4 for fp32 queries: with
duplicated ids, empty, one-token and multi-tile documents, twin mode and replicated rows (small
batches), several query-tile pairs (large batches), sign codes with token scales, the weighted / TopK /
SmoothSim reducers, the fused residual stream and the cascade.
"""

import ctypes

import numpy as np
import pytest

from oracle import reference_cpu as ref

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-4, 1e-4


def _engine(e, fn):
    from maxsim_b200 import _lib

    prev = _lib.get_engine()
    _lib.set_engine(e)
    try:
        return fn()
    finally:
        _lib.set_engine(prev)


def _ragged(rng, num_docs):
    kinds = rng.integers(0, 10, size=num_docs)
    lengths = np.where(kinds == 0, 0, np.where(kinds == 1, 1, np.where(kinds == 9, rng.integers(200, 1500, size=num_docs),
                                                                        rng.integers(2, 160, size=num_docs))))
    off = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    docs = rng.standard_normal((int(off[-1]), 128)).astype(np.float32)
    return docs, off


def _candidates(rng, off, n):
    """n ids (fewer than one document in 16) with a duplicate, an empty and a one-token document."""
    lengths = np.diff(off)
    ids = rng.choice(len(off) - 1, size=n - 3, replace=False)
    empty = np.flatnonzero(lengths == 0)[:1]
    one = np.flatnonzero(lengths == 1)[:1]
    ids = np.concatenate([ids, empty, one, ids[:1]]).astype(np.int64)
    assert ids.shape[0] * 16 < len(off) - 1
    return ids


def _oracle_int8(oracle_c, q, packed, off):
    B, Q, dim = q.shape
    D = len(off) - 1
    codes, qs = ref.quantize_query_int8(q.reshape(-1, dim))
    out = np.empty((B, D), np.float32)
    oracle_c.oracle_int4_int8q_scores(
        codes.ctypes.data_as(ctypes.c_void_p), qs.ctypes.data_as(ctypes.c_void_p), B, Q, dim,
        packed.data.ctypes.data_as(ctypes.c_void_p),
        None if packed.token_scale is None else packed.token_scale.ctypes.data_as(ctypes.c_void_p),
        ctypes.c_float(packed.scale), off.ctypes.data_as(ctypes.c_void_p), ctypes.c_int64(D), None, ctypes.c_int64(0),
        out.ctypes.data_as(ctypes.c_void_p), 8)
    return out


@pytest.mark.parametrize("gran", ["token", "tensor"])
@pytest.mark.parametrize("batch,qtok", [(1, 24), (2, 32), (3, 20), (7, 20), (40, 24)])
def test_int4_candidates_equal_the_full_scan(oracle_c, gran, batch, qtok):
    import maxsim_b200 as m
    from maxsim_b200 import _lib
    from maxsim_b200 import _maxsim_cuda as mc

    rng = np.random.default_rng(500 + 7 * batch + qtok)
    docs, off = _ragged(rng, 1200)
    packed = m.pack_int4_symmetric(docs, off, scale_granularity=gran)
    h = m.int4_to_device(packed).data
    q = rng.standard_normal((batch, qtok, 128)).astype(np.float32)
    ids = _candidates(rng, off, 60)
    i8 = mc._opts(query_mode=_lib.QUERY_I8)
    # int8 queries: exact, against the full scan and the oracle
    full8 = _engine(2, lambda: h.maxsim_batch_int8q(q))
    cand8 = _engine(2, lambda: h._score(q, i8, ids))
    np.testing.assert_array_equal(cand8, full8[:, ids])
    np.testing.assert_array_equal(cand8, _oracle_int8(oracle_c, q, packed, off)[:, ids])
    np.testing.assert_array_equal(_engine(1, lambda: h._score(q, i8, ids)), cand8)
    # fp32 queries (digit planes): the full scan's values; the SIMT engine's within tolerance
    full = _engine(2, lambda: h.maxsim_batch(q))
    cand = _engine(2, lambda: h.score_candidates_batch(q, ids))
    np.testing.assert_array_equal(cand, full[:, ids])
    np.testing.assert_allclose(cand, _engine(1, lambda: h.score_candidates_batch(q, ids)), rtol=RTOL, atol=ATOL)
    assert np.all(cand[:, np.diff(off)[ids] == 0] == 0)


@pytest.mark.parametrize("reducer,kw", [("weighted_maxsim", "w"), ("topk2", None), ("topk4", None), ("smoothsim", "t")])
@pytest.mark.parametrize("batch", [1, 9])
def test_reducers_on_candidates(reducer, kw, batch):
    import maxsim_b200 as m

    rng = np.random.default_rng(17 + batch)
    docs, off = _ragged(rng, 900)
    h = m.int4_to_device(m.pack_int4_symmetric(docs, off, scale_granularity="token")).data
    q = rng.standard_normal((batch, 20, 128)).astype(np.float32)
    ids = _candidates(rng, off, 50)
    extra = {}
    if kw == "w":
        extra["query_weights"] = rng.uniform(0.5, 1.5, size=20).astype(np.float32)
    elif kw == "t":
        extra["temperature"] = 0.2
    full = _engine(2, lambda: h.score_batch(q, reducer, **extra))
    cand = _engine(2, lambda: h.score_candidates_batch(q, ids, reducer, **extra))
    np.testing.assert_array_equal(cand, full[:, ids])
    np.testing.assert_allclose(cand, _engine(1, lambda: h.score_candidates_batch(q, ids, reducer, **extra)),
                               rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("batch", [1, 5])
@pytest.mark.parametrize("token_scale", [False, True])
def test_sign_code_candidates(batch, token_scale):
    from maxsim_b200 import _lib
    from maxsim_b200 import _maxsim_cuda as mc

    rng = np.random.default_rng(33 + batch)
    docs, off = _ragged(rng, 1000)
    packed = ref.pack_signs(docs)
    ts = rng.uniform(0.5, 2.0, size=docs.shape[0]).astype(np.float16).astype(np.float32) if token_scale else None
    h = mc.CudaPackedDocs(packed, off, 128)
    if ts is not None:
        h.set_token_scale_vector(ts)
    q = rng.standard_normal((batch, 20, 128)).astype(np.float32)
    ids = _candidates(rng, off, 50)
    full = _engine(2, lambda: h.score_batch(q, use_token_scale=token_scale))
    cand = _engine(2, lambda: h.score_candidates_batch(q, ids, use_token_scale=token_scale))
    np.testing.assert_array_equal(cand, full[:, ids])
    want = ref.score_binary_fp32(q, packed, 128, off, token_scale=ts)[:, ids]
    np.testing.assert_allclose(cand, want, rtol=RTOL, atol=ATOL)
    i8 = h._binary_opts(1.0, False, token_scale, query_mode=_lib.QUERY_I8)
    cand8 = _engine(2, lambda: h._score(q, i8, ids))
    np.testing.assert_array_equal(cand8, ref.score_binary_int8q(q, packed, off, token_scale=ts)[:, ids])


@pytest.mark.parametrize("batch", [1, 4])
def test_residual_candidates_and_cascade(batch):
    from maxsim_b200 import sdk

    rng = np.random.default_rng(71 + batch)
    docs, off = ref.clustered_corpus(1600, 20, 200, seed=batch)
    ids_text = [f"d{i}" for i in range(1600)]
    index = sdk.Index.from_embeddings(ids_text, docs, off, mode="int4_residual")
    rr = sdk.Reranker(index, device="cuda")
    h = rr.corpus.int4_packed.prefix_data  # one handle holds the prefix and the residual stream
    q = ref.clustered_queries(docs, off, batch, 24, seed=batch + 9)
    ids = _candidates(rng, off, 40) if np.any(np.diff(off) == 0) else rng.choice(1600, 40, replace=False)
    full = _engine(2, lambda: h.score_residual_batch(q))
    cand = _engine(2, lambda: h.score_residual_candidates_batch(q, ids))
    np.testing.assert_array_equal(cand, full[:, ids])
    np.testing.assert_allclose(cand, _engine(1, lambda: h.score_residual_candidates_batch(q, ids)), rtol=RTOL,
                               atol=ATOL)
    # the cascade's per-row rescoring lists (M = 64 < D / 16): the top-10 of the residual scores over each
    # row's 64 best prefix documents, exactly as the full scans give them
    s_tc, i_tc = _engine(2, lambda: h.cascade_topk_batch(q, 10, 64))
    prefix = _engine(2, lambda: h.score_batch(q))
    _, top_m = ref.topk_rows(prefix, 64)
    masked = np.full_like(full, -np.inf)
    for row in range(batch):
        masked[row, top_m[row]] = full[row, top_m[row]]
    want_s, want_i = ref.topk_rows(masked, 10)
    np.testing.assert_array_equal(i_tc, want_i)
    np.testing.assert_array_equal(s_tc, want_s)
