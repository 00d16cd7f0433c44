"""Load-to-GPU path: ``Reranker.load`` streams a saved index into device memory.

The streamed handle must hold the same bytes as the host path's upload (``Corpus.load`` then
``Reranker``), so every search result is identical, including with chunk boundaries that cut tokens
and with a document range (a shard), whose per-document scores equal the full corpus's.  Bad token
scales are rejected on the device with the host path's error, and a handle whose upload is open
refuses to score.
"""

import numpy as np
import pytest

from oracle import reference_cpu as ref

pytestmark = pytest.mark.gpu
MODES = ["int4", "int4_per_token", "int4_residual"]


def _saved(tmp_path, mode, docs=57, seed=41):
    import maxsim_b200 as m

    d, off = ref.clustered_corpus(docs, 0, 40, seed=seed)
    ids = [f"doc-{i}" for i in range(docs)]
    idx = m.Index.from_embeddings(ids, d, off, mode=mode)
    path = tmp_path / f"{mode}.npz"
    idx.save(path)
    q = ref.clustered_queries(d, off, 3, 9, seed=seed + 1)
    return path, idx, q


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("int4_query", ["fp32", "int8"])
def test_streamed_load_matches_host_load(tmp_path, mode, int4_query):
    import maxsim_b200 as m
    from maxsim_b200.loader import load_reranker

    path, _, q = _saved(tmp_path, mode)
    host = m.Reranker.from_corpus(m.Index.load(path), device="cuda", int4_query=int4_query)
    stats = {}
    # 1000-byte chunks cut tokens (64 B each) mid-row and use every staging buffer many times
    streamed = load_reranker(path, int4_query=int4_query, chunk_bytes=1000, staging_buffers=2, stats=stats)
    default = m.Reranker.load(path, device="cuda", int4_query=int4_query)
    assert stats["tokens"] == host.corpus.int4_packed.doc_offsets[-1]
    kw = {"rescore_candidates": 20} if mode == "int4_residual" else {}
    want_s, want_i = host.search_arrays(q, k=7, **kw)
    for rr in (streamed, default):
        got_s, got_i = rr.search_arrays(q, k=7, **kw)
        np.testing.assert_array_equal(got_i, want_i)
        np.testing.assert_array_equal(got_s, want_s)
        assert rr.corpus.doc_ids == host.corpus.doc_ids
        res = rr.search(q[0], k=3)
        assert [r.doc_id for r in res] == [x.doc_id for x in host.search(q[0], k=3)]


@pytest.mark.parametrize("mode", MODES)
def test_streamed_doc_range_is_a_shard(tmp_path, mode):
    import maxsim_b200 as m
    from maxsim_b200 import experimental as ex
    from maxsim_b200.cascade import residual_score
    from maxsim_b200.loader import load_resident_corpus

    path, _, q = _saved(tmp_path, mode)
    full = m.Reranker.load(path, device="cuda").corpus
    lo, hi = 11, 43
    shard = load_resident_corpus(path, doc_range=(lo, hi), chunk_bytes=4096)
    assert shard.doc_ids == full.doc_ids[lo:hi]
    if mode == "int4_residual":
        want = residual_score(q, full.int4_packed, device="cuda")
        got = residual_score(q, shard.int4_packed, device="cuda")
    else:
        want = ex.int4_maxsim(q, full.int4_packed, device="cuda")
        got = ex.int4_maxsim(q, shard.int4_packed, device="cuda")
    np.testing.assert_array_equal(got, want[:, lo:hi])
    with pytest.raises(ValueError, match="doc_range"):
        load_resident_corpus(path, doc_range=(5, 5))


def test_streamed_load_rejects_bad_token_scales(tmp_path):
    import maxsim_b200 as m

    path, _, _ = _saved(tmp_path, "int4_per_token")
    with np.load(path) as data:
        arrays = {k: data[k] for k in data.files}
    for bad in (-1.0, 0.0, np.inf, np.nan):
        arrays["int4_token_scale"] = arrays["int4_token_scale"].copy()
        arrays["int4_token_scale"][17] = bad
        broken = tmp_path / "broken.npz"
        np.savez_compressed(broken, **arrays)
        with pytest.raises(ValueError, match="token_scale values must be finite and > 0"):
            m.Reranker.load(broken, device="cuda")


def test_open_upload_refuses_to_score():
    from maxsim_b200 import _lib
    from maxsim_b200._maxsim_cuda import CudaInt4PackedDocs

    offsets = np.array([0, 3, 5], np.int64)
    h = CudaInt4PackedDocs._for_upload(offsets, 5, 128, 1.0, _lib.UPLOAD_TOKEN_SCALES)
    q = np.ones((1, 2, 128), np.float32)
    with pytest.raises(ValueError, match="upload has not finished"):
        h.topk_batch(q, 1)
    codes = np.zeros((5, 64), np.uint8)
    scales = np.ones(5, np.float32)
    t = np.zeros(1, np.int64)
    import ctypes

    ticket = ctypes.c_int64()
    _lib.check(_lib.lib.msb_docs_upload(h._h, _lib.ARRAY_CODES, 0, codes.ctypes.data, codes.nbytes,
                                        ctypes.byref(ticket)))
    with pytest.raises(ValueError, match="exceeds the array"):
        _lib.check(_lib.lib.msb_docs_upload(h._h, _lib.ARRAY_TOKEN_SCALES, 4, scales.ctypes.data, scales.nbytes,
                                            ctypes.byref(ticket)))
    _lib.check(_lib.lib.msb_docs_upload(h._h, _lib.ARRAY_TOKEN_SCALES, 0, scales.ctypes.data, scales.nbytes,
                                        ctypes.byref(ticket)))
    _lib.check(_lib.lib.msb_docs_upload_wait(h._h, ticket.value))
    _lib.check(_lib.lib.msb_docs_upload_finish(h._h, ctypes.c_float(1.0)))
    s, i = h.topk_batch(q, 1)
    assert s.shape == (1, 1) and float(s[0, 0]) == 0.0
    del t


def test_sharded_reranker_load_streams_each_rank_shard(tmp_path):
    import maxsim_b200 as m
    from maxsim_b200 import experimental as ex
    from maxsim_b200.sharded import ShardedReranker, shard_bounds

    path, _, q = _saved(tmp_path, "int4_per_token", docs=61)
    full = m.Reranker.load(path, device="cuda").corpus
    want = ex.int4_maxsim(q, full.int4_packed, device="cuda")
    bounds = shard_bounds(full.int4_packed.doc_offsets, 2)
    for rank in range(2):
        sr = ShardedReranker.load(path, rank=rank, world_size=2, chunk_bytes=3000)
        lo, hi = int(bounds[rank]), int(bounds[rank + 1])
        assert (sr.info.doc_lo, sr.info.doc_hi, sr.info.num_docs_total) == (lo, hi, 61)
        got = sr.local.maxsim_batch(q)
        np.testing.assert_array_equal(got, want[:, lo:hi])


@pytest.mark.parametrize("name,message", [("int4_data", "packed.values must be symmetric"),
                                          ("residual_int4_data", "residual_values must be symmetric")])
def test_streamed_load_rejects_minus_eight_like_the_host_path(tmp_path, name, message):
    import maxsim_b200 as m

    path, _, _ = _saved(tmp_path, "int4_residual")
    with np.load(path) as data:
        arrays = {k: data[k] for k in data.files}
    for byte in (0x08, 0x80, 0x8F):
        arrays[name] = arrays[name].copy()
        arrays[name][arrays[name].shape[0] - 1, 63] = byte  # the very last byte of the codes
        broken = tmp_path / "broken.npz"
        np.savez_compressed(broken, **arrays)
        with pytest.raises(ValueError, match=message):
            m.Index.load(broken)
        with pytest.raises(ValueError, match=message):
            m.Reranker.load(broken, device="cuda")
