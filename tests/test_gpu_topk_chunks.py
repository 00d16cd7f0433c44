"""Two-stage top-k over few long rows: chunks of a row selected by separate blocks, then merged.

A full-scan top-k of a handle with at least 32,768 documents and a small batch splits each score row into
chunks of about 2,048 documents (every chunk at least k long); each block selects its chunk's top-k
(score desc, id asc) and the shard merge kernel forms the row's top-k.  Ids and scores must equal the
oracle's top-k of the whole row exactly, with exact ties placed in different chunks (duplicated
documents), empty documents (score 0) among negative scores, and k from 1 to 700.
"""

import ctypes

import numpy as np
import pytest

from oracle import reference_cpu as ref

pytestmark = pytest.mark.gpu


def _oracle(oracle_c, q, packed, off):
    B, Q, dim = q.shape
    D = len(off) - 1
    codes, qs = ref.quantize_query_int8(q.reshape(-1, dim))
    out = np.empty((B, D), np.float32)
    oracle_c.oracle_int4_int8q_scores(
        codes.ctypes.data_as(ctypes.c_void_p), qs.ctypes.data_as(ctypes.c_void_p), B, Q, dim,
        packed.data.ctypes.data_as(ctypes.c_void_p), packed.token_scale.ctypes.data_as(ctypes.c_void_p),
        ctypes.c_float(packed.scale), off.ctypes.data_as(ctypes.c_void_p), ctypes.c_int64(D), None, ctypes.c_int64(0),
        out.ctypes.data_as(ctypes.c_void_p), 8)
    return out


@pytest.mark.parametrize("batch,k", [(1, 1), (1, 10), (3, 37), (2, 700)])
def test_chunked_topk_equals_the_oracle(oracle_c, batch, k):
    import maxsim_b200 as m

    rng = np.random.default_rng(900 + k)
    num_docs = 40000
    lengths = rng.integers(1, 12, size=num_docs)
    lengths[[11, 4000, 37000]] = 0  # empty documents: score 0
    dups = [9001, 25002, 39998]  # copies of document 5 in other chunks: exact ties across chunks
    lengths[dups] = lengths[5]
    off = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    docs = rng.standard_normal((int(off[-1]), 128)).astype(np.float32)
    for d in dups:
        docs[off[d]:off[d + 1]] = docs[off[5]:off[6]]
    q = rng.standard_normal((batch, 16, 128)).astype(np.float32)
    q[:, :2] = docs[off[5]:off[5] + 1]  # the duplicated documents rank at the top
    packed = m.pack_int4_symmetric(docs, off, scale_granularity="token")
    h = m.int4_to_device(packed).data
    want_s, want_i = ref.topk_rows(_oracle(oracle_c, q, packed, off), k)
    s, i = h.topk_batch_int8q(q, k)
    np.testing.assert_array_equal(i, want_i)
    np.testing.assert_array_equal(s, want_s)
