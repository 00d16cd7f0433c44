"""Replicated query rows (option ``tc_row_replicas``) against the oracle and the unreplicated kernel.

A pass whose int8 query rows fit one tile of at most 32 (64) rows copies them
four (two) times over the TMEM lane quarters; each epilogue warp then takes one
slice of 32 (64) columns of every token tile and a document's row maximum is
completed across the copies when the document is flushed.  The scores must
equal the C oracle's restatement of the reference kernel bit for bit, and the
unreplicated kernel's, on ragged corpora (empty, one-token and multi-tile
documents: ends that fall before, inside and after a warp's slice) with the
boundaries of both replication factors (32 / 33 and 64 / 65 rows), on both
operand paths (int8 copy by TMA, int4 rows expanded in shared memory), with
per-token scales (biased and unbiased accumulators) and a tensor scale, for
sign codes, for the top-k entry point and for the fused top-k.
"""

import ctypes

import numpy as np
import pytest

from oracle import reference_cpu as ref

pytestmark = pytest.mark.gpu

SHAPES = [(1, 1), (1, 24), (1, 32), (4, 8), (1, 33), (2, 24), (2, 32), (3, 21), (5, 13), (1, 96)]


def _oracle_scores(oracle_c, q, values_packed, token_scale, scale, off):
    B, Q, dim = q.shape
    D = len(off) - 1
    codes, qs = ref.quantize_query_int8(q.reshape(-1, dim))
    out = np.empty((B, D), np.float32)
    oracle_c.oracle_int4_int8q_scores(
        codes.ctypes.data_as(ctypes.c_void_p), qs.ctypes.data_as(ctypes.c_void_p), B, Q, dim,
        values_packed.ctypes.data_as(ctypes.c_void_p),
        None if token_scale is None else token_scale.ctypes.data_as(ctypes.c_void_p), ctypes.c_float(scale),
        off.ctypes.data_as(ctypes.c_void_p), ctypes.c_int64(D), None, ctypes.c_int64(0),
        out.ctypes.data_as(ctypes.c_void_p), 8)
    return out


def _ragged(rng, num_docs):
    """Empty, one-token, short and multi-tile documents."""
    kinds = rng.integers(0, 10, size=num_docs)
    lengths = np.where(kinds == 0, 0, np.where(kinds == 1, 1, np.where(kinds == 9, rng.integers(200, 3000, size=num_docs),
                                                                        rng.integers(2, 160, size=num_docs))))
    off = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    docs = rng.standard_normal((int(off[-1]), 128)).astype(np.float32)
    return docs, off


def _options(**kv):
    from maxsim_b200 import _lib

    prev = {k: _lib.get_option(k) for k in kv}
    for k, v in kv.items():
        _lib.set_option(k, v)
    return prev


@pytest.fixture(params=[1, 0], ids=["int8-copy", "expand"])
def tc_path(request):
    """The tensor-core engine on either operand path, replication on."""
    from maxsim_b200 import _lib

    prev_engine = _lib.get_engine()
    prev = _options(tc_int8_cache=request.param, tc_f16_cache=0, tc_row_replicas=1)
    _lib.set_engine(2)
    yield request.param
    _lib.set_engine(prev_engine)
    _options(**prev)


def _unreplicated(fn):
    prev = _options(tc_row_replicas=0)
    try:
        return fn()
    finally:
        _options(**prev)


@pytest.mark.parametrize("gran", ["token", "tensor", "token-large"])
@pytest.mark.parametrize("batch,qtok", SHAPES)
def test_replicated_rows_int4_exact(oracle_c, tc_path, gran, batch, qtok):
    import maxsim_b200 as m

    rng = np.random.default_rng(4000 + 13 * batch + qtok)
    docs, off = _ragged(rng, 400)
    q = rng.standard_normal((batch, qtok, 128)).astype(np.float32)
    packed = m.pack_int4_symmetric(docs, off, scale_granularity="tensor" if gran == "tensor" else "token")
    if gran == "token-large":
        # a token scale of 2^110 keeps the unbiased accumulators (s * 2^23 would not be exact)
        packed.token_scale[rng.choice(packed.token_scale.shape[0], size=50, replace=False)] = np.float32(2.0 ** 110)
    dev = m.int4_to_device(packed)
    want = _oracle_scores(oracle_c, q, packed.data, packed.token_scale, packed.scale, off)
    got = dev.data.maxsim_batch_int8q(q)
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal(_unreplicated(lambda: dev.data.maxsim_batch_int8q(q)), got)


@pytest.mark.parametrize("batch,qtok", [(1, 20), (1, 32), (2, 30), (3, 20)])
@pytest.mark.parametrize("token_scale", [False, True])
def test_replicated_rows_sign_codes_exact(tc_path, batch, qtok, token_scale):
    from maxsim_b200 import _maxsim_cuda as mc

    rng = np.random.default_rng(77 + batch * qtok)
    lengths = np.where(rng.integers(0, 8, size=300) == 0, 0, rng.integers(1, 300, size=300))
    off = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    docs = rng.standard_normal((int(off[-1]), 128)).astype(np.float32)
    ts = rng.uniform(0.5, 2.0, size=docs.shape[0]).astype(np.float16).astype(np.float32) if token_scale else None
    h = mc.CudaPackedDocs(ref.pack_signs(docs), off, 128)
    if ts is not None:
        h.set_token_scale_vector(ts)
    q = rng.standard_normal((batch, qtok, 128)).astype(np.float32)
    want = ref.score_binary_int8q(q, ref.pack_signs(docs), off, token_scale=ts)
    got = h.maxsim_batch_int8q(q, 1.0, False, token_scale)
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal(_unreplicated(lambda: h.maxsim_batch_int8q(q, 1.0, False, token_scale)), got)


@pytest.mark.parametrize("fused", [0, 1])
def test_replicated_rows_topk_exact(oracle_c, tc_path, fused):
    import maxsim_b200 as m

    docs, off = ref.clustered_corpus(3000, 64, 400, seed=11)
    q = ref.clustered_queries(docs, off, 2, 24, seed=12)
    packed = m.pack_int4_symmetric(docs, off, scale_granularity="token")
    dev = m.int4_to_device(packed)
    full = _oracle_scores(oracle_c, q, packed.data, packed.token_scale, packed.scale, off)
    prev = _options(tc_fused_topk=fused)
    try:
        for b in (1, 2):  # 24 rows: four copies; 48 rows: two
            want_s, want_i = ref.topk_rows(full[:b], 10)
            s, i = dev.data.topk_batch_int8q(q[:b], 10)
            np.testing.assert_array_equal(i, want_i)
            np.testing.assert_array_equal(s, want_s)
    finally:
        _options(**prev)
