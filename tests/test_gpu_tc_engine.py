"""Tensor-core engine parity: tcgen05 scan vs the exact oracle and vs the SIMT engine.

int8-query x int4 scores are exact integer dots followed by the reference
kernel's fp32 epilogue, so both engines must agree bit for bit with the C
oracle on ragged corpora that exercise tile and work-range boundaries: empty
documents, one-token documents, documents longer than a work range, query
batches that do not fill the last query tile and query lengths 1..128.
"""

import ctypes

import numpy as np
import pytest

from oracle import reference_cpu as ref

pytestmark = pytest.mark.gpu


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


def _ragged(rng, num_docs, lengths=None):
    if lengths is None:
        kinds = rng.integers(0, 10, size=num_docs)
        lengths = np.where(kinds == 0, 0, np.where(kinds == 1, 1, np.where(kinds == 9, rng.integers(200, 3000, size=num_docs),
                                                                            rng.integers(2, 160, size=num_docs))))
    off = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    docs = rng.standard_normal((int(off[-1]), 128)).astype(np.float32)
    return docs, off


def _run(engine, fn):
    from maxsim_b200 import _lib

    prev = _lib.get_engine()
    _lib.set_engine(engine)
    try:
        return fn()
    finally:
        _lib.set_engine(prev)


@pytest.fixture(autouse=True, params=[(1, 1), (0, 1), (0, 0)], ids=["f16-copy", "int8-copy", "expand"])
def tc_operands(request):
    """Run every test with each tensor-core operand path: f16 tiles streamed by TMA from the resident f16
    copy of the corpus (per-token scales only; fp32 accumulators), int8 tiles from the resident int8
    copy, and raw int4 rows expanded in shared memory per tile.  Handles built in a test start with
    the setting of that test."""
    from maxsim_b200 import _lib

    prev = (_lib.get_option("tc_f16_cache"), _lib.get_option("tc_int8_cache"))
    _lib.set_option("tc_f16_cache", request.param[0])
    _lib.set_option("tc_int8_cache", request.param[1])
    yield request.param
    _lib.set_option("tc_f16_cache", prev[0])
    _lib.set_option("tc_int8_cache", prev[1])


@pytest.mark.parametrize("gran", ["token", "tensor"])
@pytest.mark.parametrize("batch,qtok", [(1, 1), (3, 24), (11, 24), (12, 24), (23, 24), (4, 32), (2, 100), (2, 128),
                                        (7, 20)])
def test_tc_int8_scores_exact(oracle_c, gran, batch, qtok):
    import maxsim_b200 as m

    rng = np.random.default_rng(1000 + batch * 7 + qtok)
    docs, off = _ragged(rng, 300)
    q = rng.standard_normal((batch, qtok, 128)).astype(np.float32)
    q[0, -1] = 0.0
    packed = m.pack_int4_symmetric(docs, off, scale_granularity=gran)
    dev = m.int4_to_device(packed)
    want = _oracle_scores(oracle_c, q, packed.data, packed.token_scale, packed.scale, off)
    tc = _run(2, lambda: dev.data.maxsim_batch_int8q(q))
    simt = _run(1, lambda: dev.data.maxsim_batch_int8q(q))
    np.testing.assert_array_equal(simt, want)
    np.testing.assert_array_equal(tc, want)


@pytest.mark.parametrize("gran", ["token", "tensor"])
def test_tc_topk_exact_on_clustered_corpus(oracle_c, gran):
    import maxsim_b200 as m

    docs, off = ref.clustered_corpus(2000, 64, 192, seed=0)
    q = ref.clustered_queries(docs, off, 4, 32, seed=1)
    packed = m.pack_int4_symmetric(docs, off, scale_granularity=gran)
    dev = m.int4_to_device(packed)
    full = _oracle_scores(oracle_c, q, packed.data, packed.token_scale, packed.scale, off)
    want_s, want_i = ref.topk_rows(full, 10)
    s, i = _run(2, lambda: dev.data.topk_batch_int8q(q, 10))
    np.testing.assert_array_equal(i, want_i)
    np.testing.assert_array_equal(s, want_s)


def test_tc_repeat_calls_identical_and_workspace_reused():
    import maxsim_b200 as m

    rng = np.random.default_rng(77)
    docs, off = _ragged(rng, 500)
    dev = m.int4_to_device(m.pack_int4_symmetric(docs, off, scale_granularity="token"))
    q1 = rng.standard_normal((9, 24, 128)).astype(np.float32)
    q2 = rng.standard_normal((2, 5, 128)).astype(np.float32)
    a = _run(2, lambda: dev.data.maxsim_batch_int8q(q1))
    b = _run(2, lambda: dev.data.maxsim_batch_int8q(q2))
    c = _run(2, lambda: dev.data.maxsim_batch_int8q(q1))
    np.testing.assert_array_equal(a, c)
    np.testing.assert_array_equal(b, _run(1, lambda: dev.data.maxsim_batch_int8q(q2)))
