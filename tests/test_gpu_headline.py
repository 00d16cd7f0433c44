"""Parity at the benchmark's own geometry, bit for bit against the C oracle.

``bench.py`` times 64 queries x 24 tokens (int8 per row) against 1,030-token
pages through the default tensor-core path: the resident int8 copy of the
codes read by tiled TMA, biased accumulators (per-token scales), 13 query
tiles of 5 queries (6 full tile pairs, then the 13th tile in a twin-mode launch
of its own) and 2 x SM-count document ranges.  The tests here run that geometry on 2,048 pages and require
the whole score matrix and the top-10 ids and scores to equal the C oracle's
restatement of the reference kernel exactly (the int8 x int4 dots are
integers; the fp32 epilogue is the reference's).  They also pin the variant
chosen for token scales too large for the biased accumulators, and token
scales at the extremes of the fp32 range.
"""

import ctypes
import os

import numpy as np
import pytest

from oracle import reference_cpu as ref

pytestmark = pytest.mark.gpu

PAGE_TOKENS = 1030
DIM = 128


def _pages(n_pages, seed):
    """Per-page Gaussian centroid + N(0, 0.3^2) patch noise, L2-normalised, packed per-token int4
    (chunked, so the fp32 tokens never exist all at once)."""
    rng = np.random.default_rng(seed)
    cent = rng.standard_normal((n_pages, DIM)).astype(np.float32)
    cent /= np.linalg.norm(cent, axis=1, keepdims=True)
    n_tok = n_pages * PAGE_TOKENS
    codes = np.empty((n_tok, DIM // 2), np.uint8)
    scales = np.empty(n_tok, np.float32)
    for p0 in range(0, n_pages, 128):
        p1 = min(n_pages, p0 + 128)
        x = np.repeat(cent[p0:p1], PAGE_TOKENS, axis=0)
        x += np.float32(0.3) * rng.standard_normal(x.shape, dtype=np.float32)
        x /= np.linalg.norm(x, axis=1, keepdims=True)
        data, _, _, ts = ref.pack_int4(x, "token")
        codes[p0 * PAGE_TOKENS:p1 * PAGE_TOKENS] = data
        scales[p0 * PAGE_TOKENS:p1 * PAGE_TOKENS] = ts
    off = np.arange(n_pages + 1, dtype=np.int64) * PAGE_TOKENS
    return codes, scales, off, cent


def _queries(cent, batch, qtok, seed):
    rng = np.random.default_rng(seed)
    targets = rng.integers(0, cent.shape[0], size=batch)
    q = np.repeat(cent[targets][:, None, :], qtok, axis=1)
    q = q + np.float32(0.3) * rng.standard_normal(q.shape, dtype=np.float32)
    return (q / np.linalg.norm(q, axis=2, keepdims=True)).astype(np.float32)


def _oracle(oracle_c, q, codes, token_scale, scale, off):
    B, Q, _ = q.shape
    D = len(off) - 1
    qc, qs = ref.quantize_query_int8(q.reshape(-1, DIM))
    out = np.empty((B, D), np.float32)
    rc = oracle_c.oracle_int4_int8q_scores_docs(
        qc.ctypes.data_as(ctypes.c_void_p), qs.ctypes.data_as(ctypes.c_void_p), B, Q, DIM,
        codes.ctypes.data_as(ctypes.c_void_p),
        None if token_scale is None else token_scale.ctypes.data_as(ctypes.c_void_p), ctypes.c_float(scale),
        off.ctypes.data_as(ctypes.c_void_p), ctypes.c_int64(D), None, ctypes.c_int64(0),
        out.ctypes.data_as(ctypes.c_void_p), os.cpu_count() or 1)
    assert rc == 0
    return out


@pytest.fixture
def default_engine():
    """The routing bench.py measures: automatic engine choice, int8 copy on, f16 copy off."""
    from maxsim_b200 import _lib

    prev = (_lib.get_engine(), _lib.get_option("tc_int8_cache"), _lib.get_option("tc_f16_cache"))
    _lib.set_engine(0)
    _lib.set_option("tc_int8_cache", 1)
    _lib.set_option("tc_f16_cache", 0)
    yield
    _lib.set_engine(prev[0])
    _lib.set_option("tc_int8_cache", prev[1])
    _lib.set_option("tc_f16_cache", prev[2])


def test_headline_geometry_bit_exact(oracle_c, default_engine):
    from maxsim_b200 import _maxsim_cuda as mc

    codes, scales, off, cent = _pages(2048, seed=20260713)
    q = _queries(cent, 64, 24, seed=20260714)
    h = mc.CudaInt4PackedDocs(codes, off, DIM, 1.0)
    h.set_token_scale_vector(scales)
    want = _oracle(oracle_c, q, codes, scales, 1.0, off)
    got = h.maxsim_batch_int8q(q)
    np.testing.assert_array_equal(got, want)
    s, i = h.topk_batch_int8q(q, 10)
    want_s, want_i = ref.topk_rows(want, 10)
    np.testing.assert_array_equal(i, want_i)
    np.testing.assert_array_equal(s, want_s)
    # a second batch through the same workspace (cached work units) and a batch of one query
    q2 = _queries(cent, 64, 24, seed=20260715)
    np.testing.assert_array_equal(h.maxsim_batch_int8q(q2), _oracle(oracle_c, q2, codes, scales, 1.0, off))
    np.testing.assert_array_equal(h.maxsim_batch_int8q(q[:1]), want[:1])


@pytest.mark.parametrize("extreme", ["large_small", "too_large", "subnormal"])
def test_token_scale_extremes_exact(oracle_c, default_engine, extreme):
    """Token scales below 2^104 keep the biased accumulators (s * 2^23 exact, also for subnormal s);
    a corpus holding a larger one is scanned by the unbiased variant.  Both equal the oracle."""
    from maxsim_b200 import _maxsim_cuda as mc

    rng = np.random.default_rng(5)
    lengths = rng.integers(1, 400, size=300)
    off = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    docs = rng.standard_normal((int(off[-1]), DIM)).astype(np.float32)
    codes, _, _, scales = ref.pack_int4(docs, "token")
    scales = scales.copy()
    pick = rng.choice(scales.shape[0], size=scales.shape[0] // 10, replace=False)
    if extreme == "large_small":
        scales[pick] = np.float32(2.0 ** 103) * rng.uniform(1.0, 1.99, size=pick.shape[0]).astype(np.float32)
        scales[pick[::2]] = np.float32(3e-30)
    elif extreme == "too_large":
        scales[pick] = np.float32(2.0 ** 110)
    else:
        scales[pick] = np.float32(1e-41)  # subnormal
    q = rng.standard_normal((7, 20, DIM)).astype(np.float32)
    h = mc.CudaInt4PackedDocs(codes, off, DIM, 1.0)
    h.set_token_scale_vector(scales)
    want = _oracle(oracle_c, q, codes, scales, 1.0, off)
    np.testing.assert_array_equal(h.maxsim_batch_int8q(q), want)
    # replacing the scales re-checks their range: back to ordinary scales
    _, _, _, plain = ref.pack_int4(docs, "token")
    h.set_token_scale_vector(plain)
    np.testing.assert_array_equal(h.maxsim_batch_int8q(q), _oracle(oracle_c, q, codes, plain, 1.0, off))
