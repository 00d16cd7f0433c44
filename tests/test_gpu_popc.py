"""The AND + popcount sign-code engine (engine 3) against the oracle and the other engines.

int8 queries: the bit-plane dot is the reference's integer dot (sum of +-q), so
scores equal the oracle's restatement of maxsim_binary_int8q_dim128_kernel bit
for bit, with and without per-token scales and per-document scales.  fp32
queries: rows as the 23-bit fixed-point integers of the tensor-core digit
planes, so scores equal the tensor-core engine's bit for bit (scalar document
scale) and the reference's fp32 sums within 1e-4; weighted MaxSim folds the
weights into the row scales as the tensor-core engine does.  Ragged corpora with
empty and one-token documents, query lengths 1..32, batches that leave a warp's
query group partly empty, and candidate lists.
"""

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


def _corpus(seed, num_docs=300):
    rng = np.random.default_rng(seed)
    kinds = rng.integers(0, 8, size=num_docs)
    lengths = np.where(kinds == 0, 0, np.where(kinds == 1, 1, rng.integers(2, 180, size=num_docs)))
    off = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    docs = rng.standard_normal((int(off[-1]), 128)).astype(np.float32)
    return rng, docs, off


def _handle(docs, off, token_scale=None, doc_scale=None):
    from maxsim_b200 import _maxsim_cuda as mc

    h = mc.CudaPackedDocs(ref.pack_signs(docs), off, 128)
    if token_scale is not None:
        h.set_token_scale_vector(token_scale)
    if doc_scale is not None:
        h.set_scale_vector(doc_scale)
    return h


@pytest.mark.parametrize("batch,qtok", [(1, 20), (3, 24), (5, 7), (2, 32), (4, 1)])
@pytest.mark.parametrize("scales", ["none", "token", "token+doc"])
def test_popc_int8_queries_bit_exact(batch, qtok, scales):
    rng, docs, off = _corpus(100 + batch * 31 + qtok)
    D, N = len(off) - 1, int(off[-1])
    ts = rng.uniform(0.25, 2.0, size=N).astype(np.float16).astype(np.float32) if scales != "none" else None
    ds = rng.uniform(0.5, 1.5, size=D).astype(np.float32) if scales == "token+doc" else None
    h = _handle(docs, off, ts, ds)
    q = rng.standard_normal((batch, qtok, 128)).astype(np.float32)
    use_ts, use_ds = ts is not None, ds is not None
    got = _engine(3, lambda: h.maxsim_batch_int8q(q, 1.0, use_ds, use_ts))
    want = ref.score_binary_int8q(q, ref.pack_signs(docs), off, token_scale=ts,
                                  doc_scale=ds if use_ds else 1.0)
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal(got, _engine(1, lambda: h.maxsim_batch_int8q(q, 1.0, use_ds, use_ts)))


@pytest.mark.parametrize("batch,qtok", [(1, 20), (3, 24), (2, 32), (6, 5)])
@pytest.mark.parametrize("token_scale", [False, True])
def test_popc_fp32_queries_equal_the_tensor_core_engine(batch, qtok, token_scale):
    rng, docs, off = _corpus(200 + batch * 7 + qtok)
    N = int(off[-1])
    # 4-bit log-coded style scales: powers of two times a few mantissas
    ts = (2.0 ** rng.integers(-3, 3, size=N) * rng.choice([1.0, 1.25, 1.5], size=N)).astype(np.float32)
    h = _handle(docs, off, ts if token_scale else None)
    q = rng.standard_normal((batch, qtok, 128)).astype(np.float32)
    q[0, 0] = 0.0  # an all-zero row
    got = _engine(3, lambda: h.maxsim_batch(q, 0.75, False, token_scale))
    tc = _engine(2, lambda: h.maxsim_batch(q, 0.75, False, token_scale))
    np.testing.assert_array_equal(got, tc)
    want = ref.score_binary_fp32(q, ref.pack_signs(docs), 128, off, token_scale=ts if token_scale else None,
                                 doc_scale=0.75)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)


def test_popc_weighted_and_candidates():
    rng, docs, off = _corpus(300)
    D, N = len(off) - 1, int(off[-1])
    ts = rng.uniform(0.5, 1.5, size=N).astype(np.float32)
    h = _handle(docs, off, ts)
    q = rng.standard_normal((3, 20, 128)).astype(np.float32)
    w = rng.uniform(0.5, 1.5, size=20).astype(np.float32)
    got = _engine(3, lambda: h.score_batch(q, "weighted_maxsim", w, use_token_scale=True))
    tc = _engine(2, lambda: h.score_batch(q, "weighted_maxsim", w, use_token_scale=True))
    np.testing.assert_array_equal(got, tc)
    cands = np.sort(rng.choice(D, size=40, replace=False)).astype(np.int64)
    gc = _engine(3, lambda: h.score_candidates_batch(q, cands, use_token_scale=True))
    full = _engine(3, lambda: h.score_batch(q, use_token_scale=True))
    np.testing.assert_array_equal(gc, full[:, cands])
    want = ref.score_binary_fp32(q, ref.pack_signs(docs), 128, off, token_scale=ts)
    np.testing.assert_allclose(full, want, rtol=RTOL, atol=ATOL)
