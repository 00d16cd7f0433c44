"""fp32 queries on the tensor-core engine: int8 digit planes of the query (dim 128, int4 and sign codes).

Each query row is scaled by 2^S so that its largest magnitude lies in [2^21, 2^22], rounded to
integers and split into three signed base-256 digits; the engine's int8 MMAs give each digit plane's
dot with a token exactly, and the epilogue combines them as fl(65536 d2 + fl(d0 + 256 d1)) (one fused
multiply-add), multiplies by the token scale, takes the maxima, scales them back by 2^-S and sums the
rows in order.  ``_digit_model`` restates that arithmetic in numpy, so the engine must match it bit for
bit; against the reference's fp32 scoring (the float64 oracle) the only error is the query's rounding
to 23 bits and the one rounding of each dot, far inside the fp32 paths' 1e-4 tolerance.

The same holds, each with its own restatement, for sign-code corpora (a +-1 int8 copy), weighted
MaxSim (weights folded into the row scales), the fused residual streams (two accumulators per query
tile, int4 or sign-code prefix), the TopK2 / TopK4 reducers (per-row lists merged across threads),
and candidate lists long enough to be gathered from a full scan.
"""

import numpy as np
import pytest

from oracle import reference_cpu as ref

pytestmark = pytest.mark.gpu


@pytest.fixture
def engine():
    from maxsim_b200 import _lib

    prev = _lib.get_engine()
    yield _lib
    _lib.set_engine(prev)


def _digits(q):
    """[R, 128] fp32 -> (three int64 digit planes [3, R, 128], qscale [R] fp32)."""
    q = np.asarray(q, np.float32)
    m = np.abs(q).max(axis=1)
    _, e = np.frexp(m)
    s = np.where(m > 0, np.minimum(22 - e, 149), 0).astype(np.int64)
    qi = np.rint(np.ldexp(q, s[:, None]).astype(np.float32)).astype(np.int64)
    d0 = ((qi + 128) & 255) - 128
    r1 = (qi - d0) >> 8
    d1 = ((r1 + 128) & 255) - 128
    d2 = (r1 - d1) >> 8
    assert np.array_equal(d0 + 256 * d1 + 65536 * d2, qi) and np.abs(d2).max() <= 65
    return np.stack([d0, d1, d2]), np.ldexp(np.float32(1), -s).astype(np.float32)


def _digit_model(query, values, offsets, scale, token_scale, weights=None):
    """The engine's arithmetic for [B, Q, 128] fp32 queries against int4 values [N, 128]; weighted
    MaxSim folds each row's weight into its power-of-two scale (exact)."""
    B, Q, _ = query.shape
    digits, qscale = _digits(query.reshape(-1, 128))
    if weights is not None:
        w = np.broadcast_to(np.asarray(weights, np.float32), (B, Q)).reshape(-1)
        qscale = np.ldexp(w, np.frexp(qscale)[1] - 1).astype(np.float32)  # w * 2^-S
    vals = values.astype(np.int64)
    dots = np.einsum("kri,ti->krt", digits, vals)  # exact integers
    lo = (dots[0] + 256 * dots[1]).astype(np.float32)
    v = (dots[2].astype(np.float64) * 65536.0 + lo.astype(np.float64)).astype(np.float32)
    if token_scale is not None:
        v = v * np.asarray(token_scale, np.float32)[None, :]
    D = offsets.shape[0] - 1
    out = np.zeros((B, D), np.float32)
    for d in range(D):
        a, b = offsets[d], offsets[d + 1]
        if a == b:
            continue
        best = v[:, a:b].max(axis=1) * qscale  # [B * Q], exact power-of-two scaling
        for bi in range(B):
            acc = np.float32(0)
            for r in range(Q):
                acc = np.float32(acc + best[bi * Q + r])
            out[bi, d] = np.float32(acc * np.float32(scale))
    return out


def _corpus(num_docs, max_len, seed):
    docs, off = ref.clustered_corpus(num_docs, 0, max_len, seed=seed)
    return docs, off


@pytest.mark.parametrize("gran", ["tensor", "token"])
@pytest.mark.parametrize("batch,qtok", [(1, 32), (5, 20), (3, 7), (9, 1)])
def test_digit_planes_bit_exact_and_within_oracle(engine, gran, batch, qtok):
    import maxsim_b200 as m

    docs, off = _corpus(300, 300, seed=batch * 7 + qtok)
    q = ref.clustered_queries(docs, off, batch, qtok, seed=qtok)
    packed = m.pack_int4_symmetric(docs, off, scale_granularity=gran)
    dev = m.int4_to_device(packed)
    engine.set_engine(2)  # the tensor-core engine, or an error
    got = m.int4_maxsim(q, dev)
    want = _digit_model(q, packed.values, off, packed.scale, packed.token_scale)
    np.testing.assert_array_equal(got, want)
    exact = ref.score_int4_fp32(q, packed.values, off, scale=packed.scale, token_scale=packed.token_scale)
    np.testing.assert_allclose(got, exact, rtol=2e-6, atol=2e-6 * np.abs(exact).max())
    engine.set_engine(1)
    simt = m.int4_maxsim(q, dev)
    np.testing.assert_allclose(got, simt, rtol=1e-5, atol=1e-5 * np.abs(exact).max())
    engine.set_engine(0)
    s, i = m.topk_int4_maxsim(q, dev, 10)
    for row in range(batch):
        np.testing.assert_array_equal(s[row], np.sort(got[row])[::-1][:10])


@pytest.mark.parametrize("batched", [False, True])
@pytest.mark.parametrize("binary", [False, True])
def test_weighted_maxsim_on_digit_planes(engine, batched, binary):
    """Weighted MaxSim of fp32 queries: the row weights fold into the digit planes' row scales."""
    import maxsim_b200 as m

    docs, off = _corpus(200, 240, seed=31)
    q = ref.clustered_queries(docs, off, 3, 24, seed=32)
    rng = np.random.default_rng(33)
    w = rng.uniform(0.25, 2.0, size=(3, 24) if batched else 24).astype(np.float32)
    if binary:
        packed, h = _binary(docs, off, True)
        values = ref.unpack_signs(packed.data, 128).astype(np.int64)
        ts, scale = np.asarray(packed.token_scale, np.float32), 1.0
        run = lambda: h.score_batch(q, reducer="weighted_maxsim", query_weights=w, use_token_scale=True)
        exact = ref.score_binary_fp32(q, packed.data, 128, off, token_scale=ts, reducer="weighted_maxsim", weights=w)
    else:
        packed = m.pack_int4_symmetric(docs, off, scale_granularity="token")
        dev = m.int4_to_device(packed)
        values, ts, scale = packed.values, packed.token_scale, packed.scale
        run = lambda: m.int4_maxsim(q, dev, reducer="weighted_maxsim", query_weights=w)
        exact = ref.score_int4_fp32(q, packed.values, off, scale=scale, token_scale=ts, reducer="weighted_maxsim",
                                    weights=w)
    engine.set_engine(2)
    got = run()
    np.testing.assert_array_equal(got, _digit_model(q, values, off, scale, ts, weights=w))
    np.testing.assert_allclose(got, exact, rtol=2e-6, atol=2e-6 * np.abs(exact).max())
    engine.set_engine(1)
    np.testing.assert_allclose(run(), got, rtol=1e-5, atol=1e-5 * np.abs(exact).max())


def test_digit_planes_extreme_row_magnitudes(engine):
    """Rows of 1e-30 and 1e30 magnitude, a zero row and a one-hot row keep their relative precision."""
    import maxsim_b200 as m

    docs, off = _corpus(120, 80, seed=5)
    q = ref.clustered_queries(docs, off, 2, 8, seed=6).astype(np.float32)
    q[0, 1] *= np.float32(1e-30)
    q[0, 2] *= np.float32(1e30)
    q[1, 3] = 0.0
    q[1, 4] = 0.0
    q[1, 4, 17] = -0.25
    packed = m.pack_int4_symmetric(docs, off, scale_granularity="token")
    dev = m.int4_to_device(packed)
    engine.set_engine(2)
    got = m.int4_maxsim(q, dev)
    np.testing.assert_array_equal(got, _digit_model(q, packed.values, off, packed.scale, packed.token_scale))
    exact = ref.score_int4_fp32(q, packed.values, off, scale=packed.scale, token_scale=packed.token_scale)
    np.testing.assert_allclose(got, exact, rtol=2e-6, atol=0)


def test_digit_planes_large_corpus_many_units(engine):
    """About 330k tokens: many work units per CTA, documents crossing tiles and units."""
    import maxsim_b200 as m

    docs, off = _corpus(3000, 220, seed=9)
    q = ref.clustered_queries(docs, off, 4, 32, seed=10)
    packed = m.pack_int4_symmetric(docs, off, scale_granularity="token")
    dev = m.int4_to_device(packed)
    engine.set_engine(2)
    got = m.int4_maxsim(q, dev)
    np.testing.assert_array_equal(got, _digit_model(q, packed.values, off, packed.scale, packed.token_scale))


def test_fp32_scans_outside_the_digit_path_stay_simt(engine):
    """33 query tokens, or a query pointer that is not 16-byte aligned, run on the SIMT engine."""
    import torch
    import maxsim_b200 as m

    docs, off = _corpus(60, 50, seed=3)
    packed = m.pack_int4_symmetric(docs, off, scale_granularity="token")
    dev = m.int4_to_device(packed)
    q33 = ref.clustered_queries(docs, off, 2, 33, seed=4)
    engine.set_engine(1)
    want = m.int4_maxsim(q33, dev)
    engine.set_engine(0)
    np.testing.assert_array_equal(m.int4_maxsim(q33, dev), want)
    engine.set_engine(2)
    with pytest.raises(NotImplementedError):
        m.int4_maxsim(q33, dev)

    h = dev.data
    q = ref.clustered_queries(docs, off, 2, 16, seed=5)
    buf = torch.zeros(q.size + 4, dtype=torch.float32, device="cuda")
    view = buf[1:1 + q.size].view(q.shape)
    view.copy_(torch.from_numpy(q))
    out = torch.empty(2, h.num_docs, device="cuda")
    engine.set_engine(0)
    h.score_batch_device(view, out)
    torch.cuda.synchronize()
    engine.set_engine(1)
    np.testing.assert_array_equal(out.cpu().numpy(), m.int4_maxsim(q, dev))


# ---------------------------------------------------------------------------
# Sign-code corpora: the engine reads a resident +-1 int8 copy of the codes
# ---------------------------------------------------------------------------

def _binary(docs, off, token_scale):
    import maxsim_b200 as m

    kw = {"token_scale": "mean_abs_fp16"} if token_scale else {}
    packed = m.pack_signs(docs, off, **kw)
    return packed, m.to_device(packed, "cuda").data


@pytest.mark.parametrize("token_scale", [False, True])
@pytest.mark.parametrize("batch,qtok", [(1, 20), (6, 32), (4, 5)])
def test_binary_digit_planes_bit_exact(engine, token_scale, batch, qtok):
    docs, off = _corpus(250, 260, seed=batch + qtok)
    q = ref.clustered_queries(docs, off, batch, qtok, seed=qtok + 1)
    packed, h = _binary(docs, off, token_scale)
    signs = ref.unpack_signs(packed.data, 128).astype(np.int64)
    ts = np.asarray(packed.token_scale, np.float32) if token_scale else None
    engine.set_engine(2)
    got = h.score_batch(q, scale=0.75, use_token_scale=token_scale)
    np.testing.assert_array_equal(got, _digit_model(q, signs, off, 0.75, ts))
    exact = ref.score_binary_fp32(q, packed.data, 128, off, token_scale=ts, doc_scale=0.75)
    np.testing.assert_allclose(got, exact, rtol=2e-6, atol=2e-6 * np.abs(exact).max())
    s, i = h.topk_batch(q, 7, scale=0.75, use_token_scale=token_scale)
    for row in range(batch):
        np.testing.assert_array_equal(s[row], np.sort(got[row])[::-1][:7])


@pytest.mark.parametrize("token_scale", [False, True])
def test_binary_int8_queries_tensor_core_equals_simt(engine, token_scale):
    """int8 queries: both engines compute the exact integer dot with +-1, so the scores are identical."""
    docs, off = _corpus(300, 200, seed=21)
    q = ref.clustered_queries(docs, off, 5, 32, seed=22)
    _, h = _binary(docs, off, token_scale)
    engine.set_engine(2)
    got = h.maxsim_batch_int8q(q, scale=1.5, use_token_scale=token_scale)
    engine.set_engine(1)
    want = h.maxsim_batch_int8q(q, scale=1.5, use_token_scale=token_scale)
    np.testing.assert_array_equal(got, want)


def test_binary_document_scales_stay_simt(engine):
    import maxsim_b200 as m

    docs, off = _corpus(80, 60, seed=23)
    q = ref.clustered_queries(docs, off, 2, 16, seed=24)
    h = m.to_device(m.pack_signs(docs, off, scale="doc"), "cuda").data
    engine.set_engine(2)
    with pytest.raises(NotImplementedError):
        h.score_batch(q, use_scale_vector=True)
    engine.set_engine(1)
    want = h.score_batch(q, use_scale_vector=True)
    engine.set_engine(0)
    np.testing.assert_array_equal(h.score_batch(q, use_scale_vector=True), want)


# ---------------------------------------------------------------------------
# The fused residual stream: both int4 streams' int8 copies, two accumulators per query tile
# ---------------------------------------------------------------------------

def _digit_values(query, values):
    """Combined digit dots fl(65536 d2 + fl(d0 + 256 d1)) of every query row with every token [R, N],
    and the rows' power-of-two scales."""
    digits, qscale = _digits(query.reshape(-1, 128))
    dots = np.einsum("kri,ti->krt", digits, values.astype(np.int64))
    lo = (dots[0] + 256 * dots[1]).astype(np.float32)
    return (dots[2].astype(np.float64) * 65536.0 + lo.astype(np.float64)).astype(np.float32), qscale


def _residual_model(query, res, offsets, weights=None):
    B, Q, _ = query.shape
    v1, qscale = _digit_values(query, res["prefix_values"])
    v2, _ = _digit_values(query, res["residual_values"])
    f32 = np.float32
    a = (v1 * f32(res["prefix_scale"])) * np.asarray(res["prefix_token_scale"], f32)[None, :]
    b = (v2 * f32(res["residual_scale"])) * np.asarray(res["residual_token_scale"], f32)[None, :]
    sim = a + b  # every step a float32 operation, rounded once
    if weights is not None:
        w = np.broadcast_to(np.asarray(weights, f32), (B, Q)).reshape(-1)
        qscale = np.ldexp(w, np.frexp(qscale)[1] - 1).astype(f32)
    out = np.zeros((B, offsets.shape[0] - 1), f32)
    for d in range(offsets.shape[0] - 1):
        lo, hi = offsets[d], offsets[d + 1]
        if lo == hi:
            continue
        best = sim[:, lo:hi].max(axis=1) * qscale
        for bi in range(B):
            acc = f32(0)
            for r in range(Q):
                acc = f32(acc + best[bi * Q + r])
            out[bi, d] = acc
    return out


def _residual_corpus(num_docs, max_len, seed):
    import maxsim_b200 as m

    docs, off = _corpus(num_docs, max_len, seed)
    packed = m.pack_residual_int4(docs, off)
    res = {k: getattr(packed, k) for k in ("prefix_scale", "prefix_token_scale", "residual_scale",
                                            "residual_token_scale")}
    res["prefix_values"] = ref.unpack_nibbles(packed.prefix_data, 128)
    res["residual_values"] = ref.unpack_nibbles(packed.residual_data, 128)
    return docs, off, packed, res, m.residual_int4_to_device(packed)


@pytest.mark.parametrize("batch,qtok", [(1, 32), (4, 32), (3, 9)])
@pytest.mark.parametrize("weighted", [False, True])
def test_residual_stream_on_digit_planes(engine, batch, qtok, weighted):
    import maxsim_b200 as m

    docs, off, packed, res, dev = _residual_corpus(260, 250, seed=41 + qtok)
    q = ref.clustered_queries(docs, off, batch, qtok, seed=42)
    kw, w = {}, None
    if weighted:
        w = np.random.default_rng(43).uniform(0.5, 1.5, size=qtok).astype(np.float32)
        kw = {"reducer": "weighted_maxsim", "query_weights": w}
    engine.set_engine(2)
    got = m.residual_score(q, dev, **kw)
    np.testing.assert_array_equal(got, _residual_model(q, res, off, weights=w))
    oracle = {"prefix_values": res["prefix_values"], "prefix_scale": res["prefix_scale"],
              "prefix_token_scale": res["prefix_token_scale"], "residual_values": res["residual_values"],
              "residual_scale": res["residual_scale"], "residual_token_scale": res["residual_token_scale"]}
    exact = ref.score_residual(q, oracle, off, **({"reducer": "weighted_maxsim", "weights": w} if weighted else {}))
    np.testing.assert_allclose(got, exact, rtol=2e-6, atol=2e-6 * np.abs(exact).max())
    engine.set_engine(1)
    np.testing.assert_allclose(m.residual_score(q, dev, **kw), got, rtol=1e-5, atol=1e-5 * np.abs(exact).max())


def test_residual_stream_replaced_on_the_handle(engine):
    """Replacing or clearing a handle's residual stream drops its int8 copy: the next scan reads the new one."""
    import maxsim_b200 as m

    docs, off, packed, res, dev = _residual_corpus(150, 120, seed=51)
    q = ref.clustered_queries(docs, off, 2, 16, seed=52)
    h = dev.prefix_data
    engine.set_engine(2)
    first = h.score_residual_batch(q)
    np.testing.assert_array_equal(first, _residual_model(q, res, off))
    other = m.pack_residual_int4(docs[::-1].copy(), off)
    h.set_residual_int4(other.residual_data, float(other.residual_scale), other.residual_token_scale)
    res2 = dict(res, residual_values=ref.unpack_nibbles(other.residual_data, 128), residual_scale=other.residual_scale,
                residual_token_scale=other.residual_token_scale)
    np.testing.assert_array_equal(h.score_residual_batch(q), _residual_model(q, res2, off))
    h.clear_residual_int4()
    with pytest.raises(ValueError, match="residual"):
        h.score_residual_batch(q)


def test_candidate_lists_long_enough_read_the_full_scan(engine):
    """A candidate list naming at least one document in 16 is read out of the full tensor-core scan, a
    shorter one scanned by the same kernel over its documents only: either way its scores equal the full
    scan's columns exactly, and the SIMT engine's within 1e-4."""
    import maxsim_b200 as m

    docs, off, packed, res, dev = _residual_corpus(320, 90, seed=61)
    q = ref.clustered_queries(docs, off, 3, 20, seed=62)
    rng = np.random.default_rng(63)
    long_list = rng.integers(0, 320, size=40).astype(np.int64)   # 40 * 16 >= 320
    short_list = rng.integers(0, 320, size=15).astype(np.int64)  # 15 * 16 < 320
    int4 = m.int4_to_device(m.pack_int4_symmetric(docs, off, scale_granularity="token"))
    _, binh = _binary(docs, off, True)
    cases = [
        (lambda c=None: m.int4_maxsim(q, int4, candidate_indices=c)),
        (lambda c=None: m.residual_score(q, dev, candidate_indices=c)),
        (lambda c=None: binh.score_batch(q, use_token_scale=True) if c is None
         else binh.score_candidates_batch(q, c, use_token_scale=True)),
    ]
    for run in cases:
        engine.set_engine(0)
        full = run()
        np.testing.assert_array_equal(run(long_list), full[:, long_list])
        got_short = run(short_list)
        np.testing.assert_array_equal(got_short, full[:, short_list])
        engine.set_engine(1)
        np.testing.assert_allclose(got_short, run(short_list), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("batch,qtok", [(1, 32), (3, 16)])
def test_binary_prefix_residual_on_digit_planes(engine, batch, qtok):
    """Sign-code prefix (scale 1, per-token mean |x|) + int4 residual: the same residual kernel, reading
    the +-1 copy as the prefix stream."""
    from maxsim_b200 import cascade as casc

    docs, off = _corpus(240, 200, seed=71)
    q = ref.clustered_queries(docs, off, batch, qtok, seed=72)
    packed = casc.pack_binary_residual_int4(docs, off)
    dev = casc.binary_residual_to_device(packed)
    res = {"prefix_values": ref.unpack_signs(packed.prefix_data, 128).astype(np.int64), "prefix_scale": 1.0,
           "prefix_token_scale": packed.prefix_token_scale, "residual_values": ref.unpack_nibbles(packed.residual_data, 128),
           "residual_scale": 1.0, "residual_token_scale": packed.residual_token_scale}
    engine.set_engine(2)
    got = casc.binary_residual_score(q, dev)
    np.testing.assert_array_equal(got, _residual_model(q, res, off))
    engine.set_engine(1)
    simt = casc.binary_residual_score(q, dev)
    np.testing.assert_allclose(got, simt, rtol=1e-5, atol=1e-5 * np.abs(simt).max())


def _topk_model(query, values, offsets, scale, token_scale, K):
    """TopK reducers on digit planes: per row, the mean of the top min(K, tokens) values summed in
    descending order (one float32 division), times the row's power-of-two scale; rows summed in order."""
    B, Q, _ = query.shape
    v, qscale = _digit_values(query, values)
    if token_scale is not None:
        v = v * np.asarray(token_scale, np.float32)[None, :]
    f32 = np.float32
    out = np.zeros((B, offsets.shape[0] - 1), f32)
    for d in range(offsets.shape[0] - 1):
        lo, hi = offsets[d], offsets[d + 1]
        if lo == hi:
            continue
        top = -np.sort(-v[:, lo:hi], axis=1)[:, :min(K, hi - lo)]
        for bi in range(B):
            acc = f32(0)
            for r in range(Q):
                row = bi * Q + r
                total = f32(0)
                for x in top[row]:
                    total = f32(total + x)
                acc = f32(acc + f32(f32(total / f32(top.shape[1])) * qscale[row]))
            out[bi, d] = f32(acc * f32(scale))
    return out


@pytest.mark.parametrize("K", [2, 4])
@pytest.mark.parametrize("kind", ["token", "tensor", "binary"])
@pytest.mark.parametrize("batch,qtok", [(1, 24), (5, 16)])
def test_topk_reducers_on_digit_planes(engine, K, kind, batch, qtok):
    import maxsim_b200 as m

    docs, off = _corpus(220, 150, seed=81 + K)
    q = ref.clustered_queries(docs, off, batch, qtok, seed=82)
    reducer = f"topk{K}"
    if kind == "binary":
        packed, h = _binary(docs, off, True)
        values = ref.unpack_signs(packed.data, 128).astype(np.int64)
        ts, scale = np.asarray(packed.token_scale, np.float32), 1.0
        run = lambda: h.score_batch(q, reducer=reducer, use_token_scale=True)
        exact = ref.score_binary_fp32(q, packed.data, 128, off, token_scale=ts, reducer=reducer)
    else:
        packed = m.pack_int4_symmetric(docs, off, scale_granularity=kind)
        dev = m.int4_to_device(packed)
        values, ts, scale = packed.values, packed.token_scale, packed.scale
        run = lambda: m.int4_maxsim(q, dev, reducer=reducer)
        exact = ref.score_int4_fp32(q, values, off, scale=scale, token_scale=ts, reducer=reducer)
    assert (np.diff(off) == 1).any()  # documents shorter than K: the mean is over their tokens
    engine.set_engine(2)
    got = run()
    np.testing.assert_array_equal(got, _topk_model(q, values, off, scale, ts, K))
    np.testing.assert_allclose(got, exact, rtol=2e-6, atol=2e-6 * np.abs(exact).max())
    engine.set_engine(1)
    np.testing.assert_allclose(run(), got, rtol=1e-5, atol=1e-5 * np.abs(exact).max())


@pytest.mark.parametrize("kind", ["token", "tensor", "binary"])
@pytest.mark.parametrize("temperature", [0.1, 1.0])
@pytest.mark.parametrize("batch,qtok", [(1, 24), (5, 16)])
def test_smoothsim_on_digit_planes(engine, kind, temperature, batch, qtok):
    """SmoothSim (max + t * log sum exp((v - max) / t), every value scaled before the reduction): a running
    log-sum-exp per thread, merged across a row's four threads at each document end.  Within 1e-4 of the
    float64 oracle and of the SIMT engine (the sums of exponentials run in another order)."""
    import maxsim_b200 as m

    docs, off = _corpus(220, 300, seed=91)
    q = ref.clustered_queries(docs, off, batch, qtok, seed=92)
    kw = {"reducer": "smoothsim", "temperature": temperature}
    if kind == "binary":
        packed, h = _binary(docs, off, True)
        ts = np.asarray(packed.token_scale, np.float32)
        run = lambda: h.score_batch(q, use_token_scale=True, scale=0.75, **kw)
        exact = ref.score_binary_fp32(q, packed.data, 128, off, token_scale=ts, doc_scale=0.75, **kw)
    else:
        packed = m.pack_int4_symmetric(docs, off, scale_granularity=kind)
        dev = m.int4_to_device(packed)
        run = lambda: m.int4_maxsim(q, dev, **kw)
        exact = ref.score_int4_fp32(q, packed.values, off, scale=packed.scale, token_scale=packed.token_scale, **kw)
    engine.set_engine(2)
    got = run()
    np.testing.assert_allclose(got, exact, rtol=1e-4, atol=1e-4 * np.abs(exact).max())
    engine.set_engine(1)
    np.testing.assert_allclose(run(), got, rtol=1e-4, atol=1e-4 * np.abs(exact).max())


def test_smoothsim_large_scores_stay_finite(engine):
    """Values far above the temperature: every exponent is <= 0, so the sums stay finite (the reference's
    overflow known answer); documents of several tiles."""
    import maxsim_b200 as m

    docs, off = _corpus(40, 700, seed=93)
    q = 50.0 * ref.clustered_queries(docs, off, 3, 20, seed=94)
    packed = m.pack_int4_symmetric(docs, off, scale_granularity="token")
    dev = m.int4_to_device(packed)
    engine.set_engine(2)
    got = m.int4_maxsim(q, dev, reducer="smoothsim", temperature=0.01)
    assert np.all(np.isfinite(got))
    exact = ref.score_int4_fp32(q, packed.values, off, token_scale=packed.token_scale, reducer="smoothsim",
                                temperature=0.01)
    np.testing.assert_allclose(got, exact, rtol=1e-4, atol=1e-4 * np.abs(exact).max())
