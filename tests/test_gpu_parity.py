"""GPU parity: the CUDA library (through the C ABI) against the CPU oracle.

Tolerances (north star): integer int8-query x int4 and binary dots are exact,
so those scores must be bit-identical to the oracle's restatement of the
reference kernel's fp32 epilogue; fp32-query scores within 1e-4 relative
(atol 1e-4 absolute near zero); top-k ids identical except where scores tie
within tolerance.  Each test runs on both scan engines (SIMT and the
tensor-core engine) where the engine supports the case.
"""

import json
from pathlib import Path

import numpy as np
import pytest

from oracle import reference_cpu as ref

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).parent / "golden"
REDUCERS = ref.REDUCERS
RTOL, ATOL = 1e-4, 1e-4


@pytest.fixture(params=[1, 0], ids=["simt", "auto"])
def engine(request):
    from maxsim_b200 import _lib

    prev = _lib.get_engine()
    _lib.set_engine(request.param)
    yield request.param
    _lib.set_engine(prev)


def _assert_topk_equivalent(got_s, got_i, want_scores_full, k, rtol=RTOL, atol=ATOL):
    """ids identical except positions whose oracle scores tie within tolerance."""
    for row in range(got_i.shape[0]):
        full = want_scores_full[row]
        exp_i = ref.topk_indices(full, k)
        np.testing.assert_allclose(got_s[row], full[got_i[row]], rtol=rtol, atol=atol)
        np.testing.assert_allclose(got_s[row], full[exp_i], rtol=rtol, atol=atol)
        for pos in np.flatnonzero(got_i[row] != exp_i):
            a, b = full[got_i[row][pos]], full[exp_i[pos]]
            assert abs(a - b) <= atol + rtol * abs(b), f"row {row} pos {pos}: {a} vs {b}"


def _weights_kw(reducer, g):
    if reducer == "weighted_maxsim":
        return {"query_weights": g["weights"]}
    if reducer == "smoothsim":
        return {"temperature": 0.7}
    return {}


# ---------------------------------------------------------------------------
# int8 queries: exact
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("gran", ["tensor", "token"])
def test_int4_int8q_bit_exact(engine, golden, gran):
    import maxsim_b200 as m

    g = golden("int8q.npz")
    q, docs, off = g["query"], g["docs"], g["offsets"]
    packed = m.pack_int4_symmetric(docs, off, scale_granularity=gran)
    got = m.int4_maxsim_int8q(q, m.int4_to_device(packed))
    want = ref.score_int4_int8q(q, packed.values, off, scale=packed.scale, token_scale=packed.token_scale)
    np.testing.assert_array_equal(got, want)
    # the reference tests' own helper (rint(x/s) quantiser) at their tolerance
    np.testing.assert_allclose(got, g[f"int4_{gran}"], rtol=1e-5, atol=1e-3)
    empty = int(np.flatnonzero(np.diff(off) == 0)[0])
    assert np.all(got[:, empty] == 0.0)


@pytest.mark.parametrize("token_scale", [False, True])
def test_binary_int8q_bit_exact(engine, golden, token_scale):
    import maxsim_b200 as m

    g = golden("int8q.npz")
    q, docs, off = g["query"], g["docs"], g["offsets"]
    packed = m.to_device(m.pack_signs(docs, off, token_scale="mean_abs_fp16" if token_scale else None), "cuda")
    got = packed.data.maxsim_batch_int8q(q, 1.0, False, token_scale)
    want = ref.score_binary_int8q(q, ref.pack_signs(docs), off, token_scale=packed.token_scale if token_scale else None)
    np.testing.assert_array_equal(got, want)
    np.testing.assert_allclose(got, g["binary_ts" if token_scale else "binary"], rtol=1e-5, atol=1e-3)


def test_scale_before_max_known_answer(engine):
    import maxsim_b200 as m

    docs = np.stack([np.ones(128, np.float32),
                     np.concatenate([np.full(64, 10.0, np.float32), np.zeros(64, np.float32)])])
    packed = m.int4_to_device(m.pack_int4_symmetric(docs, np.array([0, 2]), scale_granularity="token"))
    got = m.int4_maxsim_int8q(np.ones((1, 1, 128), np.float32), packed)
    np.testing.assert_allclose(got, [[640.0]], rtol=0, atol=1e-3)


@pytest.mark.parametrize("gran", ["tensor", "token"])
def test_int8q_topk_matches_oracle_ranking(engine, gran):
    import maxsim_b200 as m

    docs, off = ref.clustered_corpus(600, 4, 40, seed=3)
    q = ref.clustered_queries(docs, off, 5, 9, seed=4)
    packed = m.pack_int4_symmetric(docs, off, scale_granularity=gran)
    dev = m.int4_to_device(packed)
    s, i = dev.data.topk_batch_int8q(q, 10)
    full = ref.score_int4_int8q(q, packed.values, off, scale=packed.scale, token_scale=packed.token_scale)
    exp_s, exp_i = ref.topk_rows(full, 10)
    np.testing.assert_array_equal(i, exp_i)  # exact scores -> exact ids
    np.testing.assert_array_equal(s, exp_s)


# ---------------------------------------------------------------------------
# fp32 queries, every reducer, full and candidate scoring
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("reducer", REDUCERS)
def test_reducers_match_reference_golden(engine, golden, reducer):
    import maxsim_b200 as m

    g = golden("scores.npz")
    q, docs, off, cands = g["query"], g["docs"], g["offsets"], g["candidates"]
    kw = _weights_kw(reducer, g)
    corpora = {
        "binary": m.pack_signs(docs, off),
        "binary_ts": m.pack_signs(docs, off, token_scale="mean_abs_fp16"),
        "binary_doc": m.pack_signs(docs, off, scale="doc"),
        "int4_tensor": m.pack_int4_symmetric(docs, off),
        "int4_token": m.pack_int4_symmetric(docs, off, scale_granularity="token"),
    }
    for name, packed in corpora.items():
        dev = m.to_device(packed, "cuda") if name.startswith("binary") else m.int4_to_device(packed)
        full = m.score(q, dev, reducer=reducer, **kw)
        cand = m.score(q, dev, reducer=reducer, candidate_indices=cands, **kw)
        np.testing.assert_allclose(full, g[f"{name}_{reducer}_full"], rtol=RTOL, atol=3e-4, err_msg=name)
        np.testing.assert_allclose(cand, g[f"{name}_{reducer}_cand"], rtol=RTOL, atol=3e-4, err_msg=name)
        if engine == 0 and reducer in ("maxsim", "weighted_maxsim", "topk2", "topk4") and name != "binary_doc":
            # full scans of fp32 queries run on the tensor-core digit planes (the exact dot of the query
            # rounded to 23 bits, one rounding), candidate lists on fp32 FMA chains
            np.testing.assert_allclose(cand, np.take(full, cands, axis=-1), rtol=2e-6, atol=2e-6 * np.abs(full).max(),
                                       err_msg=f"{name}: candidates vs full")
        else:
            np.testing.assert_array_equal(cand, np.take(full, cands, axis=-1), err_msg=f"{name}: candidates != full")
    res = m.residual_int4_to_device(m.pack_residual_int4(docs, off))
    full = m.residual_score(q, res, reducer=reducer, **kw)
    cand = m.residual_score(q, res, reducer=reducer, candidate_indices=cands, **kw)
    np.testing.assert_allclose(full, g[f"residual_{reducer}_full"], rtol=RTOL, atol=3e-4)
    np.testing.assert_allclose(cand, g[f"residual_{reducer}_cand"], rtol=RTOL, atol=3e-4)
    if engine == 0 and reducer in ("maxsim", "weighted_maxsim"):
        # the full scan runs on the tensor-core digit planes, candidate lists on fp32 FMA chains
        np.testing.assert_allclose(cand, np.take(full, cands, axis=-1), rtol=2e-6, atol=2e-6 * np.abs(full).max())
    else:
        np.testing.assert_array_equal(cand, np.take(full, cands, axis=-1))


@pytest.mark.parametrize("gran", ["tensor", "token"])
def test_int4_fp32_clustered_vs_float64_oracle(engine, gran):
    import maxsim_b200 as m

    docs, off = ref.clustered_corpus(400, 0, 60, seed=11)
    q = ref.clustered_queries(docs, off, 3, 32, seed=12)
    packed = m.pack_int4_symmetric(docs, off, scale_granularity=gran)
    dev = m.int4_to_device(packed)
    got = m.int4_maxsim(q, dev)
    want = ref.score_int4_fp32(q, packed.values, off, scale=packed.scale, token_scale=packed.token_scale)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)
    s, i = m.topk_int4_maxsim(q, dev, 10)
    _assert_topk_equivalent(s, i, want, 10)


def test_binary_fp32_topk_ties_and_doc_scale(engine, golden):
    import maxsim_b200 as m

    g = golden("scores.npz")
    dev = m.to_device(m.pack_signs(g["tie_docs"]), "cuda")
    s, i = m.topk_maxsim(g["tie_query"], dev, k=3)
    np.testing.assert_array_equal(i, g["tie_top_indices"])
    np.testing.assert_allclose(s, g["tie_top_scores"], atol=1e-5)
    signs = np.array([1, -1, 1, -1, 1, -1, 1, -1], dtype=np.float32)
    docs = np.stack([signs, signs * 10.0, -signs])
    dev = m.to_device(m.pack_signs(docs, scale="doc"), "cuda")
    s, i = m.topk_maxsim(signs.reshape(1, 1, 8), dev, k=2)
    np.testing.assert_array_equal(i, [[1, 0]])


def test_cascade_matches_reference_golden(engine, golden):
    import maxsim_b200 as m

    g = golden("scores.npz")
    res = m.residual_int4_to_device(m.pack_residual_int4(g["c_docs"], g["c_offsets"]))
    for mm in (10, 40, 160):
        s, i = m.cascade_topk(g["c_query"], res, 5, candidates=mm)
        np.testing.assert_array_equal(i, g[f"cascade_m{mm}_indices"])
        np.testing.assert_allclose(s, g[f"cascade_m{mm}_scores"], rtol=RTOL, atol=ATOL)


def test_sdk_search_matches_reference_golden(engine):
    import maxsim_b200 as m

    want = json.loads((GOLDEN / "sdk_search.json").read_text())
    inputs = np.load(GOLDEN / "index_inputs.npz")
    for mode, rows in want.items():
        reranker = m.Reranker.load(GOLDEN / f"index_{mode}.npz", device="cuda")
        got = reranker.search(inputs["query"], k=3)
        for grow, wrow in zip(got, rows):
            assert [r.doc_id for r in grow] == [w[0] for w in wrow], mode
            np.testing.assert_allclose([r.score for r in grow], [w[1] for w in wrow], rtol=RTOL, atol=ATOL)
            assert [r.rank for r in grow] == [1, 2, 3]


def test_sdk_rerank_matches_reference_golden(engine):
    """Reranker.rerank on a candidate list with a duplicate id, every corpus mode."""
    import maxsim_b200 as m

    want = json.loads((GOLDEN / "sdk_rerank.json").read_text())
    inputs = np.load(GOLDEN / "index_inputs.npz")
    for mode, rows in want.items():
        reranker = m.Reranker.load(GOLDEN / f"index_{mode}.npz", device="cuda")
        got = reranker.rerank(inputs["query"], ["doc-4", "doc-1", "doc-5", "doc-1"], k=2)
        for grow, wrow in zip(got, rows):
            assert [r.doc_id for r in grow] == [w[0] for w in wrow], mode
            np.testing.assert_allclose([r.score for r in grow], [w[1] for w in wrow], rtol=RTOL, atol=ATOL)
            assert [r.rank for r in grow] == [w[2] for w in wrow], mode


def test_sdk_int8_query_search_and_rerank(engine):
    import maxsim_b200 as m

    docs, off = ref.clustered_corpus(64, 1, 30, seed=21)
    q = ref.clustered_queries(docs, off, 2, 7, seed=22)
    ids = [f"doc-{i}" for i in range(64)]
    idx = m.Index.from_embeddings(ids, docs, off, mode="max_quality")
    rr = m.Reranker(idx, device="cuda", int4_query="int8")
    got = rr.search(q, k=5)
    p = idx.int4_packed
    full = ref.score_int4_int8q(q, p.values, off, token_scale=p.token_scale)
    for row, res in enumerate(got):
        exp = ref.topk_indices(full[row], 5)
        assert [r.doc_id for r in res] == [ids[j] for j in exp]
        np.testing.assert_array_equal([np.float32(r.score) for r in res], full[row][exp])
    rer = rr.rerank(q, ["doc-3", "doc-1", "doc-2", "doc-3"], k=2)
    assert len(rer) == 2 and len(rer[0]) == 2


# ---------------------------------------------------------------------------
# edge cases
# ---------------------------------------------------------------------------

def test_empty_batches_queries_and_docs(engine):
    import maxsim_b200 as m

    docs = np.random.default_rng(1).standard_normal((5, 128)).astype(np.float32)
    off = np.array([0, 0, 2, 2, 3, 5], dtype=np.int64)
    packed = m.pack_int4_symmetric(docs, off, scale_granularity="token")
    dev = m.int4_to_device(packed)
    assert m.int4_maxsim(np.zeros((0, 3, 128), np.float32), dev).shape == (0, 5)
    np.testing.assert_array_equal(m.int4_maxsim(np.zeros((2, 0, 128), np.float32), dev), np.zeros((2, 5)))
    got = m.int4_maxsim(np.ones((1, 2, 128), np.float32), dev)
    for d in range(5):
        if off[d] == off[d + 1]:
            assert got[0, d] == 0.0
    s, i = m.topk_int4_maxsim(np.ones((1, 2, 128), np.float32), dev, 5)
    assert sorted(i[0].tolist()) == [0, 1, 2, 3, 4]


def test_k_bounds_raise_value_error(engine):
    import maxsim_b200 as m

    dev = m.int4_to_device(m.pack_int4_symmetric(np.ones((4, 128), np.float32), np.array([0, 2, 4])))
    with pytest.raises(ValueError):
        dev.data.topk_batch(np.ones((1, 1, 128), np.float32), 3)
    with pytest.raises(ValueError):
        dev.data.topk_batch(np.ones((1, 1, 128), np.float32), 0)


def test_device_packers_bit_exact(engine):
    import torch

    from maxsim_b200 import _lib

    rng = np.random.default_rng(5)
    x = rng.standard_normal((1000, 128)).astype(np.float32)
    x[7] = 0.0
    xt = torch.from_numpy(x).cuda()
    codes = torch.empty((1000, 64), dtype=torch.uint8, device="cuda")
    ts = torch.empty(1000, dtype=torch.float32, device="cuda")
    _lib.check(_lib.lib.msb_pack_int4_device(xt.data_ptr(), 1000, 128, 1, codes.data_ptr(), ts.data_ptr(), None, None))
    torch.cuda.synchronize()
    data, _, _, want_ts = ref.pack_int4(x, "token")
    np.testing.assert_array_equal(codes.cpu().numpy(), data)
    np.testing.assert_array_equal(ts.cpu().numpy(), want_ts)
    import ctypes

    tscale = ctypes.c_float()
    _lib.check(_lib.lib.msb_pack_int4_device(xt.data_ptr(), 1000, 128, 0, codes.data_ptr(), None,
                                             ctypes.byref(tscale), None))
    torch.cuda.synchronize()
    data, _, scale, _ = ref.pack_int4(x, "tensor")
    np.testing.assert_array_equal(codes.cpu().numpy(), data)
    assert tscale.value == np.float32(scale)
    bits = torch.empty((1000, 16), dtype=torch.uint8, device="cuda")
    mabs = torch.empty(1000, dtype=torch.float32, device="cuda")
    _lib.check(_lib.lib.msb_pack_signs_device(xt.data_ptr(), 1000, 128, bits.data_ptr(), mabs.data_ptr(), None))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits.cpu().numpy(), ref.pack_signs(x))
    np.testing.assert_allclose(mabs.cpu().numpy(), ref.mean_abs_token_scale(x), rtol=1e-7)


def test_quantizer_matches_kernel_formula(engine):
    import torch

    from maxsim_b200 import _lib

    rng = np.random.default_rng(9)
    q = rng.standard_normal((777, 128)).astype(np.float32)
    q[3] = 0.0
    qt = torch.from_numpy(q).cuda()
    codes = torch.empty((777, 128), dtype=torch.int8, device="cuda")
    scales = torch.empty(777, dtype=torch.float32, device="cuda")
    _lib.check(_lib.lib.msb_quantize_query_int8_device(qt.data_ptr(), 777, 128, codes.data_ptr(), scales.data_ptr(),
                                                       None))
    torch.cuda.synchronize()
    c, s = ref.quantize_query_int8(q)
    np.testing.assert_array_equal(codes.cpu().numpy(), c)
    np.testing.assert_array_equal(scales.cpu().numpy(), s)


def test_generic_dims_and_host_packed_functions(engine):
    import maxsim_b200 as m
    from maxsim_b200 import _maxsim_cuda as mc

    rng = np.random.default_rng(2)
    docs = rng.standard_normal((30, 24)).astype(np.float32)
    off = np.array([0, 4, 11, 19, 30])
    q = rng.standard_normal((3, 5, 24)).astype(np.float32)
    packed = m.pack_signs(docs, off)
    want = ref.score_binary_fp32(q, ref.pack_signs(docs), 24, off)
    np.testing.assert_allclose(m.maxsim(q, packed), want, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(mc.maxsim_cuda_batch(q, packed.data, off, 24), want, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(mc.maxsim_cuda(q[1], packed.data, off, 24), want[1], rtol=RTOL, atol=ATOL)
    p4 = m.pack_int4_symmetric(docs, off)
    np.testing.assert_allclose(m.int4_maxsim(q, p4), ref.score_int4_fp32(q, p4.values, off, scale=p4.scale),
                               rtol=RTOL, atol=ATOL)


def test_workspace_grows_and_reuse_is_consistent(engine):
    import maxsim_b200 as m

    docs, off = ref.clustered_corpus(50, 1, 20, seed=8)
    dev = m.int4_to_device(m.pack_int4_symmetric(docs, off, scale_granularity="token"))
    rng = np.random.default_rng(0)
    shapes = [(2, 5), (3, 17), (2, 5)]
    ws = []
    for b, qt in shapes:
        q = rng.standard_normal((b, qt, 128)).astype(np.float32)
        a = dev.data.maxsim_batch_int8q(q)
        bb = dev.data.maxsim_batch_int8q(q)
        np.testing.assert_array_equal(a, bb)
        ws.append(dev.data.workspace_bytes)
    assert ws[0] <= ws[1] == ws[2]
