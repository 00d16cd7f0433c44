"""Pin the CPU oracle against golden vectors produced by the reference itself.

The fixtures in ``tests/golden`` were written by ``tests/golden/make_golden.py``
running the unmodified reference package; these tests prove the restatement in
``oracle/`` reproduces them before the oracle is trusted as the GPU checker.
"""

import ctypes
import json

import numpy as np
import pytest

from oracle import reference_cpu as ref

REDUCERS = ref.REDUCERS


def test_int4_packing_matches_reference(golden):
    g = golden("formats.npz")
    for gran in ("tensor", "token"):
        data, values, scale, ts = ref.pack_int4(g["docs"], gran)
        np.testing.assert_array_equal(data, g[f"int4_{gran}_data"])
        np.testing.assert_array_equal(values, g[f"int4_{gran}_values"])
        assert scale == float(g[f"int4_{gran}_scale"])
        if gran == "token":
            np.testing.assert_array_equal(ts, g["int4_token_token_scale"])
        np.testing.assert_array_equal(ref.unpack_nibbles(data, 128), values)


def test_residual_packing_matches_reference(golden):
    g = golden("formats.npz")
    res = ref.pack_residual_int4(g["docs"])
    for name in ("prefix_data", "prefix_values", "prefix_token_scale", "residual_data", "residual_values",
                 "residual_token_scale"):
        np.testing.assert_array_equal(res[name], g[f"residual_{name}"])


def test_binary_packing_and_token_scales_match_reference(golden):
    g = golden("formats.npz")
    np.testing.assert_array_equal(ref.pack_signs(g["docs"]), g["binary_data"])
    for kind in ("mean_abs", "l2", "mean_abs_fp16", "mean_abs_u8", "mean_abs_u4"):
        np.testing.assert_array_equal(ref.token_scale(g["docs"], kind), g[f"binary_token_scale_{kind}"])


def test_bit_order_little_endian_zero_is_positive():
    docs = np.array([[0.0, -1, 1, -1, -1, -1, -1, -1]], dtype=np.float32)
    assert ref.pack_signs(docs)[0, 0] == 0b00000101


@pytest.mark.parametrize("reducer", REDUCERS)
def test_reducer_scores_match_reference(golden, reducer):
    g = golden("scores.npz")
    q, docs, off, cands = g["query"], g["docs"], g["offsets"], g["candidates"]
    kw = {"weights": g["weights"]} if reducer == "weighted_maxsim" else {}
    if reducer == "smoothsim":
        kw = {"temperature": 0.7}
    bpacked = ref.pack_signs(docs)
    ts = ref.token_scale(docs, "mean_abs_fp16")
    doc_scale = np.zeros(len(off) - 1, dtype=np.float32)
    for d in range(len(off) - 1):
        s, e = off[d], off[d + 1]
        if s != e:
            doc_scale[d] = np.float32(np.mean(np.abs(docs[s:e]), dtype=np.float64))
    _, vt, st, _ = ref.pack_int4(docs, "tensor")
    _, vp, _, tsp = ref.pack_int4(docs, "token")
    res = ref.pack_residual_int4(docs)
    for cand, suffix in ((None, "full"), (cands, "cand")):
        got = {
            "binary": ref.score_binary_fp32(q, bpacked, 128, off, reducer=reducer, candidates=cand, **kw),
            "binary_ts": ref.score_binary_fp32(q, bpacked, 128, off, token_scale=ts, reducer=reducer,
                                               candidates=cand, **kw),
            "binary_doc": ref.score_binary_fp32(q, bpacked, 128, off, doc_scale=doc_scale, reducer=reducer,
                                                candidates=cand, **kw),
            "int4_tensor": ref.score_int4_fp32(q, vt, off, scale=st, reducer=reducer, candidates=cand, **kw),
            "int4_token": ref.score_int4_fp32(q, vp, off, token_scale=tsp, reducer=reducer, candidates=cand, **kw),
            "residual": ref.score_residual(q, res, off, reducer=reducer, candidates=cand, **kw),
        }
        for name, value in got.items():
            np.testing.assert_allclose(value, g[f"{name}_{reducer}_{suffix}"], rtol=2e-5, atol=2e-4,
                                       err_msg=f"{name} {reducer} {suffix}")


def test_topk_ties_go_to_lower_ids(golden):
    g = golden("scores.npz")
    scores = ref.score_binary_fp32(g["tie_query"], ref.pack_signs(g["tie_docs"]), 8, np.arange(5))
    s, i = ref.topk_rows(scores, 3)
    np.testing.assert_array_equal(i, g["tie_top_indices"])
    np.testing.assert_allclose(s, g["tie_top_scores"], atol=1e-6)


def test_int4_topk_and_cascade_match_reference(golden):
    g = golden("scores.npz")
    q, docs, off = g["c_query"], g["c_docs"], g["c_offsets"]
    _, vp, _, tsp = ref.pack_int4(docs, "token")
    scores = ref.score_int4_fp32(q, vp, off, token_scale=tsp)
    s, i = ref.topk_rows(scores, 10)
    np.testing.assert_array_equal(i, g["c_int4_top_indices"])
    np.testing.assert_allclose(s, g["c_int4_top_scores"], rtol=1e-5, atol=1e-5)
    res = ref.pack_residual_int4(docs)
    for m in (10, 40, 160):
        cs, ci = ref.cascade_topk(q, res, off, 5, m)
        np.testing.assert_array_equal(ci, g[f"cascade_m{m}_indices"])
        np.testing.assert_allclose(cs, g[f"cascade_m{m}_scores"], rtol=1e-5, atol=1e-5)


def test_binary_maxsim_matches_reference_cpp_lut(golden):
    g = golden("scores.npz")
    if "c_binary_lut" not in g:
        pytest.skip("reference C++ extension was not built when fixtures were generated")
    got = ref.score_binary_fp32(g["c_query"], ref.pack_signs(g["c_docs"]), 128, g["c_offsets"])
    np.testing.assert_allclose(got, g["c_binary_lut"], rtol=1e-5, atol=1e-4)


def test_int8q_oracle_matches_reference_test_helpers(golden):
    """The reference test helpers quantise with rint(x/s); the kernel formula
    rint(x*(1/s)) can differ by one code, so this is the reference tests' own
    tolerance (rtol=1e-5, atol=1e-3)."""
    g = golden("int8q.npz")
    q, docs, off = g["query"], g["docs"], g["offsets"]
    for gran in ("tensor", "token"):
        _, vals, scale, ts = ref.pack_int4(docs, gran)
        got = ref.score_int4_int8q(q, vals, off, scale=scale, token_scale=ts)
        np.testing.assert_allclose(got, g[f"int4_{gran}"], rtol=1e-5, atol=1e-3)
    packed = ref.pack_signs(docs)
    np.testing.assert_allclose(ref.score_binary_int8q(q, packed, off), g["binary"], rtol=1e-5, atol=1e-3)
    ts = ref.token_scale(docs, "mean_abs_fp16")
    np.testing.assert_allclose(ref.score_binary_int8q(q, packed, off, token_scale=ts), g["binary_ts"],
                               rtol=1e-5, atol=1e-3)


def test_scale_before_max_known_answer():
    """tests/test_int4_int8q.py:110-134 of the reference: expected 640.0."""
    docs = np.stack([np.ones(128, np.float32),
                     np.concatenate([np.full(64, 10.0, np.float32), np.zeros(64, np.float32)])])
    off = np.array([0, 2], dtype=np.int64)
    _, vals, scale, ts = ref.pack_int4(docs, "token")
    got = ref.score_int4_int8q(np.ones((1, 1, 128), np.float32), vals, off, scale=scale, token_scale=ts)
    np.testing.assert_allclose(got, [[640.0]], rtol=0, atol=1e-3)


def test_quantizer_uses_reciprocal_multiply():
    """Kernel formula x*(1/s) differs from x/s on some inputs; the oracle must
    follow the kernel (cuda_extension.cu:1473-1485)."""
    rng = np.random.default_rng(3)
    q = rng.standard_normal((4096, 128)).astype(np.float32)
    codes, scales = ref.quantize_query_int8(q)
    inv = (np.float32(1) / scales).astype(np.float32)
    np.testing.assert_array_equal(codes, np.clip(np.rint((q * inv[:, None]).astype(np.float32)), -127, 127))
    assert np.abs(codes).max() == 127


def test_c_oracle_matches_numpy_oracle(golden, oracle_c):
    g = golden("int8q.npz")
    q, docs, off = g["query"], g["docs"], g["offsets"]
    B, Q, D = q.shape[0], q.shape[1], len(off) - 1
    codes = np.empty((B * Q, 128), np.int8)
    qs = np.empty(B * Q, np.float32)
    f = oracle_c.oracle_quantize_int8
    f(q.ctypes.data_as(ctypes.c_void_p), ctypes.c_int64(B * Q), ctypes.c_int(128),
      codes.ctypes.data_as(ctypes.c_void_p), qs.ctypes.data_as(ctypes.c_void_p))
    c_np, s_np = ref.quantize_query_int8(q.reshape(-1, 128))
    np.testing.assert_array_equal(codes, c_np)
    np.testing.assert_array_equal(qs, s_np)
    for gran in ("tensor", "token"):
        data, vals, scale, ts = ref.pack_int4(docs, gran)
        out = np.empty((B, D), np.float32)
        oracle_c.oracle_int4_int8q_scores(
            codes.ctypes.data_as(ctypes.c_void_p), qs.ctypes.data_as(ctypes.c_void_p), B, Q, 128,
            data.ctypes.data_as(ctypes.c_void_p),
            None if ts is None else ts.ctypes.data_as(ctypes.c_void_p), ctypes.c_float(scale),
            off.ctypes.data_as(ctypes.c_void_p), ctypes.c_int64(D), None, ctypes.c_int64(0),
            out.ctypes.data_as(ctypes.c_void_p), 2)
        np.testing.assert_array_equal(out, ref.score_int4_int8q(q, vals, off, scale=scale, token_scale=ts))


def test_index_files_have_reference_layout():
    from pathlib import Path

    gdir = Path(__file__).parent / "golden"
    search = json.loads((gdir / "sdk_search.json").read_text())
    assert set(search) >= {"binary", "int4_per_token", "int4_residual", "max_quality"}
    with np.load(gdir / "index_int4_per_token.npz") as z:
        assert int(z["schema_version"]) == 2
        assert str(z["format"]) == "maxsim_corpus"
        assert z["int4_data"].dtype == np.uint8 and z["int4_token_scale"].dtype == np.float32


@pytest.mark.parametrize("mode", ["binary", "binary_token_scale", "binary_token_scale_u8", "binary_token_scale_u4",
                                  "int4", "int4_per_token", "int4_residual", "binary_q40", "pooled_binary",
                                  "max_compression", "max_speed", "balanced", "compact", "max_quality", "auto"])
def test_index_from_embeddings_writes_the_reference_arrays(tmp_path, mode):
    """Index.from_embeddings + save (host packing, calibration, pooling) reproduces the
    npz arrays the reference wrote for the same inputs, key for key."""
    from pathlib import Path

    import maxsim_b200 as m

    gdir = Path(__file__).parent / "golden"
    inp = np.load(gdir / "index_inputs.npz")
    ids = [f"doc-{i}" for i in range(len(inp["offsets"]) - 1)]
    idx = m.Index.from_embeddings(ids, inp["docs"], inp["offsets"], mode=mode, metadata={"seed": 17})
    idx.save(tmp_path / "out.npz")
    with np.load(gdir / f"index_{mode}.npz") as want, np.load(tmp_path / "out.npz") as got:
        assert set(got.keys()) == set(want.keys()), mode
        for k in want.keys():
            if k == "metadata_json":
                assert json.loads(str(got[k])) == json.loads(str(want[k])), mode
            else:
                np.testing.assert_array_equal(got[k], want[k], err_msg=f"{mode}:{k}")


def test_binary_residual_host_pack_matches_oracle():
    """Host packing of the binary-prefix residual format equals the oracle restatement
    (parity unpinned: the reference has no such format)."""
    import maxsim_b200 as m

    docs, off = ref.clustered_corpus(40, 0, 50, seed=5)
    docs[3] = 0.0  # an all-zero token: mean |x| = 0, residual int4 scale falls back to 1
    want = ref.pack_binary_residual(docs)
    got = m.pack_binary_residual_int4(docs, off)
    np.testing.assert_array_equal(got.prefix_data, want["bits"])
    np.testing.assert_array_equal(got.prefix_token_scale, want["prefix_token_scale"])
    np.testing.assert_array_equal(got.residual_data, want["residual_data"])
    np.testing.assert_array_equal(got.residual_token_scale, want["residual_token_scale"])
    # the fused reconstruction is closer to x than the sign prefix alone
    p = ref.unpack_signs(want["bits"], 128) * want["prefix_token_scale"][:, None]
    r = want["residual_values"] * want["residual_token_scale"][:, None]
    assert np.abs(docs - (p + r)).mean() < 0.25 * np.abs(docs - p).mean()


def test_binary_residual_oracle_matches_reference(golden):
    """The binary-prefix residual format: the oracle's packing and scores against the reference's own
    residual code run on the same format (signs as int4 codes +-1 with the per-token mean |x| as prefix
    token scales, ``tests/golden/make_golden.py``)."""
    g = golden("binres.npz")
    res = ref.pack_binary_residual(g["docs"])
    np.testing.assert_array_equal(res["prefix_token_scale"], g["prefix_token_scale"])
    np.testing.assert_array_equal(res["residual_values"], g["residual_values"])
    np.testing.assert_array_equal(res["residual_data"], g["residual_data"])
    np.testing.assert_array_equal(res["residual_token_scale"], g["residual_token_scale"])
    for reducer in REDUCERS:
        kw = dict(reducer=reducer, temperature=0.1 if reducer == "smoothsim" else 1.0)
        if reducer == "weighted_maxsim":
            kw["weights"] = g["weights"]
        got = ref.score_binary_residual(g["query"], res, g["offsets"], **kw)
        np.testing.assert_allclose(got, g[f"{reducer}_full"], rtol=1e-4, atol=1e-4)
    for m in (10, 40, 120):
        s, i = ref.binary_cascade_topk(g["query"], res, g["offsets"], 5, m)
        np.testing.assert_array_equal(i, g[f"cascade_m{m}_indices"])
        np.testing.assert_allclose(s, g[f"cascade_m{m}_scores"], rtol=1e-4, atol=1e-4)


def test_binary_residual_packer_matches_reference(golden):
    """The library's host packer writes the same streams as the reference-built fixture."""
    import maxsim_b200 as m

    g = golden("binres.npz")
    p = m.pack_binary_residual_int4(g["docs"], g["offsets"])
    np.testing.assert_array_equal(p.prefix_token_scale, g["prefix_token_scale"])
    np.testing.assert_array_equal(p.residual_values, g["residual_values"])
    np.testing.assert_array_equal(p.residual_data, g["residual_data"])
    np.testing.assert_array_equal(p.residual_token_scale, g["residual_token_scale"])
    np.testing.assert_array_equal(ref.unpack_signs(p.prefix_data, 128) > 0, g["docs"] >= 0)
