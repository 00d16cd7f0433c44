"""Generate golden vectors by running the reference maxsim package itself.

Run in a container where the reference project is available (read-only) and
its CPU extension has been compiled by ``make -C oracle``::

    python tests/golden/make_golden.py [--reference /path/to/maxsim]

It imports the reference's Python package from ``<reference>/src`` (with the
``_maxsim_cpp`` module built from the reference's own C++ source into
``oracle/_ref``) and writes small seeded fixtures to ``tests/golden/``:

* ``formats.npz``   -- int4 (tensor / per-token), residual and binary packing,
                       token-scale variants, log codes
* ``scores.npz``    -- CPU scores of every reducer for binary / int4 / residual
                       corpora (full and candidate scoring), top-k with ties,
                       the residual cascade, ``maxsim_lut``
* ``int8q.npz``     -- the reference tests' int8-query NumPy helper outputs
                       (``tests/test_int4_int8q.py``, ``tests/test_binary_int8q.py``)
* ``index_<mode>.npz`` -- ``Index.save`` files written by the reference for
                       every corpus mode (npz layout golden)
* ``binres.npz``    -- the binary-prefix residual cascade scored and cascaded
                       by the reference's residual code (``--only-binres``
                       writes this file alone)
* ``sdk_search.json`` -- ``Reranker(device="cpu").search`` results
* ``sdk_rerank.json`` -- ``Reranker(device="cpu").rerank`` results on a candidate list

The fixtures are committed; the GPU box never needs the reference.
"""

from __future__ import annotations

import argparse
import os
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
REDUCERS = ("maxsim", "weighted_maxsim", "topk2", "topk4", "smoothsim")


def _load_reference(ref_root: Path):
    ext = sorted((REPO / "oracle" / "_ref").glob("_maxsim_cpp*.so"))
    if ext:
        spec = importlib.util.spec_from_file_location("maxsim._maxsim_cpp", ext[0])
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        sys.modules["maxsim._maxsim_cpp"] = mod
    sys.path.insert(0, str(ref_root / "src"))
    import maxsim  # noqa: E402  (the reference package)

    return maxsim


def _load_test_helper(ref_root: Path, name: str, func: str):
    spec = importlib.util.spec_from_file_location(f"_ref_{name}", ref_root / "tests" / f"{name}.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return getattr(mod, func)


def _ragged(num_docs, seed, dim=128, lo=1, hi=9, empty_at=2):
    rng = np.random.default_rng(seed)
    lengths = rng.integers(lo, hi, size=num_docs)
    if empty_at is not None:
        lengths[min(empty_at, num_docs - 1)] = 0
    offsets = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    docs = rng.standard_normal((int(offsets[-1]), dim)).astype(np.float32)
    return docs, offsets


def binary_residual_golden(cascade, experimental) -> None:
    """``binres.npz``: the binary-prefix residual cascade (sign bits scaled by the per-token mean |x|, plus
    the per-token int4 residual of x - mean|x| * sign(x)) scored by the reference's own code.  The reference
    has no sign-code prefix, but its residual cascade takes any symmetric int4 prefix: the signs as int4
    codes +-1 with prefix scale 1 and the mean |x| as the prefix's token scales reconstruct exactly the
    sign-code prefix, and the residual is packed by the reference's per-token int4 packer.  Its CPU
    ``residual_score`` (the fused reconstruction) and ``cascade_topk`` (prefix scan, stable top-M, rescoring)
    then give the scores and cascades this format must reproduce."""
    docs, off = _ragged(120, seed=81, lo=2, hi=16, empty_at=5)
    query = np.random.default_rng(83).standard_normal((3, 16, 128)).astype(np.float32)
    weights = np.random.default_rng(84).uniform(0.5, 1.5, size=16).astype(np.float32)
    signs = np.where(docs >= 0, 1, -1).astype(np.int8)
    mean_abs = np.mean(np.abs(docs), axis=1, dtype=np.float64).astype(np.float32)
    residual = (docs - mean_abs[:, None] * signs.astype(np.float32)).astype(np.float32)
    rpk = experimental.pack_int4_symmetric(residual, off, scale_granularity="token")
    assert float(rpk.scale) == 1.0
    packed = cascade.ResidualInt4PackedDocs(
        prefix_data=experimental._pack_signed_int4_values(signs), prefix_values=signs, prefix_scale=1.0,
        prefix_token_scale=mean_abs, residual_data=rpk.data, residual_values=rpk.values,
        residual_scale=float(rpk.scale), residual_token_scale=rpk.token_scale, doc_offsets=rpk.doc_offsets,
        dim=128, num_docs=int(off.shape[0] - 1), device="cpu")
    out = dict(docs=docs, offsets=off, query=query, weights=weights, prefix_token_scale=mean_abs,
               residual_values=rpk.values, residual_data=rpk.data, residual_token_scale=rpk.token_scale)
    for reducer in REDUCERS:
        kw = dict(reducer=reducer, temperature=0.1 if reducer == "smoothsim" else 1.0)
        if reducer == "weighted_maxsim":
            kw["query_weights"] = weights
        out[f"{reducer}_full"] = cascade.residual_score(query, packed, device="cpu", **kw)
    for m in (10, 40, 120):
        cs, ci = cascade.cascade_topk(query, packed, 5, candidates=m, device="cpu")
        out[f"cascade_m{m}_scores"] = cs
        out[f"cascade_m{m}_indices"] = ci
    np.savez_compressed(HERE / "binres.npz", **out)


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("MAXSIM_REFERENCE"),
                        help="path of the reference source tree (or set MAXSIM_REFERENCE)")
    parser.add_argument("--only-binres", action="store_true", help="write binres.npz alone")
    args = parser.parse_args()
    if not args.reference:
        parser.error("give --reference or set MAXSIM_REFERENCE")
    ref_root = Path(args.reference)
    ms = _load_reference(ref_root)
    from maxsim import cascade, experimental  # reference modules

    binary_residual_golden(cascade, experimental)
    if args.only_binres:
        print("binres.npz written to", HERE)
        return

    out_formats: dict[str, np.ndarray] = {}
    out_scores: dict[str, np.ndarray] = {}

    # ---- formats ---------------------------------------------------------
    docs, offsets = _ragged(24, seed=11)
    docs[3] = 0.0  # an all-zero token exercises the zero-scale rule
    out_formats["docs"] = docs
    out_formats["offsets"] = offsets
    for gran in ("tensor", "token"):
        p = experimental.pack_int4_symmetric(docs, offsets, scale_granularity=gran)
        out_formats[f"int4_{gran}_data"] = p.data
        out_formats[f"int4_{gran}_values"] = p.values
        out_formats[f"int4_{gran}_scale"] = np.array(p.scale, dtype=np.float64)
        if p.token_scale is not None:
            out_formats[f"int4_{gran}_token_scale"] = p.token_scale
    r = cascade.pack_residual_int4(docs, offsets)
    for name in ("prefix_data", "prefix_values", "prefix_token_scale", "residual_data", "residual_values",
                 "residual_token_scale"):
        out_formats[f"residual_{name}"] = getattr(r, name)
    out_formats["residual_prefix_scale"] = np.array(r.prefix_scale, dtype=np.float64)
    out_formats["residual_residual_scale"] = np.array(r.residual_scale, dtype=np.float64)
    b = ms.pack_signs(docs, offsets)
    out_formats["binary_data"] = b.data
    for kind in ("mean_abs", "l2", "mean_abs_fp16", "mean_abs_u8", "mean_abs_u4"):
        out_formats[f"binary_token_scale_{kind}"] = ms.pack_signs(docs, offsets, token_scale=kind).token_scale
    out_formats["binary_doc_scale"] = ms.pack_signs(docs, offsets, scale="doc").scale
    out_formats["binary_global_scale"] = np.array(ms.pack_signs(docs, offsets, scale="global").scale)

    # ---- scores ----------------------------------------------------------
    rng = np.random.default_rng(20260713)
    lengths = np.array([0, 1, 2, 3, 4, 7, 9, 17], dtype=np.int64)
    s_off = np.concatenate(([0], np.cumsum(lengths))).astype(np.int64)
    s_docs = rng.normal(size=(int(s_off[-1]), 128)).astype(np.float32)
    s_query = rng.normal(size=(2, 5, 128)).astype(np.float32)
    s_weights = np.array([[1.0, 0.25, 1.5, 0.0, 0.75], [0.5, 2.0, 0.125, 1.0, 0.25]], dtype=np.float32)
    s_cands = np.array([5, 1, 5, 0, 2, 7], dtype=np.int64)
    out_scores.update(docs=s_docs, offsets=s_off, query=s_query, weights=s_weights, candidates=s_cands)

    binary = ms.pack_signs(s_docs, s_off)
    binary_ts = ms.pack_signs(s_docs, s_off, token_scale="mean_abs_fp16")
    binary_doc = ms.pack_signs(s_docs, s_off, scale="doc")
    int4_t = experimental.pack_int4_symmetric(s_docs, s_off)
    int4_p = experimental.pack_int4_symmetric(s_docs, s_off, scale_granularity="token")
    resid = cascade.pack_residual_int4(s_docs, s_off)
    for reducer in REDUCERS:
        kw = {"query_weights": s_weights} if reducer == "weighted_maxsim" else {}
        if reducer == "smoothsim":
            kw = {"temperature": 0.7}
        for name, packed in (("binary", binary), ("binary_ts", binary_ts), ("binary_doc", binary_doc),
                             ("int4_tensor", int4_t), ("int4_token", int4_p)):
            out_scores[f"{name}_{reducer}_full"] = ms.score(s_query, packed, reducer=reducer, device="cpu", **kw)
            out_scores[f"{name}_{reducer}_cand"] = ms.score(
                s_query, packed, reducer=reducer, device="cpu", candidate_indices=s_cands, **kw)
        out_scores[f"residual_{reducer}_full"] = cascade.residual_score(s_query, resid, device="cpu", reducer=reducer, **kw)
        out_scores[f"residual_{reducer}_cand"] = cascade.residual_score(
            s_query, resid, device="cpu", reducer=reducer, candidate_indices=s_cands, **kw)

    # top-k with ties (tests/test_api_reference.py:443 style)
    tie_docs = np.array([[1] * 8, [1] * 8, [-1] * 8, [1, -1] * 4], dtype=np.float32)
    tie_q = np.array([[[1] * 8], [[-1] * 8]], dtype=np.float32)
    ts, ti = ms.topk_maxsim(tie_q, ms.pack_signs(tie_docs), k=3)
    out_scores.update(tie_docs=tie_docs, tie_query=tie_q, tie_top_scores=ts, tie_top_indices=ti)

    # larger clustered corpus: top-k and cascade
    c_docs, c_off = _ragged(160, seed=5, lo=2, hi=16, empty_at=7)
    c_query = np.random.default_rng(6).standard_normal((3, 8, 128)).astype(np.float32)
    c_res = cascade.pack_residual_int4(c_docs, c_off)
    out_scores.update(c_docs=c_docs, c_offsets=c_off, c_query=c_query)
    for m in (10, 40, 160):
        cs, ci = cascade.cascade_topk(c_query, c_res, 5, candidates=m, device="cpu")
        out_scores[f"cascade_m{m}_scores"] = cs
        out_scores[f"cascade_m{m}_indices"] = ci
    c_int4 = experimental.pack_int4_symmetric(c_docs, c_off, scale_granularity="token")
    ks, ki = experimental.topk_int4_maxsim(c_query, c_int4, 10, device="cpu")
    out_scores.update(c_int4_top_scores=ks, c_int4_top_indices=ki)
    lut = [sys.modules["maxsim._maxsim_cpp"].maxsim_lut(q, ms.pack_signs(c_docs, c_off).data, c_off, 128, 1.0)
           for q in c_query] if "maxsim._maxsim_cpp" in sys.modules else []
    if lut:
        out_scores["c_binary_lut"] = np.stack(lut)

    # ---- int8q helpers of the reference tests ---------------------------
    int4_helper = _load_test_helper(ref_root, "test_int4_int8q", "_reference_int8q_scores")
    bin_helper = _load_test_helper(ref_root, "test_binary_int8q", "_reference_binary_int8q_scores")
    q_docs, q_off = _ragged(150, seed=71)
    q_query = np.random.default_rng(73).standard_normal((2, 5, 128)).astype(np.float32)
    q_query[1, -1] = 0.0
    out_int8q = dict(docs=q_docs, offsets=q_off, query=q_query)
    for gran in ("tensor", "token"):
        p = experimental.pack_int4_symmetric(q_docs, q_off, scale_granularity=gran)
        out_int8q[f"int4_{gran}"] = int4_helper(p, q_query)
    out_int8q["binary"] = bin_helper(q_docs, q_off, q_query)
    fp16 = ms.pack_signs(q_docs, q_off, token_scale="mean_abs_fp16")
    out_int8q["binary_ts"] = bin_helper(q_docs, q_off, q_query, token_scales=fp16.token_scale)

    np.savez_compressed(HERE / "formats.npz", **out_formats)
    np.savez_compressed(HERE / "scores.npz", **out_scores)
    np.savez_compressed(HERE / "int8q.npz", **out_int8q)

    # ---- Index.save layout per mode --------------------------------------
    i_docs, i_off = _ragged(6, seed=17, lo=2, hi=7, empty_at=None)
    ids = [f"doc-{i}" for i in range(6)]
    search = {}
    iq = np.random.default_rng(18).standard_normal((2, 3, 128)).astype(np.float32)
    rerank = {}
    for mode in ("binary", "binary_token_scale", "binary_token_scale_u8", "binary_token_scale_u4", "int4",
                 "int4_per_token", "int4_residual", "max_speed", "balanced", "compact", "max_quality", "auto",
                 "binary_q40", "pooled_binary", "max_compression"):
        idx = ms.Index.from_embeddings(ids, i_docs, i_off, mode=mode, metadata={"seed": 17})
        idx.save(HERE / f"index_{mode}.npz")
        reranker = ms.Reranker(idx, device="cpu")
        res = reranker.search(iq, k=3)
        search[mode] = [[(r.doc_id, float(r.score), r.rank) for r in row] for row in res]
        rr = reranker.rerank(iq, ["doc-4", "doc-1", "doc-5", "doc-1"], k=2)
        rerank[mode] = [[(r.doc_id, float(r.score), r.rank) for r in row] for row in rr]
    (HERE / "sdk_rerank.json").write_text(json.dumps(rerank, indent=1, sort_keys=True))
    np.savez_compressed(HERE / "index_inputs.npz", docs=i_docs, offsets=i_off, query=iq)
    (HERE / "sdk_search.json").write_text(json.dumps(search, indent=1, sort_keys=True))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
