"""The reference's own, unmodified Python package running on this library.

``tests/install_reference.py`` installs the reference package from its source
tree into ``baseline/_ref``.  Its modules import their CUDA extension as
``maxsim._maxsim_cuda`` (``src/maxsim/_api.py:13-16``,
``src/maxsim/experimental.py:279``) and probe it with ``hasattr`` /
``getattr``, so a missing method silently changes their routing instead of
failing.  Here ``sys.modules["maxsim._maxsim_cuda"]`` is this library's
``maxsim_b200._maxsim_cuda`` before the reference package is imported, which
is the whole integration.

* CPU: every attribute the reference probes exists on the module and on its
  two handle classes, and the reference package resolved its extension to it.
* GPU: ``Index.from_embeddings`` -> ``Reranker(device="cuda").search`` of the
  reference package, for int4_per_token with int4_query="int8" (bit-exact
  against the C oracle's restatement of the reference kernel), int4_per_token
  with fp32 queries, int4_residual with rescore_candidates, binary and
  binary_token_scale (against the reference's own CPU search, 1e-4 relative,
  ids equal except where scores tie within that tolerance).

Skipped when the reference package is not installed.
"""

import sys
from pathlib import Path

import numpy as np
import pytest

from oracle import reference_cpu as ref

REPO = Path(__file__).resolve().parent.parent
REF_DIR = REPO / "baseline" / "_ref"
RTOL, ATOL = 1e-4, 1e-4

# Attributes the reference's modules look up on the extension (file:line in src/maxsim).
MODULE_ATTRS = ["CudaPackedDocs", "CudaInt4PackedDocs", "maxsim_cuda", "maxsim_cuda_batch"]  # _api 127/357/371
BINARY_ATTRS = ["set_scale_vector", "set_token_scale_vector", "has_scale_vector", "topk_lut_batch", "maxsim_batch",
                "topk_batch", "score_batch", "score_candidates_batch", "topk_centroid_batch", "maxsim_batch_int8q",
                "topk_batch_int8q", "packed_size"]  # _api 134-138/287/467/619/704/719, experimental 64/159
INT4_ATTRS = ["set_token_scale_vector", "set_residual_int4", "has_token_scale_vector", "has_residual_int4",
              "maxsim_batch", "maxsim_batch_int8q", "topk_batch", "topk_batch_int8q", "score_batch",
              "score_candidates_batch", "score_residual_batch", "score_residual_candidates_batch", "dim", "num_docs",
              "num_tokens", "packed_size"]  # experimental 292/390/450/515/519, cascade 107/249/571-576


def _reference():
    """The reference package with this library as its CUDA extension (imported once per process)."""
    if not (REF_DIR / "maxsim" / "__init__.py").exists():
        pytest.skip("reference package not installed (python tests/install_reference.py --reference <path>)")
    from maxsim_b200 import _maxsim_cuda as shim

    mod = sys.modules.get("maxsim")
    if mod is None:
        sys.modules["maxsim._maxsim_cuda"] = shim
        sys.path.insert(0, str(REF_DIR))
        try:
            import maxsim as mod
        finally:
            sys.path.remove(str(REF_DIR))
    assert Path(mod.__file__).resolve().is_relative_to(REF_DIR.resolve()), mod.__file__
    assert mod._api._maxsim_cuda is shim
    return mod


def test_reference_package_binds_this_library_and_finds_every_probed_attribute():
    mx = _reference()
    from maxsim_b200 import _maxsim_cuda as shim

    assert [a for a in MODULE_ATTRS if not hasattr(shim, a)] == []
    assert [a for a in BINARY_ATTRS if not hasattr(shim.CudaPackedDocs, a)] == []
    assert [a for a in INT4_ATTRS if not hasattr(shim.CudaInt4PackedDocs, a)] == []
    import importlib

    experimental = importlib.import_module("maxsim.experimental")
    cascade = importlib.import_module("maxsim.cascade")
    assert getattr(experimental, "_maxsim_cuda", shim) is shim
    assert getattr(cascade, "_maxsim_cuda", shim) is shim
    assert mx.Index is mx.Corpus


def _corpus(seed=0):
    docs, off = ref.clustered_corpus(300, 20, 120, seed=seed)
    q = ref.clustered_queries(docs, off, 3, 16, seed=seed + 1)
    ids = [f"doc-{i}" for i in range(300)]
    return ids, docs, off, q


def _arrays(results, ids):
    pos = {d: i for i, d in enumerate(ids)}
    s = np.array([[r.score for r in row] for row in results], np.float32)
    i = np.array([[pos[r.doc_id] for r in row] for row in results], np.int64)
    return s, i


def _assert_close_topk(got, want):
    gs, gi = got
    ws, wi = want
    np.testing.assert_allclose(gs, ws, rtol=RTOL, atol=ATOL)
    for row in range(gi.shape[0]):
        for pos in np.flatnonzero(gi[row] != wi[row]):
            assert abs(gs[row, pos] - ws[row, pos]) <= ATOL + RTOL * abs(ws[row, pos])


@pytest.mark.gpu
def test_int4_per_token_int8_queries_bit_exact():
    mx = _reference()
    ids, docs, off, q = _corpus(3)
    index = mx.Index.from_embeddings(ids, docs, off, mode="int4_per_token")
    got = _arrays(mx.Reranker(index, device="cuda", int4_query="int8").search(q, k=10), ids)
    p = index.int4_packed
    full = ref.score_int4_int8q(q, p.values, off, scale=p.scale, token_scale=p.token_scale)
    want_s, want_i = ref.topk_rows(full, 10)
    np.testing.assert_array_equal(got[1], want_i)
    np.testing.assert_array_equal(got[0], want_s)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["int4_per_token", "int4", "binary", "binary_token_scale"])
def test_fp32_queries_match_the_reference_cpu_search(mode):
    mx = _reference()
    ids, docs, off, q = _corpus(5)
    index = mx.Index.from_embeddings(ids, docs, off, mode=mode)
    want = _arrays(mx.Reranker(index, device="cpu").search(q, k=10), ids)
    got = _arrays(mx.Reranker(index, device="cuda").search(q, k=10), ids)
    _assert_close_topk(got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("m", [None, 32])
def test_int4_residual_with_rescore_candidates_matches_the_reference_cpu(m):
    mx = _reference()
    ids, docs, off, q = _corpus(7)
    index = mx.Index.from_embeddings(ids, docs, off, mode="int4_residual")
    want = _arrays(mx.Reranker(index, device="cpu").search(q, k=10, rescore_candidates=m), ids)
    got = _arrays(mx.Reranker(index, device="cuda").search(q, k=10, rescore_candidates=m), ids)
    _assert_close_topk(got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("reducer,kw", [("weighted_maxsim", "w"), ("topk2", None), ("topk4", None),
                                        ("smoothsim", "t")])
def test_binary_reducers_match_the_reference_cpu(reducer, kw):
    mx = _reference()
    ids, docs, off, q = _corpus(9)
    index = mx.Index.from_embeddings(ids, docs, off, mode="binary_token_scale")
    extra = {}
    if kw == "w":
        extra["query_weights"] = np.random.default_rng(1).uniform(0.5, 1.5, size=q.shape[1]).astype(np.float32)
    elif kw == "t":
        extra["temperature"] = 0.1
    want = _arrays(mx.Reranker(index, device="cpu").search(q, k=10, reducer=reducer, **extra), ids)
    got = _arrays(mx.Reranker(index, device="cuda").search(q, k=10, reducer=reducer, **extra), ids)
    _assert_close_topk(got, want)
