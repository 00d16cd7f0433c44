"""Binary-prefix residual cascade on the GPU against the oracle restatement and the reference's own code.

Format: sign bits scaled by the per-token mean |x|, plus a per-token int4
residual of x - mean|x| * sign(x).  The reference has no sign-code prefix, but
its residual cascade accepts any symmetric int4 prefix: the signs as int4 codes
+-1 with the mean |x| as the prefix's token scales are the same format, and
``tests/golden/binres.npz`` holds what the reference's ``residual_score`` and
``cascade_topk`` return for it.  Parity: fp32 scores within the fp32
tolerance, top-k ids exact, against both.
"""

import numpy as np
import pytest

from oracle import reference_cpu as ref

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-4, 1e-4


@pytest.fixture(scope="module")
def corpus():
    import maxsim_b200 as m

    docs, off = ref.clustered_corpus(300, 0, 120, seed=41)
    q = ref.clustered_queries(docs, off, 3, 16, seed=42)
    packed = m.pack_binary_residual_int4(docs, off)
    return docs, off, q, ref.pack_binary_residual(docs), m.binary_residual_to_device(packed)


@pytest.mark.parametrize("reducer", ["maxsim", "weighted_maxsim", "topk2", "topk4", "smoothsim"])
def test_fused_scores_and_candidates(corpus, reducer):
    import maxsim_b200 as m

    docs, off, q, res, dev = corpus
    kw = dict(reducer=reducer, temperature=0.1 if reducer == "smoothsim" else 1.0)
    w = np.random.default_rng(3).uniform(0.5, 1.5, size=q.shape[1]).astype(np.float32)
    if reducer == "weighted_maxsim":
        kw["query_weights"] = w
    want = ref.score_binary_residual(q, res, off, **{("weights" if k == "query_weights" else k): v
                                                      for k, v in kw.items()})
    got = m.binary_residual_score(q, dev, **kw)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)
    cands = np.array([7, 0, 299, 150, 7], np.int64)
    got_c = m.binary_residual_score(q, dev, candidate_indices=cands, **kw)
    if reducer in ("maxsim", "weighted_maxsim"):
        # the full scan runs on the tensor-core digit planes, a short candidate list on fp32 FMA chains
        np.testing.assert_allclose(got_c, got[:, cands], rtol=2e-6, atol=2e-6 * np.abs(got).max())
    else:
        np.testing.assert_array_equal(got_c, got[:, cands])  # both on the SIMT engine: identical


def test_prefix_scores_are_the_scaled_sign_scan(corpus):
    import maxsim_b200 as m

    docs, off, q, res, dev = corpus
    want = ref.score_binary_fp32(q, res["bits"], 128, off, token_scale=res["prefix_token_scale"])
    np.testing.assert_allclose(m.binary_prefix_score(q, dev), want, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("m_cand", [10, 40, 300])
def test_cascade_topk_matches_oracle(corpus, m_cand):
    import maxsim_b200 as m

    docs, off, q, res, dev = corpus
    want_s, want_i = ref.binary_cascade_topk(q, res, off, 5, m_cand)
    s, i = m.binary_cascade_topk(q, dev, 5, candidates=m_cand)
    np.testing.assert_array_equal(i, want_i)
    np.testing.assert_allclose(s, want_s, rtol=RTOL, atol=ATOL)


def test_cascade_rejects_bad_sizes(corpus):
    import maxsim_b200 as m

    docs, off, q, res, dev = corpus
    with pytest.raises(ValueError):
        m.binary_cascade_topk(q, dev, 6, candidates=5)
    with pytest.raises(ValueError):
        m.binary_cascade_topk(q, dev, 5, candidates=301)


@pytest.fixture(scope="module")
def reference_made(golden):
    """The fixture the reference's own residual code scored (``tests/golden/binres.npz``), uploaded."""
    import maxsim_b200 as m

    g = golden("binres.npz")
    return g, m.binary_residual_to_device(m.pack_binary_residual_int4(g["docs"], g["offsets"]))


@pytest.mark.parametrize("reducer", ["maxsim", "weighted_maxsim", "topk2", "topk4", "smoothsim"])
def test_scores_match_reference_golden(reference_made, reducer):
    import maxsim_b200 as m

    g, dev = reference_made
    kw = dict(reducer=reducer, temperature=0.1 if reducer == "smoothsim" else 1.0)
    if reducer == "weighted_maxsim":
        kw["query_weights"] = g["weights"]
    np.testing.assert_allclose(m.binary_residual_score(g["query"], dev, **kw), g[f"{reducer}_full"],
                               rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("m_cand", [10, 40, 120])
def test_cascade_matches_reference_golden(reference_made, m_cand):
    import maxsim_b200 as m

    g, dev = reference_made
    s, i = m.binary_cascade_topk(g["query"], dev, 5, candidates=m_cand)
    np.testing.assert_array_equal(i, g[f"cascade_m{m_cand}_indices"])
    np.testing.assert_allclose(s, g[f"cascade_m{m_cand}_scores"], rtol=RTOL, atol=ATOL)
