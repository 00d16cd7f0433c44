"""int4 codes x fp32 queries at dim 128: the register-blocked scan against the general scan.

The blocked scan runs when the query pointer is 16-byte aligned; a query that starts 4 bytes into its
buffer takes the general kernel.  Both compute each row's dot as one FMA chain over the dims in order,
so max, weighted and top-k scores must be bit-identical; the smooth reducer sums exponentials in a
different order and is compared to 1e-6.  Every case is also held to the float64 oracle at 1e-4.  Ragged documents (empty, shorter and longer than a warp's
32 lanes and the general kernel's 128 threads), query-token counts that are not multiples of the row group, per-row candidate lists and
the two-stream residual are all covered, and the scores are checked against the float64 oracle.
"""

import numpy as np
import pytest

from oracle import reference_cpu as ref

pytestmark = pytest.mark.gpu

REDUCERS = {"maxsim": 0, "weighted_maxsim": 1, "topk2": 2, "topk4": 3, "smoothsim": 4}


@pytest.fixture(autouse=True)
def simt_engine():
    """MaxSim scans of aligned fp32 queries with up to 32 tokens would otherwise run on the
    tensor-core engine; this file compares the two SIMT kernels."""
    from maxsim_b200 import _lib

    prev = _lib.get_engine()
    _lib.set_engine(1)
    yield
    _lib.set_engine(prev)


def _handle(gran, residual, seed=5, num_docs=41, max_len=300):
    import maxsim_b200 as m
    from maxsim_b200._maxsim_cuda import CudaInt4PackedDocs

    rng = np.random.default_rng(seed)
    lengths = rng.integers(0, max_len, size=num_docs)
    lengths[[3, 17]] = 0
    lengths[9] = min(max_len, 129)
    offsets = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    n = int(offsets[-1])
    mode = "int4_residual" if residual else ("int4_per_token" if gran == "token" else "int4")
    docs = rng.standard_normal((n, 128)).astype(np.float32)
    idx = m.Index.from_embeddings([f"d{i}" for i in range(num_docs)], docs, offsets, mode=mode)
    p = idx.int4_packed
    data, scale, ts = ((p.prefix_data, p.prefix_scale, p.prefix_token_scale) if residual
                       else (p.data, p.scale, p.token_scale))
    h = CudaInt4PackedDocs(data, offsets, 128, float(scale))
    if ts is not None:
        h.set_token_scale_vector(ts)
    if residual:
        h.set_residual_int4(p.residual_data, float(p.residual_scale), p.residual_token_scale)
    return h, p, offsets


def _scores(h, q, aligned, reducer, weights=None, candidates=None, residual=False):
    import torch

    B, Q, D = q.shape
    buf = torch.zeros(B * Q * D + 4, dtype=torch.float32, device="cuda")
    at = 0 if aligned else 1  # one float in: 4-byte aligned only
    view = buf[at:at + B * Q * D].view(B, Q, D)
    view.copy_(torch.from_numpy(q))
    T = h.num_docs if candidates is None else candidates.shape[0]
    out = torch.empty(B, T, dtype=torch.float32, device="cuda")
    cand = None if candidates is None else torch.from_numpy(candidates).cuda()
    kw = {"reducer": REDUCERS[reducer], "use_residual": residual}
    if weights is not None:  # a device call takes device weights
        kw.update(weights=torch.from_numpy(weights).cuda(), weight_rows=1)
    h.score_batch_device(view, out, candidates=cand, **kw)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("residual,gran", [(False, "tensor"), (False, "token"), (True, "token")])
@pytest.mark.parametrize("qtok", [1, 7, 32, 41])
@pytest.mark.parametrize("reducer", list(REDUCERS))
def test_blocked_scan_matches_general_scan(residual, gran, qtok, reducer):
    h, p, offsets = _handle(gran, residual)
    rng = np.random.default_rng(qtok)
    q = rng.standard_normal((3, qtok, 128)).astype(np.float32)
    weights = rng.random(qtok).astype(np.float32) + 0.5 if reducer == "weighted_maxsim" else None
    got = _scores(h, q, True, reducer, weights, residual=residual)
    want = _scores(h, q, False, reducer, weights, residual=residual)
    if reducer == "smoothsim":
        np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-6)
    else:
        np.testing.assert_array_equal(got, want)
    # and both against the float64 oracle (the reference's reducers), 1e-4 of the score magnitude
    kw = {"reducer": reducer, "weights": weights}
    if residual:
        exact = ref.score_residual(q, {"prefix_values": p.prefix_values, "prefix_scale": p.prefix_scale,
                                       "prefix_token_scale": p.prefix_token_scale,
                                       "residual_values": p.residual_values, "residual_scale": p.residual_scale,
                                       "residual_token_scale": p.residual_token_scale}, offsets, **kw)
    else:
        exact = ref.score_int4_fp32(q, p.values, offsets, scale=p.scale, token_scale=p.token_scale, **kw)
    np.testing.assert_allclose(got, exact, rtol=1e-4, atol=1e-4 * max(1.0, float(np.abs(exact).max())))


@pytest.mark.parametrize("residual", [False, True])
def test_blocked_scan_large_grid(residual):
    """3,001 documents x 5 queries of 32 rows: 15,005 single-warp blocks, two row groups each."""
    h, _, _ = _handle("token", residual, seed=12, num_docs=3001, max_len=40)
    q = np.random.default_rng(4).standard_normal((5, 32, 128)).astype(np.float32)
    for reducer in ("maxsim", "topk2"):
        got = _scores(h, q, True, reducer, residual=residual)
        want = _scores(h, q, False, reducer, residual=residual)
        np.testing.assert_array_equal(got, want)


def test_blocked_scan_candidates_and_oracle():
    h, p, offsets = _handle("token", False, seed=9)
    rng = np.random.default_rng(2)
    q = rng.standard_normal((2, 32, 128)).astype(np.float32)
    cand = rng.integers(0, h.num_docs, size=23).astype(np.int64)
    got = _scores(h, q, True, "maxsim", candidates=cand)
    want = _scores(h, q, False, "maxsim", candidates=cand)
    np.testing.assert_array_equal(got, want)
    vals = ref.unpack_nibbles(p.data, 128).astype(np.float64) * p.token_scale[:, None].astype(np.float64)
    full = np.zeros((2, h.num_docs))
    for d in range(h.num_docs):
        tok = vals[offsets[d]:offsets[d + 1]] * float(p.scale)
        if tok.shape[0]:
            full[:, d] = (q.astype(np.float64) @ tok.T).max(axis=2).sum(axis=1)
    # fp32 FMA chains against float64: 1e-4 relative to the score magnitude
    np.testing.assert_allclose(got, full[:, cand], rtol=1e-4, atol=1e-4 * np.abs(full).max())


def test_device_calls_refuse_host_pointers():
    """A host array handed to a *_device call is refused on the host, before any launch."""
    import torch

    h, _, _ = _handle("tensor", False)
    q = torch.zeros(1, 4, 128, device="cuda")
    out = torch.empty(1, h.num_docs, device="cuda")
    w = np.ones(4, np.float32)
    with pytest.raises(ValueError, match="opts.weights must be device memory"):
        h.score_batch_device(q, out, reducer=REDUCERS["weighted_maxsim"], weights=w, weight_rows=1)
    with pytest.raises(ValueError, match="query must be device memory"):
        h.score_batch_device(torch.zeros(1, 4, 128), out)
    with pytest.raises(ValueError, match="out must be device memory"):
        h.score_batch_device(q, torch.empty(1, h.num_docs))
    # the handle still scores afterwards
    h.score_batch_device(q, out)
    torch.cuda.synchronize()
    assert float(out.abs().max()) == 0.0
