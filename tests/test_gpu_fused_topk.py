"""Full-scan top-k selected inside the tensor-core scan (option tc_fused_topk; off by default, measured
slower than selecting from the score matrix).

Each CTA keeps the k best documents of every query in shared memory (score desc, document asc) and writes
them as a candidate block; a merge kernel forms the final [B, k] from the blocks and a block of the
corpus's first empty documents (score 0, never in a tile).  The results must equal the unfused path
(score matrix + row-wise selection) exactly, and the oracle's top-k: with exact ties between duplicated
documents, empty documents that outrank negative scores, k above the number of non-empty documents,
twin mode (one query tile), lists that fill the shared-memory room, and a batch too large to fuse.
"""

import numpy as np
import pytest

from oracle import reference_cpu as ref

pytestmark = pytest.mark.gpu


def _both(fn):
    from maxsim_b200 import _lib

    prev = _lib.get_option("tc_fused_topk")
    try:
        _lib.set_option("tc_fused_topk", 1)
        fused = fn()
        _lib.set_option("tc_fused_topk", 0)
        plain = fn()
    finally:
        _lib.set_option("tc_fused_topk", prev)
    return fused, plain


def _corpus(seed, num_docs=400, dup=True, empties=True):
    """Ragged documents of 1-299 tokens; documents 3, 50, 51 and the last are empty; document 300 is a copy
    of document 10 (exact ties across work units)."""
    rng = np.random.default_rng(seed)
    lengths = rng.integers(1, 300, size=num_docs)
    if empties:
        lengths[[3, 50, 51, num_docs - 1]] = 0
    if dup:
        lengths[300] = lengths[10]
    off = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    docs = rng.standard_normal((int(off[-1]), 128)).astype(np.float32)
    if dup:
        docs[off[300]:off[301]] = docs[off[10]:off[11]]
    return rng, docs, off


@pytest.mark.parametrize("batch,qtok,k", [(64, 24, 10), (1, 24, 10), (3, 20, 37), (128, 8, 8), (200, 4, 10)])
def test_fused_equals_unfused_and_oracle_int8(oracle_c, batch, qtok, k):
    import maxsim_b200 as m

    rng, docs, off = _corpus(11 + batch)
    q = rng.standard_normal((batch, qtok, 128)).astype(np.float32)
    q[0, :4] = docs[off[10]:off[10] + 4]  # the duplicated pair near the top of row 0
    packed = m.pack_int4_symmetric(docs, off, scale_granularity="token")
    h = m.int4_to_device(packed).data
    (fs, fi), (ps, pi) = _both(lambda: h.topk_batch_int8q(q, k))
    np.testing.assert_array_equal(fi, pi)
    np.testing.assert_array_equal(fs, ps)
    full = ref.score_int4_int8q(q, packed.values, off, token_scale=packed.token_scale)
    want_s, want_i = ref.topk_rows(full, k)
    np.testing.assert_array_equal(fi, want_i)
    np.testing.assert_array_equal(fs, want_s)


def test_empty_documents_outrank_negative_scores():
    """Queries opposite to every document: all scores negative, so the empty documents (score 0) lead the
    top-k in id order, then the least negative documents."""
    import maxsim_b200 as m

    rng, docs, off = _corpus(5, num_docs=120, dup=False)
    centre = docs.mean(axis=0)
    q = np.broadcast_to(-centre / np.linalg.norm(centre), (2, 3, 128)).astype(np.float32).copy()
    docs_pos = np.abs(docs) * np.sign(centre)[None, :]  # every token on the centre's side
    packed = m.pack_int4_symmetric(docs_pos.astype(np.float32), off, scale_granularity="token")
    h = m.int4_to_device(packed).data
    (fs, fi), (ps, pi) = _both(lambda: h.topk_batch_int8q(q, 8))
    np.testing.assert_array_equal(fi, pi)
    np.testing.assert_array_equal(fs, ps)
    np.testing.assert_array_equal(fi[:, :4], [[3, 50, 51, 119]] * 2)
    assert np.all(fs[:, :4] == 0.0) and np.all(fs[:, 4:] < 0.0)


@pytest.mark.parametrize("mode", ["binary_fp32", "int4_fp32", "int4_tensor_int8"])
def test_fused_other_variants(mode):
    """Digit planes (fp32 queries) over sign codes and int4, and the tensor-scale int8 variant."""
    import maxsim_b200 as m

    rng, docs, off = _corpus(21)
    q = rng.standard_normal((5, 20, 128)).astype(np.float32)
    if mode == "binary_fp32":
        packed = m.to_device(m.pack_signs(docs, off, token_scale="mean_abs_fp16"), "cuda")
        run = lambda: packed.data.topk_batch(q, 10, use_token_scale=True)
    elif mode == "int4_fp32":
        h = m.int4_to_device(m.pack_int4_symmetric(docs, off, scale_granularity="token")).data
        run = lambda: h.topk_batch(q, 10)
    else:
        h = m.int4_to_device(m.pack_int4_symmetric(docs, off, scale_granularity="tensor")).data
        run = lambda: h.topk_batch_int8q(q, 10)
    (fs, fi), (ps, pi) = _both(run)
    np.testing.assert_array_equal(fi, pi)
    np.testing.assert_array_equal(fs, ps)


def test_fused_device_entry_point_and_repeat():
    import torch

    import maxsim_b200 as m

    rng, docs, off = _corpus(31)
    h = m.int4_to_device(m.pack_int4_symmetric(docs, off, scale_granularity="token")).data
    q = torch.from_numpy(rng.standard_normal((7, 24, 128)).astype(np.float32)).cuda()
    outs = []
    for _ in range(2):
        s = torch.empty((7, 10), dtype=torch.float32, device="cuda")
        i = torch.empty((7, 10), dtype=torch.int64, device="cuda")
        h.topk_batch_device(q, 10, s, i, int8_query=True)
        torch.cuda.synchronize()
        outs.append((s.cpu().numpy(), i.cpu().numpy()))
    np.testing.assert_array_equal(outs[0][1], outs[1][1])
    want_s, want_i = h.topk_batch_int8q(q.cpu().numpy(), 10)
    np.testing.assert_array_equal(outs[0][1], want_i)
    np.testing.assert_array_equal(outs[0][0], want_s)
