"""Document-sharded search on CPU ranks (gloo): shard planning and the merge protocol.

The GPU path (``ShardedReranker.search_device``) scans a contiguous document
shard per rank, writes its local top-k (local ids, padded to exactly k entries
with (-inf, INT64_MAX)) into one send block, all-gathers the blocks and merges
them in (score desc, global id asc) order.  These tests run that protocol with
two gloo ranks, local scores from the oracle and the host statement of the
merge kernel, and check that the merged result is identical to the
single-process top-k over the whole corpus, including ties across the shard
boundary and a shard holding fewer than k documents.
"""

import os
import socket

import numpy as np
import pytest

from maxsim_b200.sharded import (merge_shard_topk_host, merge_topk_host, pack_shard_block, shard_bounds,
                                 shard_offsets)
from oracle import reference_cpu as ref


def _offsets(rng, num_docs, lo=0, hi=40):
    return np.concatenate([[0], np.cumsum(rng.integers(lo, hi, size=num_docs))]).astype(np.int64)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_bounds_cover_and_balance(world):
    rng = np.random.default_rng(world)
    off = _offsets(rng, 500, 1, 60)
    b = shard_bounds(off, world)
    assert b[0] == 0 and b[-1] == 500 and len(b) == world + 1
    assert np.all(np.diff(b) >= 1)
    tokens = off[b[1:]] - off[b[:-1]]
    # each shard is within one document of an equal token share
    assert np.all(np.abs(tokens - off[-1] / world) <= 60)


def test_shard_bounds_rejects_more_ranks_than_documents():
    with pytest.raises(ValueError, match="fewer documents than ranks"):
        shard_bounds(np.array([0, 3, 5], np.int64), 3)
    with pytest.raises(ValueError):
        shard_bounds(np.array([0, 3], np.int64), 0)


def test_shard_offsets_rebased():
    off = np.array([0, 4, 4, 9, 15], np.int64)
    np.testing.assert_array_equal(shard_offsets(off, 1, 4), [0, 0, 5, 11])
    np.testing.assert_array_equal(shard_offsets(off, 0, 1), [0, 4])


def test_merge_orders_ties_by_global_id_and_skips_padding():
    neg = np.float32(-np.inf)
    big = np.iinfo(np.int64).max
    scores = np.array([[[3.0, 1.0, neg]], [[3.0, 2.0, 1.0]]], np.float32)  # [world, B, k]
    ids = np.array([[[7, 2, big]], [[4, 9, 11]]], np.int64)
    s, i = merge_topk_host(scores, ids, 3)
    np.testing.assert_array_equal(i, [[4, 7, 9]])
    np.testing.assert_array_equal(s, [[3.0, 3.0, 2.0]])


def test_shard_block_merge_adds_first_documents_and_keeps_padding():
    neg = np.float32(-np.inf)
    big = np.iinfo(np.int64).max
    b0 = pack_shard_block(np.array([[3.0, 1.0, neg]], np.float32), np.array([[7, 2, big]], np.int64))
    b1 = pack_shard_block(np.array([[3.0, 2.0, 1.0]], np.float32), np.array([[0, 5, 6]], np.int64))
    s, i = merge_shard_topk_host(np.concatenate([b0, b1]), 2, 1, 3, [0, 4])
    np.testing.assert_array_equal(i, [[4, 7, 9]])
    np.testing.assert_array_equal(s, [[3.0, 3.0, 2.0]])


def _corpus(seed=11):
    rng = np.random.default_rng(seed)
    off = _offsets(rng, 23, 0, 30)
    docs = rng.standard_normal((int(off[-1]), 128)).astype(np.float32)
    # duplicate a document across the two shards so their scores tie exactly
    d_src, d_dst = 2, 20
    n_src = int(off[d_src + 1] - off[d_src])
    lengths = np.diff(off)
    lengths[d_dst] = n_src
    new_off = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    new_docs = np.concatenate([docs[off[d]:off[d + 1]] if d != d_dst else docs[off[d_src]:off[d_src + 1]]
                               for d in range(23)]).astype(np.float32)
    q = rng.standard_normal((3, 9, 128)).astype(np.float32)
    return new_off, new_docs, q


def _rank_main(rank, world, port, k, bounds, result_path):
    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        off, docs, q = _corpus()
        data, values, scale, ts = ref.pack_int4(docs, "token")
        lo, hi = int(bounds[rank]), int(bounds[rank + 1])
        loc_off = shard_offsets(off, lo, hi)
        loc_vals = values[off[lo]:off[hi]]
        loc_scores = ref.score_int4_int8q(q, loc_vals, loc_off, scale=scale, token_scale=ts[off[lo]:off[hi]])
        k_local = min(k, hi - lo)
        s, i = ref.topk_rows(loc_scores, k_local)
        pad_s = np.full((q.shape[0], k), -np.inf, np.float32)
        pad_i = np.full((q.shape[0], k), np.iinfo(np.int64).max, np.int64)
        pad_s[:, :k_local], pad_i[:, :k_local] = s, i  # local ids; the merge adds the rank's first document
        send = torch.from_numpy(pack_shard_block(pad_s, pad_i))
        blocks = [torch.empty_like(send) for _ in range(world)]
        dist.all_gather(blocks, send)
        ms, mi = merge_shard_topk_host(torch.cat(blocks).numpy(), world, q.shape[0], k, bounds[:-1])
        if rank == 0:
            np.savez(result_path, s=ms, i=mi)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


@pytest.mark.parametrize("k,split", [(5, None), (6, 20)])
def test_two_gloo_ranks_merge_equals_single_process(tmp_path, k, split):
    """Two CPU ranks: the merged top-k equals the whole-corpus top-k exactly.

    ``split=20`` leaves the second rank only 3 documents (< k), exercising the
    padding; the duplicated document (ids 2 and 20) ties across the shards.
    """
    import torch.multiprocessing as mp

    off, docs, q = _corpus()
    data, values, scale, ts = ref.pack_int4(docs, "token")
    full = ref.score_int4_int8q(q, values, off, scale=scale, token_scale=ts)
    want_s, want_i = ref.topk_rows(full, k)
    assert full[0, 2] == full[0, 20]  # the planted tie
    bounds = shard_bounds(off, 2) if split is None else np.array([0, split, 23], np.int64)
    result = str(tmp_path / "merged.npz")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    mp.spawn(_rank_main, args=(2, _free_port(), k, bounds, result), nprocs=2, join=True)
    got = np.load(result)
    np.testing.assert_array_equal(got["i"], want_i)
    np.testing.assert_array_equal(got["s"], want_s)
