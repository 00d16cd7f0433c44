"""Document-sharded search over NCCL on two and four GPUs against single-GPU search.

Two or four ranks (one process per GPU, NCCL over 127.0.0.1) each hold a
contiguous document shard; ``ShardedReranker.search`` must return exactly the
top-k of one handle holding the whole corpus: same ids, same scores, ties
across shard boundaries resolved to the lower global id.  One case leaves the
second shard fewer documents than k.  Skipped with fewer GPUs than ranks.
"""

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _corpus():
    rng = np.random.default_rng(21)
    lengths = rng.integers(1, 300, size=301)
    lengths[300] = lengths[3]
    off = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    docs = rng.standard_normal((int(off[-1]), 128)).astype(np.float32)
    docs[off[300]:off[301]] = docs[off[3]:off[4]]  # document 300 duplicates document 3 (exact tie)
    q = rng.standard_normal((6, 24, 128)).astype(np.float32)
    q[:, :4] = docs[off[3]:off[3] + 4]  # make the duplicated pair rank near the top
    return off, docs, q


def _rank_main(rank, world, port, k, split, result_path):
    import torch
    import torch.distributed as dist

    import maxsim_b200 as m
    from maxsim_b200 import _maxsim_cuda as mc
    from maxsim_b200.sharded import ShardedReranker, ShardInfo, shard_bounds, shard_offsets

    torch.cuda.set_device(rank)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        off, docs, q = _corpus()
        packed = m.pack_int4_symmetric(docs, off, scale_granularity="token")
        bounds = shard_bounds(off, world) if split is None else np.array([0, split, len(off) - 1], np.int64)
        assert len(bounds) == world + 1
        lo, hi = int(bounds[rank]), int(bounds[rank + 1])
        t_lo, t_hi = int(off[lo]), int(off[hi])
        local = mc.CudaInt4PackedDocs(np.ascontiguousarray(packed.data[t_lo:t_hi]), shard_offsets(off, lo, hi), 128,
                                      1.0)
        local.set_token_scale_vector(np.ascontiguousarray(packed.token_scale[t_lo:t_hi]))
        info = ShardInfo(rank=rank, world_size=world, doc_lo=lo, doc_hi=hi, num_docs_total=len(off) - 1)
        s, i = ShardedReranker(local, info, int8_query=True).search(q, k)
        if rank == 0:
            full = m.int4_to_device(packed).data
            want_s, want_i = full.topk_batch_int8q(q, k)
            np.savez(result_path, s=s, i=i, want_s=want_s, want_i=want_i)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,k,split", [(2, 10, None), (2, 12, 292), (4, 10, None)])
def test_sharded_search_equals_single_gpu(tmp_path, world, k, split):
    import torch

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    result = str(tmp_path / "sharded.npz")
    mp.spawn(_rank_main, args=(world, _free_port(), k, split, result), nprocs=world, join=True)
    got = np.load(result)
    np.testing.assert_array_equal(got["i"], got["want_i"])
    np.testing.assert_array_equal(got["s"], got["want_s"])
    assert any(3 in row and 300 in row for row in got["i"])  # the cross-shard tie is inside the top-k


@pytest.mark.parametrize("world,batch,k", [(2, 3, 10), (8, 64, 10), (40, 5, 7), (3, 2, 700)])
def test_merge_kernel_equals_host_statement(world, batch, k):
    """msb_merge_shard_topk_device on one GPU, fed a gathered buffer as the all-gather leaves it: ranks with
    ties inside and across shards, a short shard padded with (-inf, INT64_MAX), more ranks than a warp has
    lanes, and long lists; equal to the host statement of the merge."""
    import ctypes

    import torch

    from maxsim_b200 import _lib
    from maxsim_b200.sharded import merge_shard_topk_host, pack_shard_block

    rng = np.random.default_rng(world * 100 + k)
    sizes = rng.integers(k // 2, 3 * k, size=world)
    sizes[0] = max(1, k // 3)  # a shard with fewer than k documents
    first = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.int64)
    blocks = []
    for r in range(world):
        # coarse scores so that ties are common, within and across shards
        full = rng.integers(-20, 20, size=(batch, int(sizes[r]))).astype(np.float32) * np.float32(0.25)
        s = np.full((batch, k), -np.inf, np.float32)
        i = np.full((batch, k), np.iinfo(np.int64).max, np.int64)
        for b in range(batch):
            order = np.lexsort((np.arange(sizes[r]), -full[b]))[:k]
            s[b, :len(order)], i[b, :len(order)] = full[b][order], order
        blocks.append(pack_shard_block(s, i))
    gathered = np.concatenate(blocks)
    want_s, want_i = merge_shard_topk_host(gathered, world, batch, k, first)
    g = torch.from_numpy(gathered).cuda()
    fd = torch.from_numpy(first).cuda()
    out_s = torch.empty((batch, k), dtype=torch.float32, device="cuda")
    out_i = torch.empty((batch, k), dtype=torch.int64, device="cuda")
    _lib.check(_lib.lib.msb_merge_shard_topk_device(ctypes.c_void_p(g.data_ptr()), world, batch, k,
                                                    ctypes.c_void_p(fd.data_ptr()), ctypes.c_void_p(out_s.data_ptr()),
                                                    ctypes.c_void_p(out_i.data_ptr()), None))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out_i.cpu().numpy(), want_i)
    np.testing.assert_array_equal(out_s.cpu().numpy(), want_s)
