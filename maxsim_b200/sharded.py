"""Document-sharded multi-GPU search: one process per GPU, NCCL all-gather merge.

The reference is single-GPU; this is the one parallel strategy the scoring
path admits.  Documents are independent, so each rank holds a contiguous
document shard (balanced by token count), scans it with the int4 / binary
kernels and keeps a local top-k with *global* document ids.  The only
exchange is an all-gather of ``[batch, k]`` scores and ids (``B*k*12`` bytes
per rank) over NVLink, followed by an on-device merge with the same
(score desc, id asc) order as the single-GPU path, so sharded results are
bit-identical to single-GPU results.

The collective goes through ``torch.distributed`` (backend ``nccl`` on GPUs,
``gloo`` in the CPU tests); the merge is ``msb_topk_rows_device``.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np


def shard_bounds(offsets: np.ndarray, world_size: int) -> np.ndarray:
    """Contiguous document shards with near-equal token counts.

    Returns ``bounds`` of length ``world_size + 1``: rank ``r`` owns documents
    ``[bounds[r], bounds[r+1])``.  Every rank gets at least one document when
    there are enough documents.
    """
    offsets = np.asarray(offsets, dtype=np.int64)
    num_docs = offsets.shape[0] - 1
    if world_size < 1:
        raise ValueError("world_size must be >= 1")
    if num_docs < world_size:
        raise ValueError("fewer documents than ranks")
    total = int(offsets[-1])
    bounds = [0]
    for r in range(1, world_size):
        target = total * r / world_size
        d = int(np.searchsorted(offsets, target, side="left"))
        d = min(max(d, bounds[-1] + 1), num_docs - (world_size - r))
        bounds.append(d)
    bounds.append(num_docs)
    return np.asarray(bounds, dtype=np.int64)


def shard_offsets(offsets: np.ndarray, lo: int, hi: int) -> np.ndarray:
    """Offsets of documents ``[lo, hi)`` rebased to start at 0."""
    offsets = np.asarray(offsets, dtype=np.int64)
    return offsets[lo:hi + 1] - offsets[lo]


@dataclass
class ShardInfo:
    rank: int
    world_size: int
    doc_lo: int          # global id of this rank's first document
    doc_hi: int
    num_docs_total: int


class ShardedReranker:
    """Top-k search over a document-sharded corpus.

    ``local`` is this rank's resident corpus handle (``CudaInt4PackedDocs`` or
    ``CudaPackedDocs``) holding documents ``[info.doc_lo, info.doc_hi)``.
    ``search_device`` is the hot path (device tensors in and out, no host
    synchronisation); ``search`` is the host-buffer convenience wrapper.

    Per call: the local top-k is written straight into this rank's send block
    (``[B, k]`` fp32 scores, then ``[B, k]`` int64 local ids: ``16*B*k``
    bytes), one ``all_gather_into_tensor`` concatenates the blocks in rank
    order, and ``msb_merge_shard_topk_device`` merges them in place into the
    output buffers (global id = local id + the rank's first document).  All
    buffers are allocated once per (batch, k) and reused.  ``first_docs``
    (every rank's first global document, in rank order) is gathered from the
    ranks on the first search when not given.
    """

    def __init__(self, local, info: ShardInfo, *, int8_query: bool = True, group=None, first_docs=None):
        import torch
        import torch.distributed as dist

        self.local = local
        self.info = info
        self.int8_query = bool(int8_query)
        self.group = group
        self._torch = torch
        self._dist = dist
        self._bufs = {}
        self._first_docs = None if first_docs is None else np.asarray(first_docs, dtype=np.int64)
        self._first_docs_dev = {}

    @classmethod
    def load(cls, path, *, rank: int, world_size: int, int8_query: bool = True, group=None, **load_kw):
        """This rank's shard of a saved int4 index, streamed from the file into the current CUDA
        device (``maxsim_b200.loader``): each rank reads only its own documents' bytes."""
        from maxsim_b200.loader import load_resident_corpus

        with np.load(path, allow_pickle=False) as data:
            offsets = np.ascontiguousarray(data["doc_offsets"], dtype=np.int64)
        bounds = shard_bounds(offsets, world_size)
        lo, hi = int(bounds[rank]), int(bounds[rank + 1])
        corpus = load_resident_corpus(path, doc_range=(lo, hi), **load_kw)
        if corpus.mode not in ("int4", "int4_per_token"):
            raise ValueError("ShardedReranker.load supports the int4 and int4_per_token modes")
        info = ShardInfo(rank=rank, world_size=world_size, doc_lo=lo, doc_hi=hi,
                         num_docs_total=offsets.shape[0] - 1)
        return cls(corpus.int4_packed.data, info, int8_query=int8_query, group=group, first_docs=bounds[:-1])

    def _first_docs_on(self, device):
        """Every rank's first global document id, as a device tensor (gathered once if not given)."""
        t = self._torch
        if self._first_docs is None:
            mine = t.tensor([self.info.doc_lo], dtype=t.int64, device=device)
            allr = t.empty(self.info.world_size, dtype=t.int64, device=device)
            self._dist.all_gather_into_tensor(allr, mine, group=self.group)
            self._first_docs = allr.cpu().numpy()
        key = str(device)
        if key not in self._first_docs_dev:
            self._first_docs_dev[key] = t.as_tensor(self._first_docs, dtype=t.int64).to(device)
        return self._first_docs_dev[key]

    def _buffers(self, batch: int, k: int, device):
        key = (batch, k, str(device))
        if key not in self._bufs:
            t = self._torch
            w = self.info.world_size
            n = batch * k
            send = t.empty(2 * n, dtype=t.int64, device=device)  # [scores fp32 (8*n bytes reserved) | ids]
            self._bufs[key] = dict(
                send=send,
                loc_s=send[:n].view(t.float32)[:n].view(batch, k),
                loc_i=send[n:].view(batch, k),
                gathered=t.empty(w * 2 * n, dtype=t.int64, device=device),
                out_s=t.empty((batch, k), dtype=t.float32, device=device),
                out_i=t.empty((batch, k), dtype=t.int64, device=device),
            )
        return self._bufs[key]

    def search_device(self, query, k: int):
        """``query``: device fp32 ``[B, Q, dim]``.  Returns device ``(scores, ids)`` ``[B, k]`` (buffers
        reused by the next call with the same batch and k)."""
        from maxsim_b200 import _lib

        t = self._torch
        batch = int(query.shape[0])
        k = int(k)
        local_docs = self.info.doc_hi - self.info.doc_lo
        if k < 1 or k > self.info.num_docs_total:
            raise ValueError("k must be between 1 and the number of documents")
        k_local = min(k, local_docs)
        stream = t.cuda.current_stream(query.device).cuda_stream
        buf = self._buffers(batch, k, query.device)
        if self.info.world_size == 1:
            self.local.topk_batch_device(query, k, buf["out_s"], buf["out_i"], int8_query=self.int8_query,
                                         stream=stream)
            if self.info.doc_lo:
                buf["out_i"].add_(self.info.doc_lo)
            return buf["out_s"], buf["out_i"]
        first_docs = self._first_docs_on(query.device)
        if k_local == k:
            self.local.topk_batch_device(query, k, buf["loc_s"], buf["loc_i"], int8_query=self.int8_query,
                                         stream=stream)
        else:
            # Every rank contributes exactly k entries so the all-gather shapes agree; a shard with fewer
            # than k documents pads with (-inf, INT64_MAX), which the merge order never selects while
            # k <= the total number of documents.
            part = self._buffers(batch, k_local, query.device)
            self.local.topk_batch_device(query, k_local, part["out_s"], part["out_i"],
                                         int8_query=self.int8_query, stream=stream)
            buf["loc_s"].fill_(float("-inf"))
            buf["loc_i"].fill_(np.iinfo(np.int64).max)
            buf["loc_s"][:, :k_local].copy_(part["out_s"])
            buf["loc_i"][:, :k_local].copy_(part["out_i"])
        self._dist.all_gather_into_tensor(buf["gathered"], buf["send"], group=self.group)
        _lib.check(_lib.lib.msb_merge_shard_topk_device(
            ctypes.c_void_p(buf["gathered"].data_ptr()), self.info.world_size, batch, k,
            ctypes.c_void_p(first_docs.data_ptr()), ctypes.c_void_p(buf["out_s"].data_ptr()),
            ctypes.c_void_p(buf["out_i"].data_ptr()), ctypes.c_void_p(stream)))
        return buf["out_s"], buf["out_i"]

    def search(self, query_host, k: int = 10):
        """Host fp32 ``[B, Q, dim]`` in, host ``(scores, global ids)`` out (every rank gets the result)."""
        t = self._torch
        q = t.as_tensor(np.ascontiguousarray(query_host, dtype=np.float32))
        if q.ndim != 3:
            raise ValueError("query must have shape [batch, query_tokens, dim]")
        dq = q.to(f"cuda:{t.cuda.current_device()}", non_blocking=True)
        s, i = self.search_device(dq, k)
        return s.cpu().numpy(), i.cpu().numpy()


def pack_shard_block(scores: np.ndarray, local_ids: np.ndarray) -> np.ndarray:
    """One rank's send block as ``search_device`` lays it out: ``[B, k]`` fp32 scores in the first
    ``8*B*k`` bytes (the second half of them unused), then ``[B, k]`` int64 local ids; as int64
    ``[2*B*k]``."""
    s = np.ascontiguousarray(scores, dtype=np.float32)
    n = s.size
    block = np.zeros(2 * n, dtype=np.int64)
    block[:n].view(np.float32)[:n] = s.reshape(-1)
    block[n:] = np.asarray(local_ids, dtype=np.int64).reshape(-1)
    return block


def merge_shard_topk_host(gathered: np.ndarray, world: int, batch: int, k: int, first_docs) -> tuple:
    """Host statement of ``msb_merge_shard_topk_device`` (the CPU tests' merge): ``gathered`` is the
    concatenation of ``world`` blocks from :func:`pack_shard_block`; order score desc, global id asc."""
    g = np.asarray(gathered, dtype=np.int64).reshape(world, 2 * batch * k)
    n = batch * k
    big = np.iinfo(np.int64).max
    scores = np.stack([g[r, :n].view(np.float32)[:n] for r in range(world)]).reshape(world, batch, k)
    lids = g[:, n:].reshape(world, batch, k)
    gids = np.where(lids == big, big, lids + np.asarray(first_docs, np.int64)[:, None, None])
    return merge_topk_host(scores, gids, k)


def merge_topk_host(scores: np.ndarray, ids: np.ndarray, k: int):
    """Host-side statement of the merge order: score desc, global id asc.

    ``scores``/``ids``: ``[world, B, k_local]``.  Used by the CPU (gloo) tests of
    the sharding logic; the product merge runs on the GPU.
    """
    w, b, kl = scores.shape
    s = scores.transpose(1, 0, 2).reshape(b, w * kl)
    i = ids.transpose(1, 0, 2).reshape(b, w * kl)
    out_s = np.empty((b, k), np.float32)
    out_i = np.empty((b, k), np.int64)
    for r in range(b):
        order = np.lexsort((i[r], -s[r]))[:k]
        out_s[r], out_i[r] = s[r][order], i[r][order]
    return out_s, out_i
