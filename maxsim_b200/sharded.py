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
    """

    def __init__(self, local, info: ShardInfo, *, int8_query: bool = True, group=None):
        import torch
        import torch.distributed as dist

        self.local = local
        self.info = info
        self.int8_query = bool(int8_query)
        self.group = group
        self._torch = torch
        self._dist = dist
        self._bufs = {}

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
        return cls(corpus.int4_packed.data, info, int8_query=int8_query, group=group)

    def _buffers(self, batch: int, k: int, device):
        key = (batch, k)
        if key not in self._bufs:
            t = self._torch
            w = self.info.world_size
            self._bufs[key] = dict(
                loc_s=t.empty((batch, k), dtype=t.float32, device=device),
                loc_i=t.empty((batch, k), dtype=t.int64, device=device),
                all_s=t.empty((w, batch, k), dtype=t.float32, device=device),
                all_i=t.empty((w, batch, k), dtype=t.int64, device=device),
                out_s=t.empty((batch, k), dtype=t.float32, device=device),
                out_i=t.empty((batch, k), dtype=t.int64, device=device),
            )
        return self._bufs[key]

    def search_device(self, query, k: int):
        """``query``: device fp32 ``[B, Q, dim]``.  Returns device ``(scores, ids)`` ``[B, k]``."""
        from maxsim_b200 import _lib

        t = self._torch
        batch = int(query.shape[0])
        local_docs = self.info.doc_hi - self.info.doc_lo
        k_local = min(int(k), local_docs)
        if int(k) > self.info.num_docs_total:
            raise ValueError("k cannot exceed the number of documents")
        # Every rank contributes exactly k entries so the all-gather shapes agree; a shard with fewer
        # than k documents pads with (-inf, INT64_MAX), which the merge order never selects while
        # k <= the total number of documents.
        stream = t.cuda.current_stream(query.device).cuda_stream
        buf = self._buffers(batch, int(k), query.device)
        if k_local == int(k):
            self.local.topk_batch_device(query, k_local, buf["loc_s"], buf["loc_i"], int8_query=self.int8_query,
                                         stream=stream)
            buf["loc_i"].add_(self.info.doc_lo)
        else:
            part = self._buffers(batch, k_local, query.device)
            self.local.topk_batch_device(query, k_local, part["loc_s"], part["loc_i"], int8_query=self.int8_query,
                                         stream=stream)
            buf["loc_s"].fill_(float("-inf"))
            buf["loc_i"].fill_(np.iinfo(np.int64).max)
            buf["loc_s"][:, :k_local].copy_(part["loc_s"])
            buf["loc_i"][:, :k_local].copy_(part["loc_i"]).add_(self.info.doc_lo)
        if self.info.world_size == 1:
            buf["out_s"].copy_(buf["loc_s"])
            buf["out_i"].copy_(buf["loc_i"])
            return buf["out_s"][:, :k], buf["out_i"][:, :k]
        self._dist.all_gather_into_tensor(buf["all_s"], buf["loc_s"], group=self.group)
        self._dist.all_gather_into_tensor(buf["all_i"], buf["loc_i"], group=self.group)
        cand_s = buf["all_s"].permute(1, 0, 2).reshape(batch, -1).contiguous()
        cand_i = buf["all_i"].permute(1, 0, 2).reshape(batch, -1).contiguous()
        out_s = t.empty((batch, int(k)), dtype=t.float32, device=query.device)
        out_i = t.empty((batch, int(k)), dtype=t.int64, device=query.device)
        _lib.check(_lib.lib.msb_topk_rows_device(
            ctypes.c_void_p(cand_s.data_ptr()), cand_s.shape[1], batch, cand_s.shape[1], int(k),
            ctypes.c_void_p(cand_i.data_ptr()), 1, ctypes.c_void_p(out_s.data_ptr()),
            ctypes.c_void_p(out_i.data_ptr()), ctypes.c_void_p(stream)))
        return out_s, out_i

    def search(self, query_host, k: int = 10):
        """Host fp32 ``[B, Q, dim]`` in, host ``(scores, global ids)`` out (every rank gets the result)."""
        t = self._torch
        q = t.as_tensor(np.ascontiguousarray(query_host, dtype=np.float32))
        if q.ndim != 3:
            raise ValueError("query must have shape [batch, query_tokens, dim]")
        dq = q.to(f"cuda:{t.cuda.current_device()}", non_blocking=True)
        s, i = self.search_device(dq, k)
        return s.cpu().numpy(), i.cpu().numpy()


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
