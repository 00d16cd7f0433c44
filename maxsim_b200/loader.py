"""Load-to-GPU path: stream a saved index straight into resident device arrays.

The reference loads an index on the host and then uploads it: ``Corpus.load``
(src/maxsim/sdk.py:331-400) decompresses every array of the ``.npz`` into host memory and
unpacks the int4 codes into int8 values (two bytes of host memory per stored byte), then
``int4_to_device`` (src/maxsim/experimental.py:271-305) builds ``CudaInt4PackedDocs``
(cpp/maxsim/cuda_extension.cu:2679-2773), which checks every token scale in a host loop and
copies each array with one synchronous ``cudaMemcpy``.

Here the large arrays (int4 codes, token scales, the residual stream) are decompressed chunk by
chunk from their zip members into page-locked staging buffers and copied asynchronously into the
handle's device arrays (``msb_docs_create_for_upload`` / ``msb_docs_upload``) while the next chunk
decompresses; the token scales are checked on the device (``msb_docs_upload_finish``).  The codes
never exist on the host as a whole, and no int8 values are made.  The small arrays (ids, offsets,
metadata) and the token scales (which the resident payload keeps on the host, as the reference's
does) are read normally.  ``doc_range`` uploads one contiguous range of documents (a shard), reading
only the bytes of that range from each member's stream.

The results are those of ``Reranker.load`` on the same file: the device arrays hold the same bytes.
"""

from __future__ import annotations

import ctypes
import json
import time
import zipfile
from pathlib import Path

import numpy as np
from numpy.lib import format as npy_format


def _native():
    """The C-ABI library, imported on first use (the package imports without a built library)."""
    from maxsim_b200 import _lib

    return _lib

_STREAMED_MODES = frozenset({"int4", "int4_per_token", "int4_residual"})


class _Member:
    """Sequential reader of one ``.npy`` member of an ``.npz`` archive (header parsed, data streamed)."""

    def __init__(self, archive: zipfile.ZipFile, name: str):
        try:
            self._fp = archive.open(name + ".npy")
        except KeyError as exc:
            raise KeyError(f"{name} is not a file in the archive") from exc
        version = npy_format.read_magic(self._fp)
        if version == (1, 0):
            shape, fortran, dtype = npy_format.read_array_header_1_0(self._fp)
        elif version == (2, 0):
            shape, fortran, dtype = npy_format.read_array_header_2_0(self._fp)
        else:
            raise ValueError(f"unsupported .npy format version {version} for {name}")
        if fortran and len(shape) > 1:
            raise ValueError(f"serialized {name} must be C-ordered")
        self.name, self.shape, self.dtype = name, tuple(int(v) for v in shape), np.dtype(dtype)
        self.row_bytes = int(np.prod(self.shape[1:], dtype=np.int64)) * self.dtype.itemsize
        self._pos = 0

    def skip(self, nbytes: int) -> None:
        if nbytes:
            self._fp.seek(nbytes, 1)  # relative: the member's stream starts with the .npy header
            self._pos += nbytes

    def read_into(self, out: np.ndarray) -> None:
        """Fill the uint8 view ``out`` with the next ``out.size`` bytes of the array data."""
        view, done = memoryview(out), 0
        while done < out.size:
            got = self._fp.readinto(view[done:])
            if not got:
                raise ValueError(f"serialized {self.name} is truncated")
            done += got
        self._pos += out.size

    def read_array(self, count: int | None = None) -> np.ndarray:
        rows = self.shape[0] if count is None else count
        out = np.empty((rows,) + self.shape[1:], dtype=self.dtype)
        self.read_into(out.reshape(-1).view(np.uint8))
        return out

    def close(self) -> None:
        self._fp.close()


class _Staging:
    """Ring of page-locked host buffers; each slot remembers the upload ticket that reads it."""

    def __init__(self, count: int, nbytes: int):
        self.nbytes = int(nbytes)
        self._ptrs, self._views, self._tickets = [], [], []
        try:
            for _ in range(count):
                ptr = ctypes.c_void_p()
                _native().check(_native().lib.msb_pinned_alloc(self.nbytes, ctypes.byref(ptr)))
                self._ptrs.append(ptr)
                self._views.append(np.ctypeslib.as_array((ctypes.c_uint8 * self.nbytes).from_address(ptr.value)))
                self._tickets.append(0)
        except BaseException:
            self.free()
            raise
        self._next = 0

    def acquire(self, handle) -> tuple[int, np.ndarray]:
        slot = self._next
        self._next = (self._next + 1) % len(self._ptrs)
        if self._tickets[slot]:
            _native().check(_native().lib.msb_docs_upload_wait(handle, self._tickets[slot]))
            self._tickets[slot] = 0
        return slot, self._views[slot]

    def submit(self, handle, slot: int, which: int, offset: int, nbytes: int) -> None:
        ticket = ctypes.c_int64()
        _native().check(_native().lib.msb_docs_upload(handle, which, offset, self._ptrs[slot], nbytes,
                                                       ctypes.byref(ticket)))
        self._tickets[slot] = int(ticket.value)

    def drain(self, handle) -> bool:
        """Wait for every copy that reads a slot; False if a wait failed (the buffers are then kept)."""
        ok = True
        for slot, ticket in enumerate(self._tickets):
            if ticket:
                ok = _native().lib.msb_docs_upload_wait(handle, ticket) == _native().MSB_OK and ok
                self._tickets[slot] = 0
        return ok

    def free(self) -> None:
        for ptr in self._ptrs:
            _native().lib.msb_pinned_free(ptr)
        self._ptrs, self._views, self._tickets = [], [], []


def _stream_member(member: _Member, handle, which: int, first_row: int, rows: int, staging: _Staging,
                   stats: dict) -> None:
    """Upload rows [first_row, first_row + rows) of ``member`` into array ``which`` at offset 0."""
    member.skip(first_row * member.row_bytes)
    remaining, offset = rows * member.row_bytes, 0
    while remaining:
        slot, buf = staging.acquire(handle)
        n = min(remaining, staging.nbytes)
        t0 = time.perf_counter()
        member.read_into(buf[:n])
        stats["read_s"] = stats.get("read_s", 0.0) + time.perf_counter() - t0
        staging.submit(handle, slot, which, offset, n)
        offset += n
        remaining -= n
    stats["bytes"] = stats.get("bytes", 0) + rows * member.row_bytes


def _upload_host(array: np.ndarray, handle, which: int, staging: _Staging) -> None:
    flat = np.ascontiguousarray(array).reshape(-1).view(np.uint8)
    for offset in range(0, flat.size, staging.nbytes):
        slot, buf = staging.acquire(handle)
        n = min(staging.nbytes, flat.size - offset)
        buf[:n] = flat[offset:offset + n]
        staging.submit(handle, slot, which, offset, n)


def _scalar(data, name):
    return np.asarray(data[name]).item()


def _u8_member(archive, name, dim):
    member = _Member(archive, name)
    if member.dtype != np.uint8:
        member.close()
        raise ValueError(f"serialized {name} must have dtype uint8")
    if len(member.shape) != 2 or member.shape[1] != dim // 2:
        member.close()
        raise ValueError("serialized packed data shape does not match dim")
    return member


def _f32_rows(archive, name, first, count, total):
    member = _Member(archive, name)
    try:
        if member.dtype != np.float32:
            raise ValueError(f"serialized {name} must have dtype float32")
        if len(member.shape) != 1 or member.shape[0] != total:
            raise ValueError(f"{name} must have shape [num_doc_tokens]")
        member.skip(first * 4)
        return member.read_array(count)
    finally:
        member.close()


def load_resident_corpus(path, *, doc_range: tuple[int, int] | None = None, chunk_bytes: int = 32 << 20,
                         staging_buffers: int = 3, stats: dict | None = None):
    """Read a saved index (``Index.save``) into a ``Corpus`` whose payload is resident on the current
    CUDA device, streaming the large arrays.  Modes other than the int4 family are read by the host
    path (``Corpus.load``) and uploaded as usual.  ``doc_range=(lo, hi)`` keeps documents [lo, hi)."""
    from maxsim_b200.cascade import ResidualInt4PackedDocs
    from maxsim_b200.experimental import Int4PackedDocs
    from maxsim_b200.sdk import Corpus, _move_corpus, _validate_offset_values
    from maxsim_b200 import _maxsim_cuda

    _lib = _native()
    lib, check = _lib.lib, _lib.check
    stats = {} if stats is None else stats
    t_start = time.perf_counter()
    source = Path(path).resolve()
    with np.load(source, allow_pickle=False) as data:
        if int(np.asarray(data["schema_version"]).item()) not in {1, 2}:
            raise ValueError("unsupported corpus schema_version")
        if str(np.asarray(data["format"]).item()) != "maxsim_corpus":
            raise ValueError("unsupported corpus format")
        mode = str(np.asarray(data["mode"]).item())
        if mode not in _STREAMED_MODES:
            corpus = Corpus.load(source)
            if doc_range is not None:
                raise ValueError(f"doc_range is supported for modes {sorted(_STREAMED_MODES)} only")
            resident = _move_corpus(corpus, "cuda")
            stats["seconds"] = time.perf_counter() - t_start
            return resident
        ids = tuple(str(v) for v in np.asarray(data["doc_ids"]))
        metadata = json.loads(str(np.asarray(data["metadata_json"]).item()))
        raw_offsets = np.asarray(data["doc_offsets"])
        if not np.issubdtype(raw_offsets.dtype, np.integer):
            raise ValueError("serialized doc_offsets must contain integers")
        offsets = np.ascontiguousarray(raw_offsets, dtype=np.int64)
        dim = int(np.asarray(data["dim"]).item())
        if dim <= 0 or dim % 8 != 0:
            raise ValueError("serialized dim must be positive and divisible by 8")
        has_token_scale = "int4_token_scale" in data.files
        prefix_scale = float(_scalar(data, "int4_scale"))
        residual_scale = float(_scalar(data, "residual_int4_scale")) if mode == "int4_residual" else 1.0
    if not np.isfinite(prefix_scale) or prefix_scale <= 0.0:
        raise ValueError("packed.scale must be a finite scalar > 0")
    if mode == "int4_residual" and (not np.isfinite(residual_scale) or residual_scale <= 0.0):
        raise ValueError("residual_scale must be a finite scalar > 0")
    if mode == "int4_residual" and not has_token_scale:
        raise ValueError("prefix_token_scale must have shape [num_doc_tokens]")
    if (mode == "int4_per_token") != has_token_scale and mode != "int4_residual":
        needs = mode == "int4_per_token"
        raise ValueError(f"mode {mode!r} {'requires' if needs else 'does not accept'} int4 token scales")
    if not ids:
        raise ValueError("corpus.doc_ids must contain at least one id")
    if len(set(ids)) != len(ids):
        raise ValueError("corpus.doc_ids must be unique")

    archive = zipfile.ZipFile(source)
    members, staging, handle = [], None, None
    try:
        codes = _u8_member(archive, "int4_data", dim)
        members.append(codes)
        total_tokens = codes.shape[0]
        _validate_offset_values(offsets, len(ids), total_tokens)
        lo, hi = (0, len(ids)) if doc_range is None else (int(doc_range[0]), int(doc_range[1]))
        if not 0 <= lo < hi <= len(ids):
            raise ValueError("doc_range must satisfy 0 <= lo < hi <= num_docs")
        t0, t1 = int(offsets[lo]), int(offsets[hi])
        local_offsets = np.ascontiguousarray(offsets[lo:hi + 1] - offsets[lo], dtype=np.int64)
        local_ids = ids[lo:hi]
        n = t1 - t0
        flags = (_lib.UPLOAD_TOKEN_SCALES if has_token_scale else 0) | \
            (_lib.UPLOAD_RESIDUAL if mode == "int4_residual" else 0)
        handle = _maxsim_cuda.CudaInt4PackedDocs._for_upload(local_offsets, n, dim, prefix_scale, flags)
        staging = _Staging(staging_buffers, chunk_bytes)
        _stream_member(codes, handle._h, _lib.ARRAY_CODES, t0, n, staging, stats)
        token_scale = None
        if has_token_scale:
            token_scale = _f32_rows(archive, "int4_token_scale", t0, n, total_tokens)
            _upload_host(token_scale, handle._h, _lib.ARRAY_TOKEN_SCALES, staging)
        residual_token_scale = None
        if mode == "int4_residual":
            residual = _u8_member(archive, "residual_int4_data", dim)
            members.append(residual)
            if residual.shape[0] != total_tokens:
                raise ValueError("residual_data must have shape [num_doc_tokens, dim / 2]")
            _stream_member(residual, handle._h, _lib.ARRAY_RESIDUAL_CODES, t0, n, staging, stats)
            residual_token_scale = _f32_rows(archive, "residual_int4_token_scale", t0, n, total_tokens)
            _upload_host(residual_token_scale, handle._h, _lib.ARRAY_RESIDUAL_TOKEN_SCALES, staging)
        status = lib.msb_docs_upload_finish(handle._h, ctypes.c_float(residual_scale))
        if status != _lib.MSB_OK:
            message = lib.msb_last_error().decode()
            # the host path's messages (experimental._validate_int4_packed, cascade._validate_residual_packed)
            for prefix, host_message in (
                    ("residual int4 codes", "residual_values must be symmetric int4 values in [-7, 7]"),
                    ("residual token scales", "residual_token_scale values must be finite and > 0"),
                    ("int4 codes", "packed.values must be symmetric int4 values in [-7, 7]"),
                    ("token scales", "packed.token_scale values must be finite and > 0")):
                if message.startswith(prefix):
                    raise ValueError(host_message)
            check(status)
    finally:
        if staging is not None:
            # no queued copy may still read a staging buffer when it is freed
            if handle is None or staging.drain(handle._h):
                staging.free()
        for member in members:
            member.close()
        archive.close()

    if mode == "int4_residual":
        payload = ResidualInt4PackedDocs(
            prefix_data=handle, prefix_values=None, prefix_scale=prefix_scale, prefix_token_scale=token_scale,
            residual_data=handle, residual_values=None, residual_scale=residual_scale,
            residual_token_scale=residual_token_scale, doc_offsets=local_offsets, dim=dim,
            num_docs=len(local_ids), device="cuda")
        object.__setattr__(payload, "_msb_validated", True)  # checked on the device and from the headers
    else:
        payload = Int4PackedDocs(data=handle, values=None, doc_offsets=local_offsets, dim=dim,
                                 num_docs=len(local_ids), scale=prefix_scale, device="cuda",
                                 token_scale=token_scale)
        object.__setattr__(payload, "_msb_validated", True)  # checked on the device and from the headers
    stats["seconds"] = time.perf_counter() - t_start
    stats["tokens"] = n
    return Corpus(doc_ids=local_ids, mode=mode, int4_packed=payload, metadata=metadata, _source_path=source)


def load_reranker(path, *, int4_query: str = "fp32", doc_range: tuple[int, int] | None = None,
                  chunk_bytes: int = 32 << 20, staging_buffers: int = 3, stats: dict | None = None):
    """``Reranker.load(path, device="cuda")`` through the streaming upload."""
    from maxsim_b200.sdk import Reranker

    corpus = load_resident_corpus(path, doc_range=doc_range, chunk_bytes=chunk_bytes,
                                  staging_buffers=staging_buffers, stats=stats)
    return Reranker._from_resident(corpus, int4_query=int4_query)


def _write_synthetic_index(path, pages: int, tokens_per_page: int, seed: int = 7, compress: bool = True) -> None:
    """A per-token int4 index in the schema ``Index.save`` writes, with random codes and scales."""
    from maxsim_b200.sdk import Index

    tiny = Path(path).with_suffix(".tiny.npz")
    ids = [f"p{i}" for i in range(2)]
    Index.from_embeddings(ids, np.ones((2, 128), np.float32), np.array([0, 1, 2]), mode="int4_per_token").save(tiny)
    with np.load(tiny) as data:
        arrays = {k: data[k] for k in data.files}
    tiny.unlink()
    rng = np.random.default_rng(seed)
    n = pages * tokens_per_page
    arrays["doc_ids"] = np.array([f"p{i}" for i in range(pages)])
    arrays["doc_offsets"] = np.arange(pages + 1, dtype=np.int64) * tokens_per_page
    values = rng.integers(-7, 8, size=(n, 128), dtype=np.int8)
    arrays["int4_data"] = ((values[:, 0::2] & 0x0F) | ((values[:, 1::2] & 0x0F) << 4)).astype(np.uint8)
    arrays["int4_token_scale"] = rng.uniform(0.01, 0.2, size=n).astype(np.float32)
    with open(path, "wb") as handle:
        (np.savez_compressed if compress else np.savez)(handle, **arrays)


def _main() -> None:
    import argparse
    import tempfile

    from maxsim_b200.sdk import Corpus, Reranker

    ap = argparse.ArgumentParser(description="time Reranker.load through the host path and the streamed path")
    ap.add_argument("--pages", type=int, default=1000)
    ap.add_argument("--tokens-per-page", type=int, default=1030)
    ap.add_argument("--stored", action="store_true", help="write the index with uncompressed members")
    args = ap.parse_args()
    with tempfile.TemporaryDirectory() as tmp:
        path = Path(tmp) / "index.npz"
        _write_synthetic_index(path, args.pages, args.tokens_per_page, compress=not args.stored)
        q = np.random.default_rng(1).standard_normal((4, 24, 128)).astype(np.float32)
        t0 = time.perf_counter()
        host = Reranker.from_corpus(Corpus.load(path), device="cuda")
        t_host = time.perf_counter() - t0
        stats = {}
        t0 = time.perf_counter()
        streamed = load_reranker(path, stats=stats)
        t_stream = time.perf_counter() - t0
        same = all(np.array_equal(a, b) for a, b in zip(host.search_arrays(q, k=10), streamed.search_arrays(q, k=10)))
        print(json.dumps({"pages": args.pages, "tokens": args.pages * args.tokens_per_page,
                          "members": "stored" if args.stored else "deflated",
                          "file_bytes": path.stat().st_size, "host_path_s": round(t_host, 3),
                          "streamed_s": round(t_stream, 3), "streamed_read_s": round(stats.get("read_s", 0.0), 3),
                          "streamed_bytes": stats.get("bytes"), "identical_results": bool(same)}))


if __name__ == "__main__":
    _main()
