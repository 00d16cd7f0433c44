"""The allocation-free top-k entry point against the regular one, through the C ABI.

msb_docs_topk_device_noalloc serves callers that cannot call cudaMalloc (a
framework allocator owns device memory, or a latency path must not add
driver allocations); it keeps its scratch in one fixed device array inside
the library.  Each check runs it twice in a row -- the second call sees the
first call's leftovers in that shared scratch -- and compares both results
with msb_docs_topk_device on the same inputs, exactly: both compute the same
integer dots and fp32 epilogue, so scores and ids agree bit for bit.  (The
allocation-free entry point always scans on the SIMT engine; for fp32 queries
the regular one is pinned to that engine too, since its tensor-core scans
round differently in the last bits.)

This file is named to be collected last, so a run that stops at the first
failure has already run every other test; it also passes on its own in a
fresh process.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _handle_int4(rng, num_docs):
    import maxsim_b200 as m

    lengths = rng.integers(0, 90, size=num_docs)
    off = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    docs = rng.standard_normal((int(off[-1]), 128)).astype(np.float32)
    return m.int4_to_device(m.pack_int4_symmetric(docs, off, scale_granularity="token")).data


def _handle_binary(rng, num_docs):
    from maxsim_b200 import _maxsim_cuda as mc
    from oracle import reference_cpu as ref

    lengths = rng.integers(1, 40, size=num_docs)
    off = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    docs = rng.standard_normal((int(off[-1]), 128)).astype(np.float32)
    h = mc.CudaPackedDocs(ref.pack_signs(docs), off, 128)
    h.set_token_scale_vector(rng.uniform(0.5, 1.5, size=int(off[-1])).astype(np.float32))
    return h


def _opts(**kw):
    from maxsim_b200 import _lib

    o = _lib.ScoreOpts()
    o.temperature = 1.0
    o.scale = 1.0
    for key, value in kw.items():
        setattr(o, key, value)
    return o


def _topk(fn, handle, q, k, opts, stream):
    import torch

    from maxsim_b200 import _lib

    s = torch.empty((q.shape[0], k), dtype=torch.float32, device="cuda")
    i = torch.empty((q.shape[0], k), dtype=torch.int64, device="cuda")
    _lib.check(fn(handle.device_handle, ctypes.c_void_p(q.data_ptr()), q.shape[0], q.shape[1], k, ctypes.byref(opts),
                  ctypes.c_void_p(s.data_ptr()), ctypes.c_void_p(i.data_ptr()), ctypes.c_void_p(stream.cuda_stream)))
    stream.synchronize()
    return s.cpu().numpy(), i.cpu().numpy()


def _check_twice(handle, queries, k, opts):
    import torch

    from maxsim_b200 import _lib

    stream = torch.cuda.Stream()
    for q_host in queries:  # two calls in a row, different shapes
        q = torch.from_numpy(q_host).cuda()
        want = _topk(_lib.lib.msb_docs_topk_device, handle, q, k, opts, stream)
        got = _topk(_lib.lib.msb_docs_topk_device_noalloc, handle, q, k, opts, stream)
        np.testing.assert_array_equal(got[1], want[1])
        np.testing.assert_array_equal(got[0], want[0])


def test_noalloc_int8_queries_match_regular_entry_point():
    from maxsim_b200 import _lib

    rng = np.random.default_rng(5)
    h = _handle_int4(rng, 900)
    queries = [rng.standard_normal((6, 24, 128)).astype(np.float32),
               rng.standard_normal((3, 7, 128)).astype(np.float32)]
    _check_twice(h, queries, 10, _opts(reducer=_lib.REDUCER_IDS["maxsim"], query_mode=_lib.QUERY_I8))


def test_noalloc_fp32_queries_match_regular_entry_point():
    from maxsim_b200 import _lib

    rng = np.random.default_rng(6)
    h = _handle_binary(rng, 700)
    queries = [rng.standard_normal((4, 20, 128)).astype(np.float32),
               rng.standard_normal((5, 9, 128)).astype(np.float32)]
    prev = _lib.get_engine()
    _lib.set_engine(1)  # the engine the allocation-free entry point scans on
    try:
        _check_twice(h, queries, 7,
                     _opts(reducer=_lib.REDUCER_IDS["topk2"], query_mode=_lib.QUERY_F32, use_token_scale=1))
    finally:
        _lib.set_engine(prev)


def test_noalloc_rejects_work_beyond_its_scratch():
    import torch

    from maxsim_b200 import _lib

    rng = np.random.default_rng(7)
    h = _handle_int4(rng, 4200)
    # 1000 x 4200 fp32 scores = 16.8 MB > the 16 MiB scratch
    q = torch.zeros((1000, 2, 128), dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError, match="fixed scratch"):
        _topk(_lib.lib.msb_docs_topk_device_noalloc, h, q, 5, _opts(query_mode=_lib.QUERY_I8),
              torch.cuda.Stream())


def test_noalloc_refuses_host_pointers():
    """A pageable host buffer given as an output (or as the query) is refused before anything is queued:
    the kernels would otherwise dereference it on the GPU."""
    import torch

    from maxsim_b200 import _lib

    rng = np.random.default_rng(8)
    h = _handle_int4(rng, 300)
    q = torch.from_numpy(rng.standard_normal((2, 8, 128)).astype(np.float32)).cuda()
    s = torch.empty((2, 5), dtype=torch.float32, device="cuda")
    i = torch.empty((2, 5), dtype=torch.int64, device="cuda")
    host_s = np.empty((2, 5), np.float32)
    host_q = np.zeros((2, 8, 128), np.float32)
    stream = torch.cuda.Stream()
    opts = _opts(query_mode=_lib.QUERY_I8)
    fn = _lib.lib.msb_docs_topk_device_noalloc
    with pytest.raises(ValueError, match="host pointer|not a CUDA pointer"):
        _lib.check(fn(h.device_handle, ctypes.c_void_p(q.data_ptr()), 2, 8, 5, ctypes.byref(opts),
                      ctypes.c_void_p(host_s.ctypes.data), ctypes.c_void_p(i.data_ptr()),
                      ctypes.c_void_p(stream.cuda_stream)))
    with pytest.raises(ValueError, match="host pointer|not a CUDA pointer"):
        _lib.check(fn(h.device_handle, ctypes.c_void_p(host_q.ctypes.data), 2, 8, 5, ctypes.byref(opts),
                      ctypes.c_void_p(s.data_ptr()), ctypes.c_void_p(i.data_ptr()),
                      ctypes.c_void_p(stream.cuda_stream)))
    stream.synchronize()
