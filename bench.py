"""Full-scan top-10 benchmark of the per-token int4 x int8-query MaxSim path.

Default workload (the north-star case, which fits one
B200): 100,000 pages x 1,030 patch tokens (dim 128; per-page Gaussian centroid
+ N(0, 0.3^2) patch noise, L2-normalised, packed on the GPU to per-token int4:
6.59 GB codes + 0.41 GB scales), 1,024 queries x 24 tokens quantised to int8
per row, batch 64, top-10.  One step = one batch of 64 queries scanned against
the whole corpus (every shard) and merged to a global top-10.  Under torchrun
each rank holds a contiguous document shard (strong scaling: fixed corpus) and
the per-rank top-10 lists meet in an NCCL all-gather + on-device merge.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Prints one JSON line (rank 0).  ``value`` is device-timed with CUDA events on
the launching stream (inputs resident in HBM); ``e2e`` times the public API
(``Reranker.search`` / ``ShardedReranker.search``) from pinned host queries to
host results.  The corpus (7 GB) is far larger than L2 (126 MB), so no flush is
needed between steps.  ``--impl reference`` times the CPU restatement of the
reference's int8-query kernel (the reference has no CPU code for this path)
on all host cores over a bounded sample of pages and extrapolates.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

NUM_PAGES = 100_000
PAGE_TOKENS = 1_030
DIM = 128
NUM_QUERIES = 1_024
QUERY_TOKENS = 24
BATCH = 64
TOP_K = 10
NOISE = 0.3
SEED = 20260713
CHUNK_PAGES = 2_000
CPU_SAMPLE_PAGES = 128  # pages per step of the CPU legs (the reference arm and cpu_baseline)
# DRAM bytes (read + write) of one tc_scan_kernel launch per corpus page, from one ncu capture of a
# 2,000-page case of the same workload (profiles/tc_scan_kernel_2000pages_full.txt: 272.37 MB read +
# 3.95 MB written).  The kernel streams the resident int8 copy of the codes (128 B per token, twice
# the int4 bytes) plus the token scales once per launch and the score matrix grows with the pages,
# so traffic scales with the pages a rank holds.
TC_DRAM_BYTES_PER_PAGE = (272.367872e6 + 3.953664e6) / 2000
METRIC = "full-scan top-10 queries/s (per-token int4 x int8 query, 100k-page corpus)"
DTYPE = "int8 x int4 (int32 accumulate, fp32 epilogue)"
DATA = "synthetic (seeded per-page centroid + noise, generated on the GPU; same corpus and queries in both arms)"
WORKLOAD = ("C4: 100,000 pages x 1,030 tokens (dim 128) per-token int4 (6.59 GB codes + 0.41 GB scales); "
            "1,024 queries x 24 tokens int8, batch 64, full-scan top-10")


# RTX 4090 medians the reference publishes for these shapes (its README and raw benchmark files), for
# context only: other hardware, and the reference times some of them per query through its SDK.
REF_4090_MS = {
    ("C0", "int4 per-token full scan, fp32 query"): 8.345, ("C0", "int4 per-token full scan, int8 query"): 2.674,
    ("C0", "int4 per-token top-10, fp32 query"): 8.385, ("C0", "int4 per-token top-10, int8 query"): 2.722,
    ("C0", "int4 tensor-scale top-10, fp32 query"): 8.158, ("C0", "int4 tensor-scale top-10, int8 query"): 2.492,
    ("C0", "int4 residual fused full scan"): 16.114, ("C0", "int4 residual candidates, M=512"): 2.803,
    ("C0", "int4 per-token candidates fp32, M=512"): 1.503,
    ("C3", "int4-prefix cascade top-10, M=512"): 15.873, ("C3", "int4-prefix cascade top-10, M=2048"): 23.746,
    ("C1", "SDK search, tensor int4 + int8 query, 256 queries one by one"): 1119.6,
    ("C2", "SDK search, binary (max_speed), 256 queries one by one"): 680.0,
    ("C2", "SDK search, binary + fp16 token scale (balanced), 256 queries one by one"): 700.0,
}


def _clustered(rng, num_docs, lo, hi, dim=DIM):
    lengths = rng.integers(lo, hi + 1, size=num_docs)
    offsets = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    cent = rng.standard_normal((num_docs, dim), dtype=np.float32)
    cent /= np.linalg.norm(cent, axis=1, keepdims=True)
    docs = np.repeat(cent, lengths, axis=0)
    docs += NOISE * rng.standard_normal(docs.shape, dtype=np.float32)
    docs /= np.linalg.norm(docs, axis=1, keepdims=True)
    return docs, offsets, cent


def _queries(rng, cent, batch, qtok, dim=DIM):
    targets = rng.integers(0, cent.shape[0], size=batch)
    q = np.repeat(cent[targets][:, None, :], qtok, axis=1)
    q = q + NOISE * rng.standard_normal(q.shape, dtype=np.float32)
    return (q / np.linalg.norm(q, axis=2, keepdims=True)).astype(np.float32)


REF_CUDA_DIR = REPO / "baseline" / "_ref_cuda"


def _reference_cuda_package():
    """The reference package with its own CUDA extension, built for sm_100a from its sources into
    baseline/_ref_cuda (``MAXSIM_BUILD_CUDA=1 MAXSIM_CUDA_ARCH=100a pip install --no-deps --target
    baseline/_ref_cuda <reference>``); None when it is not installed."""
    if not list((REF_CUDA_DIR / "maxsim").glob("_maxsim_cuda*.so")):
        return None
    sys.path.insert(0, str(REF_CUDA_DIR))
    import maxsim  # the reference package

    if maxsim._api._maxsim_cuda is None:
        raise RuntimeError("the reference CUDA extension in baseline/_ref_cuda did not load")
    return maxsim


def configs_bench(args, impl="ours"):
    """C0-C4 shapes of the reference's benchmarks (seeded synthetic data with their sizes and distributions),
    timed like the reference's harness: 5 warm-up calls, then 20 timed synchronous calls with host inputs
    and outputs; median and p95 in ms.  ``impl="reference"`` runs the same calls through the reference's
    own package and CUDA extension (built for sm_100a), on the same box; its test-only
    ``streaming_topk_batch`` (a spin lock on a global flag) is never called."""
    if impl == "reference":
        mx = _reference_cuda_package()
        if mx is None:
            print(json.dumps({"configs": "all", "impl": "reference", "unavailable":
                              "reference CUDA extension not installed in baseline/_ref_cuda"}), flush=True)
            return
        from maxsim import cascade as casc, experimental as ex
        from maxsim.sdk import Index, Reranker
    else:
        from maxsim_b200 import cascade as casc, experimental as ex
        from maxsim_b200.sdk import Index, Reranker

    def timed(fn, reps=20, warm=5):
        for _ in range(warm):
            fn()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append(1e3 * (time.perf_counter() - t0))
        ts.sort()
        return ts[len(ts) // 2], ts[int(0.95 * (len(ts) - 1))]

    def emit(cfg, op, p50, p95, note=""):
        ref = REF_4090_MS.get((cfg, op))
        print(json.dumps({"configs": cfg, "impl": impl, "op": op, "p50_ms": round(p50, 4), "p95_ms": round(p95, 4),
                          "reference_rtx4090_p50_ms": ref, "note": note}), flush=True)

    only = set(args.configs_only.split(",")) if args.configs_only else None
    rng = np.random.default_rng(SEED ^ 0x51A7)
    # C0 / C3: 4,096 docs of U[64, 192] tokens, query [4, 32, 128] from 4 target docs
    docs, off, cent = _clustered(rng, 4096, 64, 192)
    q = _queries(rng, cent, 4, 32)
    if only is None or "C0" in only or "C3" in only:
        tok = ex.int4_to_device(ex.pack_int4_symmetric(docs, off, scale_granularity="token")).data
        ten = ex.int4_to_device(ex.pack_int4_symmetric(docs, off, scale_granularity="tensor")).data
        emit("C0", "int4 per-token full scan, fp32 query", *timed(lambda: tok.maxsim_batch(q)))
        emit("C0", "int4 per-token full scan, int8 query", *timed(lambda: tok.maxsim_batch_int8q(q)))
        emit("C0", "int4 per-token top-10, fp32 query", *timed(lambda: tok.topk_batch(q, 10)))
        emit("C0", "int4 per-token top-10, int8 query", *timed(lambda: tok.topk_batch_int8q(q, 10)))
        emit("C0", "int4 tensor-scale top-10, fp32 query", *timed(lambda: ten.topk_batch(q, 10)))
        emit("C0", "int4 tensor-scale top-10, int8 query", *timed(lambda: ten.topk_batch_int8q(q, 10)))
        cand = np.sort(rng.choice(4096, size=512, replace=False)).astype(np.int64)
        emit("C0", "int4 per-token candidates fp32, M=512", *timed(lambda: tok.score_candidates_batch(q, cand)))
        resp = casc.residual_int4_to_device(casc.pack_residual_int4(docs, off))
        res = resp.prefix_data
        emit("C0", "int4 residual fused full scan", *timed(lambda: res.score_residual_batch(q)))
        emit("C0", "int4 residual candidates, M=512", *timed(lambda: res.score_residual_candidates_batch(q, cand)))
        for m in (512, 1024, 2048):
            emit("C3", f"int4-prefix cascade top-10, M={m}",
                 *timed(lambda m=m: casc.cascade_topk(q, resp, 10, candidates=m, device="cuda")))
        if impl == "ours":
            bres = casc.binary_residual_to_device(casc.pack_binary_residual_int4(docs, off))
            for m in (512, 1024, 2048):
                emit("C3", f"binary-prefix cascade top-10, M={m}",
                     *timed(lambda m=m: casc.binary_cascade_topk(q, bres, 10, candidates=m, device="cuda")),
                     note="binary sign prefix + per-token int4 residual (no reference counterpart)")
            del bres
        del tok, ten, res, resp
    del docs
    # C1 / C2: 10,171 docs of U[400, 800] tokens, 256 queries x 20 tokens
    docs, off, cent = _clustered(rng, 10171, 400, 800)
    q256 = _queries(rng, cent, 256, 20)
    ids = [f"d{i}" for i in range(10171)]
    if only is None or "C1" in only:
        rr = Reranker(Index.from_embeddings(ids, docs, off, mode="int4"), device="cuda", int4_query="int8")
        emit("C1", "SDK search, tensor int4 + int8 query, 256 queries one by one",
             *timed(lambda: [rr.search(q256[i], k=10) for i in range(256)], reps=3, warm=1))
        h1 = rr.corpus.int4_packed.data
        emit("C1", "tensor int4 top-10, int8 query, 8 batches of 32",
             *timed(lambda: [h1.topk_batch_int8q(q256[i:i + 32], 10) for i in range(0, 256, 32)], reps=5, warm=2))
        del rr, h1
    if only is None or "C2" in only:
        for mode, label in (("binary", "binary (max_speed)"),
                            ("binary_token_scale", "binary + fp16 token scale (balanced)")):
            rb = Reranker(Index.from_embeddings(ids, docs, off, mode=mode), device="cuda")
            emit("C2", f"SDK search, {label}, 256 queries one by one",
                 *timed(lambda: [rb.search(q256[i], k=10) for i in range(256)], reps=3, warm=1))
            hb = rb.corpus.packed.data
            w = rng.uniform(0.5, 1.5, size=20).astype(np.float32)
            use_ts = mode == "binary_token_scale"
            for red, kw in (("maxsim", {}), ("weighted_maxsim", {"query_weights": w}), ("topk2", {}), ("topk4", {}),
                            ("smoothsim", {"temperature": 0.1})):
                emit("C2", f"{label} full scan, reducer {red}, 256 queries in one batch",
                     *timed(lambda red=red, kw=kw: hb.score_batch(q256, reducer=red, use_token_scale=use_ts, **kw),
                            reps=5, warm=2))
            del rb, hb
    del docs
    if only is None or "C4" in only:
        # C4: the bench corpus (100,000 pages x 1,030 tokens, per-token int4), host arrays into each
        # implementation's handle, one 64-query batch of make_queries, int8 queries, top-10
        import torch

        from maxsim_b200 import _lib  # corpus generation only (the device packer, bit-exact with the reference's)

        dev = torch.device("cuda", 0)
        codes_d, scales_d = build_shard(torch, _lib, 0, NUM_PAGES, dev)
        codes_h, scales_h = codes_d.cpu().numpy(), scales_d.cpu().numpy()
        del codes_d, scales_d
        torch.cuda.empty_cache()
        qd, _ = make_queries(torch, dev)
        q64 = qd[:BATCH].cpu().numpy()
        offs = np.arange(NUM_PAGES + 1, dtype=np.int64) * PAGE_TOKENS
        if impl == "reference":
            h = mx._api._maxsim_cuda.CudaInt4PackedDocs(codes_h, offs, DIM, 1.0)
        else:
            from maxsim_b200 import _maxsim_cuda as mc

            h = mc.CudaInt4PackedDocs(codes_h, offs, DIM, 1.0)
        h.set_token_scale_vector(scales_h)
        del codes_h, scales_h
        emit("C4", "int4 per-token top-10, int8 query, one batch of 64 x 24 (100,000 pages)",
             *timed(lambda: h.topk_batch_int8q(q64, 10), reps=5, warm=2))
        del h


def c2_engines(args):
    """Sign-code scans of the C2 corpus (10,171 documents of U[400, 800] tokens, 20 query tokens) on the
    tensor-core engine and on the AND + popcount engine, batch 1 and 32, int8 and fp32 queries: one timed
    launch each (CUDA events, after one warm-up), one JSON line per case.  Wrapped by ncu for the committed
    engine comparison (profiles/popc_vs_tc_c2.txt)."""
    import torch

    from maxsim_b200 import _lib
    from maxsim_b200 import _maxsim_cuda as mc
    from oracle import reference_cpu as ref  # test infrastructure: the sign packer's restatement

    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(7)
    docs, offs, cent = _clustered(rng, 10171, 400, 800)
    qs = _queries(rng, cent, 32, 20)
    hb = mc.CudaPackedDocs(ref.pack_signs(docs), offs, DIM)
    del docs
    prev = _lib.get_engine()
    for batch in (1, 32):
        qd = torch.from_numpy(np.ascontiguousarray(qs[:batch])).to(dev)
        out = torch.empty((batch, 10171), dtype=torch.float32, device=dev)
        for int8 in (True, False):
            for eng, name in ((2, "tensor core"), (3, "popcount")):
                _lib.set_engine(eng)
                hb.score_batch_device(qd, out, int8_query=int8)
                ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
                ev[0].record()
                hb.score_batch_device(qd, out, int8_query=int8)
                ev[1].record()
                torch.cuda.synchronize()
                print(json.dumps({"c2_engines": name, "batch": batch, "query": "int8" if int8 else "fp32",
                                  "ms": round(ev[0].elapsed_time(ev[1]), 4)}), flush=True)
    _lib.set_engine(prev)


def batch_sweep(args, torch, _lib, handle, queries, device):
    """One line per batch size: scan + top-k of the whole resident corpus, CUDA events on the launching
    stream, against both roofs (algorithmic HBM bytes and int8 tensor ops of that batch)."""
    hbm_peak, bf16_peak, _, peak_kind = _peaks()
    int8_peak = _int8_gemm_tops(torch, device) or 2.0 * bf16_peak
    peak_kind += ", int8: measured cuBLASLt GEMM burst (else 2 x bf16)"
    n_tok = NUM_PAGES * PAGE_TOKENS
    stream = torch.cuda.Stream(device)
    torch.cuda.set_stream(stream)
    for b in (int(x) for x in args.batch_sweep.split(",")):
        nb = queries.shape[0] // b
        qb = queries[:nb * b].view(nb, b, QUERY_TOKENS, DIM)
        out_s = torch.empty((b, TOP_K), dtype=torch.float32, device=device)
        out_i = torch.empty((b, TOP_K), dtype=torch.int64, device=device)
        for i in range(args.warmup):
            handle.topk_batch_device(qb[i % nb], TOP_K, out_s, out_i, int8_query=True, stream=stream.cuda_stream)
        reps = max(3, args.steps)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        torch.cuda.synchronize(device)
        ev[0].record(stream)
        for i in range(reps):
            handle.topk_batch_device(qb[i % nb], TOP_K, out_s, out_i, int8_query=True, stream=stream.cuda_stream)
        ev[1].record(stream)
        torch.cuda.synchronize(device)
        ms = ev[0].elapsed_time(ev[1]) / reps
        algo_bytes = n_tok * (DIM // 2 + 4) + 8 * (NUM_PAGES + 1) + b * QUERY_TOKENS * DIM + b * TOP_K * 12
        algo_ops = 2.0 * b * QUERY_TOKENS * n_tok * DIM
        hbm_ms, tc_ms = 1e3 * algo_bytes / (hbm_peak * 1e9), 1e3 * algo_ops / (int8_peak * 1e12)
        print(json.dumps({"sweep": "batch", "batch": b, "query_rows": b * QUERY_TOKENS, "ms": ms,
                          "queries_per_s": b / (ms * 1e-3), "hbm_gbs": algo_bytes / (ms * 1e-3) / 1e9,
                          "tensor_tops": algo_ops / (ms * 1e-3) / 1e12, "hbm_roof_ms": hbm_ms, "tensor_roof_ms": tc_ms,
                          "bound": "tensor" if tc_ms > hbm_ms else "hbm", "frac_of_roof": max(hbm_ms, tc_ms) / ms,
                          "peaks": f"HBM {hbm_peak} GB/s, int8 {int8_peak} TOP/s ({peak_kind})",
                          "workload": f"C4 corpus ({NUM_PAGES} pages x {PAGE_TOKENS} tokens), int8 queries x "
                                      f"{QUERY_TOKENS} tokens, top-{TOP_K}"}), flush=True)


def _peaks():
    """(HBM GB/s, bf16 TF/s burst, bf16 TF/s sustained, source) from MEASURED_PEAKS.json (else the pool's
    fallback figures).  The file has no int8 figure: ``_int8_gemm_tops`` measures one in the same run."""
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        burst = float(d["bf16_tflops"])
        return float(d["hbm_gbs"]), burst, float(d.get("bf16_tflops_sustained", burst)), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


INT8_GEMM_N = 8192


def _int8_gemm_tops(torch, device, reps=20, warm=5):
    """Measured int8 tensor-core rate of this GPU: a cuBLASLt int8 x int8 -> int32 GEMM
    (``torch._int_mm``, 8192 x 8192 x 8192, B column-major), CUDA events over ``reps`` calls after
    ``warm`` untimed ones (a burst, like the bf16 figure of MEASURED_PEAKS.json).  The denominator of the
    headline kernel's tensor roofline; None if the library call is unavailable."""
    n = INT8_GEMM_N
    g = torch.Generator(device=device)
    g.manual_seed(1)
    try:
        a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=device, generator=g)
        b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=device, generator=g).t()
        for _ in range(warm):
            torch._int_mm(a, b)
        torch.cuda.synchronize(device)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(reps):
            torch._int_mm(a, b)
        t1.record()
        torch.cuda.synchronize(device)
        ms = t0.elapsed_time(t1) / reps
    except (RuntimeError, AttributeError):
        return None
    finally:
        a = b = None
        torch.cuda.empty_cache()
    return 2.0 * n ** 3 / (ms * 1e-3) / 1e12


# ---------------------------------------------------------------------------
# synthetic corpus on the GPU (deterministic per global page chunk)
# ---------------------------------------------------------------------------

def _chunk_centroids(torch, chunk: int, pages: int, device):
    g = torch.Generator(device=device)
    g.manual_seed(SEED * 7919 + 2 * chunk)
    c = torch.randn((pages, DIM), generator=g, device=device, dtype=torch.float32)
    return c / c.norm(dim=1, keepdim=True)


def _chunk_tokens(torch, chunk: int, pages: int, device):
    cent = _chunk_centroids(torch, chunk, pages, device)
    g = torch.Generator(device=device)
    g.manual_seed(SEED * 7919 + 2 * chunk + 1)
    x = cent.repeat_interleave(PAGE_TOKENS, dim=0)
    x.add_(torch.randn(x.shape, generator=g, device=device, dtype=torch.float32), alpha=NOISE)
    x.div_(x.norm(dim=1, keepdim=True))
    return x


def build_shard(torch, lib_mod, page_lo: int, page_hi: int, device):
    """Pack pages [page_lo, page_hi) to per-token int4 on the GPU; returns (codes, scales)."""
    n_tok = (page_hi - page_lo) * PAGE_TOKENS
    codes = torch.empty((n_tok, DIM // 2), dtype=torch.uint8, device=device)
    scales = torch.empty(n_tok, dtype=torch.float32, device=device)
    first, last = page_lo // CHUNK_PAGES, (page_hi - 1) // CHUNK_PAGES
    for chunk in range(first, last + 1):
        c_lo = chunk * CHUNK_PAGES
        pages = min(CHUNK_PAGES, NUM_PAGES - c_lo)
        lo, hi = max(page_lo, c_lo), min(page_hi, c_lo + pages)
        x = _chunk_tokens(torch, chunk, pages, device)[(lo - c_lo) * PAGE_TOKENS:(hi - c_lo) * PAGE_TOKENS]
        x = x.contiguous()
        dst = (lo - page_lo) * PAGE_TOKENS
        lib_mod.check(lib_mod.lib.msb_pack_int4_device(
            ctypes.c_void_p(x.data_ptr()), x.shape[0], DIM, 1, ctypes.c_void_p(codes[dst:].data_ptr()),
            ctypes.c_void_p(scales[dst:].data_ptr()), None,
            ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)))
        del x
    torch.cuda.synchronize(device)
    return codes, scales


def make_queries(torch, device):
    """1,024 x 24 query tokens: a random target page's centroid plus noise, L2-normalised."""
    rng = np.random.default_rng(SEED + 1)
    targets = rng.integers(0, NUM_PAGES, size=NUM_QUERIES)
    g = torch.Generator(device=device)
    g.manual_seed(SEED + 2)
    q = torch.empty((NUM_QUERIES, QUERY_TOKENS, DIM), dtype=torch.float32, device=device)
    cache = {}
    for i, p in enumerate(targets):
        chunk = int(p) // CHUNK_PAGES
        if chunk not in cache:
            cache[chunk] = _chunk_centroids(torch, chunk, min(CHUNK_PAGES, NUM_PAGES - chunk * CHUNK_PAGES), device)
        q[i] = cache[chunk][int(p) - chunk * CHUNK_PAGES]
    q.add_(torch.randn(q.shape, generator=g, device=device, dtype=torch.float32), alpha=NOISE)
    q.div_(q.norm(dim=2, keepdim=True))
    return q, targets


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = [r.split(", ") for r in Path(self.path).read_text().strip().splitlines() if r.strip()]
        os.unlink(self.path)
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[j] for r in rows if len(r) >= 9 for j in range(4) if r[5 + j].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "samples": len(sm), "reasons": reasons}


# ---------------------------------------------------------------------------
# CPU oracle legs (test infrastructure): the CPU baseline and the parity check
# ---------------------------------------------------------------------------

def _oracle_lib():
    import ctypes as C

    _oracle_ready()
    return C.CDLL(str(REPO / "oracle" / "libmaxsim_oracle.so"))


def host_pages(torch, page_ids, device):
    """The corpus pages ``page_ids`` (sorted global ids) as the GPU arm builds them -- the same seeded
    per-chunk tokens, generated on the device -- packed per-token int4 on the host by the oracle's
    restatement of the reference packer (bit-identical to the device packer the GPU arm uses).
    Returns (codes [n * PAGE_TOKENS, 64] u8, token scales [n * PAGE_TOKENS] f32, offsets [n + 1])."""
    from oracle import reference_cpu as ref  # test infrastructure: CPU baseline and parity check only

    page_ids = np.asarray(page_ids, dtype=np.int64)
    codes = np.empty((page_ids.shape[0] * PAGE_TOKENS, DIM // 2), np.uint8)
    scales = np.empty(page_ids.shape[0] * PAGE_TOKENS, np.float32)
    chunks = page_ids // CHUNK_PAGES
    at = 0
    for chunk in np.unique(chunks):
        sel = page_ids[chunks == chunk]
        pages = min(CHUNK_PAGES, NUM_PAGES - int(chunk) * CHUNK_PAGES)
        x = _chunk_tokens(torch, int(chunk), pages, device).view(pages, PAGE_TOKENS, DIM)
        rows = x[torch.as_tensor(sel - int(chunk) * CHUNK_PAGES, device=device)].reshape(-1, DIM).cpu().numpy()
        del x
        data, _, _, ts = ref.pack_int4(rows, "token")
        codes[at:at + rows.shape[0]] = data
        scales[at:at + rows.shape[0]] = ts
        at += rows.shape[0]
    offsets = np.arange(page_ids.shape[0] + 1, dtype=np.int64) * PAGE_TOKENS
    return codes, scales, offsets


def oracle_scores(oracle, queries_host, codes, scales, offsets, targets=None, threads=None):
    """C oracle (restatement of the reference int8-query kernel) scores [B, T] of int8-quantised queries."""
    import ctypes as C

    from oracle import reference_cpu as ref  # test infrastructure

    B = queries_host.shape[0]
    qc, qs = ref.quantize_query_int8(np.ascontiguousarray(queries_host, dtype=np.float32).reshape(-1, DIM))
    D = offsets.shape[0] - 1
    T = D if targets is None else targets.shape[0]
    out = np.empty((B, T), np.float32)
    rc = oracle.oracle_int4_int8q_scores_docs(
        qc.ctypes.data_as(C.c_void_p), qs.ctypes.data_as(C.c_void_p), B, queries_host.shape[1], DIM,
        codes.ctypes.data_as(C.c_void_p), scales.ctypes.data_as(C.c_void_p), C.c_float(1.0),
        offsets.ctypes.data_as(C.c_void_p), C.c_int64(D),
        None if targets is None else targets.ctypes.data_as(C.c_void_p), C.c_int64(T),
        out.ctypes.data_as(C.c_void_p), threads or (os.cpu_count() or 1))
    if rc != 0:
        raise RuntimeError("oracle scoring failed")
    return out


def reference_sample_pages(n):
    """The CPU legs' page sample: n pages spread evenly over the corpus (so over many chunks)."""
    return np.unique(np.linspace(0, NUM_PAGES - 1, n).round().astype(np.int64))


def cpu_rate(torch, device, queries_host_batches, sample_pages, steps, threads):
    """The reference's CPU path timed on the host cores: per step, one 64-query batch (the GPU arm's
    queries, batch i mod 16) scored against `sample_pages` pages of the GPU arm's corpus by the oracle's
    C restatement of the reference int8-query kernel (documents in parallel over `threads` threads),
    extrapolated to the whole corpus by NUM_PAGES / len(sample).  Returns per-step full-corpus seconds."""
    oracle = _oracle_lib()
    pages = reference_sample_pages(sample_pages)
    codes, scales, offsets = host_pages(torch, pages, device)
    per_step = []
    for i in range(steps):
        q = queries_host_batches[i % queries_host_batches.shape[0]]
        t0 = time.perf_counter()
        oracle_scores(oracle, q, codes, scales, offsets, threads=threads)
        per_step.append((time.perf_counter() - t0) * NUM_PAGES / pages.shape[0])
    return per_step, pages.shape[0]


def validate_batch(torch, handle, query_dev, targets, device, sample_pages=64):
    """Parity of one bench batch outside the timed region, against the C oracle:
    (a) each query's returned top-10 pages: scores bit-exact with the oracle's for those pages;
    (b) an evenly spread page sample: the full tensor-core score matrix equals the oracle bit for bit;
    (c) the returned top-10 is the exact (score desc, id asc) top-10 of the full score matrix;
    (d) no sampled page outside a query's top-10 outscores its 10th entry (oracle scores)."""
    oracle = _oracle_lib()
    B = query_dev.shape[0]
    top_s = torch.empty((B, TOP_K), dtype=torch.float32, device=device)
    top_i = torch.empty((B, TOP_K), dtype=torch.int64, device=device)
    full = torch.empty((B, NUM_PAGES), dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device).cuda_stream
    handle.topk_batch_device(query_dev, TOP_K, top_s, top_i, int8_query=True, stream=stream)
    handle.score_batch_device(query_dev, full, int8_query=True, stream=stream)
    torch.cuda.synchronize(device)
    top_s, top_i, full = top_s.cpu().numpy(), top_i.cpu().numpy(), full.cpu().numpy()
    q_host = query_dev.cpu().numpy()
    sample = reference_sample_pages(sample_pages)
    pages = np.unique(np.concatenate([top_i.reshape(-1), sample]))
    codes, scales, offsets = host_pages(torch, pages, device)
    local = {int(p): j for j, p in enumerate(pages)}
    topk_exact = True
    for b in range(B):
        tg = np.array([local[int(p)] for p in top_i[b]], np.int64)
        want = oracle_scores(oracle, q_host[b:b + 1], codes, scales, offsets, targets=tg)[0]
        topk_exact &= bool(np.array_equal(want, top_s[b]))
    tg = np.array([local[int(p)] for p in sample], np.int64)
    want_sample = oracle_scores(oracle, q_host, codes, scales, offsets, targets=tg)
    sample_exact = bool(np.array_equal(want_sample, full[:, sample]))
    order = np.stack([np.lexsort((np.arange(NUM_PAGES), -row))[:TOP_K] for row in full])
    topk_of_full = bool(np.array_equal(order, top_i)) and bool(np.array_equal(np.take_along_axis(full, order, 1), top_s))
    outside_ok = True
    for b in range(B):
        out = ~np.isin(sample, top_i[b])
        outside_ok &= bool(np.all(want_sample[b][out] <= top_s[b, -1]))
    return {"checked": f"batch 0 (64 queries): top-{TOP_K} pages of every query and {sample.shape[0]} evenly spread "
                       f"pages against the C oracle",
            "topk_scores_exact": topk_exact, "sample_scores_exact": sample_exact,
            "topk_is_exact_topk_of_full_scan": topk_of_full, "sample_never_beats_topk": outside_ok,
            "top1_is_query_target_page": float(np.mean(top_i[:, 0] == targets[:B])),
            "ok": bool(topk_exact and sample_exact and topk_of_full and outside_ok)}


def _oracle_ready():
    lib = REPO / "oracle" / "libmaxsim_oracle.so"
    if not lib.exists():
        subprocess.run(["make", "-C", str(REPO / "oracle"), "libmaxsim_oracle.so"], check=True,
                       stdout=subprocess.DEVNULL)


# ---------------------------------------------------------------------------
# main
# ---------------------------------------------------------------------------

def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=16)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-validate", action="store_true",
                    help="skip the after-timing parity check of batch 0 against the C oracle")
    ap.add_argument("--engine", type=int, default=0, help="0 auto, 1 SIMT, 2 tensor core")
    ap.add_argument("--pages", type=int, default=NUM_PAGES,
                    help="corpus pages (default: the C4 workload; smaller values are for profiling captures)")
    ap.add_argument("--configs-impl", choices=["ours", "reference"], default="ours",
                    help="--configs through this library or through the reference's own CUDA build (baseline/_ref_cuda)")
    ap.add_argument("--configs-only", default=None, help="comma-separated subset of C0,C1,C2,C3,C4 for --configs")
    ap.add_argument("--c2-engines", action="store_true",
                    help="time sign-code scans of the C2 corpus on the tensor-core and popcount engines")
    ap.add_argument("--configs", action="store_true",
                    help="time the reference's smaller benchmark shapes (C0-C3) through the handle and SDK calls "
                         "the reference's own benchmarks time, one JSON line per operation, instead of the bench line")
    ap.add_argument("--batch-sweep", default=None,
                    help="comma-separated batch sizes: time the scan + top-k per batch size on the resident corpus "
                         "and print one roofline line per size instead of the bench line (HBM/tensor crossover)")
    args = ap.parse_args()
    globals()["NUM_PAGES"] = args.pages
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    import torch

    if args.impl == "reference":
        run_reference(args, torch, world, rank, local_rank)
        return

    from maxsim_b200 import _lib
    from maxsim_b200 import _maxsim_cuda as mc
    from maxsim_b200.sharded import ShardedReranker, ShardInfo, shard_bounds

    if args.c2_engines:
        if rank == 0:
            torch.cuda.set_device(local_rank)
            c2_engines(args)
        return
    if args.configs:
        if rank == 0:
            torch.cuda.set_device(local_rank)
            configs_bench(args, args.configs_impl)
        return

    _lib.set_engine(args.engine)
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    offsets_all = np.arange(NUM_PAGES + 1, dtype=np.int64) * PAGE_TOKENS
    bounds = shard_bounds(offsets_all, world)
    page_lo, page_hi = int(bounds[rank]), int(bounds[rank + 1])
    codes, scales = build_shard(torch, _lib, page_lo, page_hi, device)
    local_off = np.arange(page_hi - page_lo + 1, dtype=np.int64) * PAGE_TOKENS
    handle = mc.CudaInt4PackedDocs.__new__(mc.CudaInt4PackedDocs)
    handle._h = ctypes.c_void_p()
    handle._dim = DIM
    _lib.check(_lib.lib.msb_docs_create_device(0, DIM, ctypes.c_void_p(codes.data_ptr()), codes.shape[0], None,
                                               local_off.ctypes.data_as(ctypes.c_void_p), page_hi - page_lo,
                                               ctypes.c_float(1.0), ctypes.byref(handle._h)))
    _lib.check(_lib.lib.msb_docs_set_token_scales_device(handle._h, ctypes.c_void_p(scales.data_ptr()),
                                                         scales.shape[0]))
    scales_host = scales.cpu().numpy() if world == 1 else None  # the SDK keeps a host copy, like the reference
    del codes, scales
    torch.cuda.empty_cache()

    queries, targets = make_queries(torch, device)
    n_batches = NUM_QUERIES // BATCH
    queries = queries.view(n_batches, BATCH, QUERY_TOKENS, DIM)  # one step = one [64, 24, 128] batch
    if args.batch_sweep:
        if world == 1:
            batch_sweep(args, torch, _lib, handle, queries.view(-1, QUERY_TOKENS, DIM), device)
        return
    info = ShardInfo(rank=rank, world_size=world, doc_lo=page_lo, doc_hi=page_hi, num_docs_total=NUM_PAGES)
    searcher = ShardedReranker(handle, info, int8_query=True)
    work_stream = torch.cuda.Stream(device)  # every timed launch goes to this stream
    torch.cuda.set_stream(work_stream)
    stream = work_stream

    def step(i):
        return searcher.search_device(queries[i % n_batches], TOP_K)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(device)

    for i in range(args.warmup):
        step(i)
    barrier()

    # device-timed region: per-step events on the launching stream
    launches0 = _lib.launch_count()
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    barrier()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    ev[0].record(stream)
    for i in range(args.steps):
        step(i)
        ev[i + 1].record(stream)
    barrier()
    clocks = sampler.stop()
    launches = _lib.launch_count() - launches0
    total_ms = ev[0].elapsed_time(ev[-1])
    step_ms = [ev[i].elapsed_time(ev[i + 1]) for i in range(args.steps)]
    t = torch.tensor([total_ms], dtype=torch.float64, device=device)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())

    # dominant kernel alone (scan + local top-k of this rank), events on its stream
    kern_ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    loc_s = torch.empty((BATCH, TOP_K), dtype=torch.float32, device=device)
    loc_i = torch.empty((BATCH, TOP_K), dtype=torch.int64, device=device)
    barrier()
    reps = max(3, args.steps)
    kern_ev[0].record(stream)
    for i in range(reps):
        handle.topk_batch_device(queries[i % n_batches], TOP_K, loc_s, loc_i, int8_query=True,
                                 stream=stream.cuda_stream)
    kern_ev[1].record(stream)
    barrier()
    kernel_ms = kern_ev[0].elapsed_time(kern_ev[1]) / reps

    # end-to-end through the public API: pinned host queries in, host results out
    host_q = torch.empty((n_batches, BATCH, QUERY_TOKENS, DIM), dtype=torch.float32).pin_memory()
    host_q.copy_(queries.cpu())
    if world == 1:
        from maxsim_b200.experimental import Int4PackedDocs
        from maxsim_b200.sdk import Corpus, Reranker

        resident = Int4PackedDocs(data=handle, values=None, doc_offsets=offsets_all, dim=DIM, num_docs=NUM_PAGES,
                                  scale=1.0, device="cuda", token_scale=scales_host)
        corpus = Corpus(doc_ids=tuple(f"page-{i}" for i in range(NUM_PAGES)), mode="int4_per_token",
                        int4_packed=resident)
        reranker = Reranker(corpus, device="cuda", int4_query="int8")

        def e2e_call(i):
            return reranker.search(host_q[i % n_batches].numpy(), k=TOP_K)
    else:
        def e2e_call(i):
            return searcher.search(host_q[i % n_batches].numpy(), TOP_K)
    for i in range(args.warmup):
        e2e_call(i)
    barrier()
    t0 = time.perf_counter()
    for i in range(args.steps):
        e2e_call(i)
    barrier()
    e2e_s = time.perf_counter() - t0
    e2e_t = torch.tensor([e2e_s], dtype=torch.float64, device=device)
    if dist is not None:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_s = float(e2e_t.item())

    # parity of the timed path (outside the timed region): batch 0 against the C oracle
    validation = None
    if world == 1 and not args.no_validate:
        validation = validate_batch(torch, handle, queries[0], targets, device)

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        per_step, n_pages = cpu_rate(torch, device, host_q.numpy(), CPU_SAMPLE_PAGES, 3, threads)
        full_s = statistics.median(per_step)
        cpu_baseline = {"value": BATCH / full_s, "unit": "queries/s", "cores": threads, "kind": "port",
                        "sample": f"per step one 64-query batch of this run's queries against {n_pages} evenly spread "
                                  f"pages of this run's corpus (C restatement of the reference int8-query kernel, "
                                  f"{threads} OpenMP threads over documents, {full_s * n_pages / NUM_PAGES:.2f} s per "
                                  f"step), extrapolated x{NUM_PAGES / n_pages:.1f} to the {NUM_PAGES:,} pages; "
                                  f"median of 3 steps"}

    hbm_peak, bf16_peak, bf16_sustained, peak_kind = _peaks()
    int8_measured = _int8_gemm_tops(torch, device)  # after the timed regions
    n_local = (page_hi - page_lo) * PAGE_TOKENS
    algo_bytes = n_local * (DIM // 2 + 4) + 8 * (page_hi - page_lo + 1) + BATCH * QUERY_TOKENS * DIM + BATCH * TOP_K * 12
    algo_ops = 2.0 * BATCH * QUERY_TOKENS * n_local * DIM
    achieved_gbs = algo_bytes / (kernel_ms * 1e-3) / 1e9
    achieved_tops = algo_ops / (kernel_ms * 1e-3) / 1e12
    int8_assumed = 2.0 * bf16_peak
    int8_peak = int8_measured if int8_measured else int8_assumed
    hbm_time = algo_bytes / (hbm_peak * 1e9)
    tc_time = algo_ops / (int8_peak * 1e12)
    bound = "tensor" if tc_time > hbm_time else "hbm"
    if bound == "tensor":
        roof = {"bound": "tensor", "achieved": achieved_tops, "peak": int8_peak, "unit": "TOP/s",
                "frac": achieved_tops / int8_peak,
                "peak_note": (f"measured in this run: cuBLASLt int8 GEMM burst (torch._int_mm, {INT8_GEMM_N}^3, "
                              f"CUDA events)" if int8_measured else
                              f"ASSUMED int8 dense rate = 2 x the {peak_kind} bf16 cuBLAS burst ({bf16_peak} TF/s); "
                              f"the int8 GEMM measurement was unavailable"),
                "frac_vs_2x_bf16_burst": achieved_tops / int8_assumed,
                "frac_vs_2x_bf16_sustained": achieved_tops / (2.0 * bf16_sustained),
                "int8_gemm_measured_tops": int8_measured,
                "bf16_peaks_source": f"{peak_kind} (MEASURED_PEAKS.json: burst {bf16_peak}, sustained "
                                     f"{bf16_sustained} TF/s)"}
    else:
        roof = {"bound": "hbm", "achieved": achieved_gbs, "peak": hbm_peak, "unit": "GB/s",
                "frac": achieved_gbs / hbm_peak, "peak_note": peak_kind}
    roof.update({"traffic": TC_DRAM_BYTES_PER_PAGE * (page_hi - page_lo),
                 "traffic_note": "ncu dram__bytes_read.sum + dram__bytes_write.sum per launch, 2,000-page capture "
                                 "scaled by pages; the kernel reads the resident int8 copy of the codes "
                                 "(128 B/token), so traffic is about 2x the int4 algorithmic bytes",
                 "kernel_ms": kernel_ms, "algorithmic_bytes": algo_bytes,
                 "algorithmic_ops": algo_ops, "hbm_achieved_gbs": achieved_gbs,
                 "hbm_frac": achieved_gbs / hbm_peak, "tensor_achieved_tops": achieved_tops,
                 "roofline_ms": 1e3 * max(hbm_time, tc_time)})

    value = BATCH * args.steps / (total_ms * 1e-3)
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "queries/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": DTYPE,
        "data": DATA,
        "config": bench_config(world),
        "engine": ["auto", "simt", "tensor"][args.engine],
        "step_ms": {"min": min(step_ms), "max": max(step_ms)},
        "gpu_launches": int(launches),
        "e2e": {"value": BATCH * args.steps / e2e_s, "unit": "queries/s",
                "h2d_bytes_per_step": BATCH * QUERY_TOKENS * DIM * 4,
                "d2h_bytes_per_step": BATCH * TOP_K * 12 * (1 if world == 1 else 1),
                "api": "Reranker.search(int4_query='int8')" if world == 1
                else "ShardedReranker.search"},
        "roofline": roof,
        "cpu_baseline": cpu_baseline,
        "validation": validation,
        "clocks": clocks,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    del searcher, handle
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args, torch, world, rank, local_rank):
    """Reference arm: the reference's int8-query scoring on the host cores, over this bench's own inputs.

    The reference has no CPU implementation of the int8-query path (only its CUDA kernel and NumPy test
    helpers), so the timed code is the oracle's C restatement of that kernel
    (``maxsim_int4_int8q_token_scale_dim128_kernel``, cpp/maxsim/cuda_extension.cu:1569-1627): exact
    integer dots, the kernel's fp32 epilogue, documents in parallel over every host core.  Per step it
    scores one 64-query batch of the GPU arm's queries (``make_queries``) against CPU_SAMPLE_PAGES pages
    of the GPU arm's corpus (the same seeded chunks, generated on the device, packed on the host by the
    oracle's restatement of the reference packer) and extrapolates by NUM_PAGES / sample pages to the
    whole corpus; the step time reported is that full-corpus estimate.  Under torchrun only rank 0
    runs.  The GPU is used for input generation only, outside the timed calls.
    """
    if rank != 0:
        return
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    threads = os.cpu_count() or 1
    queries, _ = make_queries(torch, device)
    qh = queries.view(NUM_QUERIES // BATCH, BATCH, QUERY_TOKENS, DIM).cpu().numpy()
    per_step, n_pages = cpu_rate(torch, device, qh, CPU_SAMPLE_PAGES, args.warmup + args.steps, threads)
    timed = per_step[args.warmup:]
    step_s = statistics.mean(timed)
    value = BATCH / step_s
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value, "unit": "queries/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": DTYPE, "data": DATA,
        "config": bench_config(world),
        "cpu_baseline": {"value": value, "unit": "queries/s", "cores": threads, "kind": "port",
                         "sample": f"per step one 64-query batch against {n_pages} of {NUM_PAGES:,} pages "
                                   f"({step_s * n_pages / NUM_PAGES:.2f} s measured per step on {threads} threads), "
                                   f"extrapolated x{NUM_PAGES / n_pages:.1f} to the whole corpus"},
        "extrapolation": {"sample_pages": n_pages, "factor": NUM_PAGES / n_pages,
                          "measured_s_per_step": step_s * n_pages / NUM_PAGES},
        "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def bench_config(world):
    """The workload description both arms print (identical keys and values)."""
    return {"workload": WORKLOAD if NUM_PAGES == 100_000 else f"profiling case: {NUM_PAGES} pages of the C4 distribution",
            "num_docs": NUM_PAGES, "num_tokens": NUM_PAGES * PAGE_TOKENS, "batch": BATCH,
            "query_tokens": QUERY_TOKENS, "k": TOP_K, "queries": f"make_queries: {NUM_QUERIES} x {QUERY_TOKENS}, seed "
                                                                 f"{SEED + 1}/{SEED + 2}",
            "parallelism": f"document shards x{world} + NCCL all-gather merge",
            "l2": f"corpus {NUM_PAGES * PAGE_TOKENS * (DIM // 2 + 4) / 1e9:.2f} GB vs 126 MB L2; no flush between steps",
            "cpu_sample": f"CPU legs: {CPU_SAMPLE_PAGES} evenly spread pages per step, extrapolated "
                          f"x{NUM_PAGES / CPU_SAMPLE_PAGES:.1f}"}


if __name__ == "__main__":
    main()
