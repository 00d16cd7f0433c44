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
# DRAM bytes (read + write) of one tc_scan_kernel launch per corpus page, from one ncu capture of a
# 2,000-page case of the same workload (profiles/tc_scan_kernel_2000pages_full.txt: 272.32 MB read +
# 4.56 MB written).  The kernel streams the resident int8 copy of the codes (128 B per token, twice
# the int4 bytes) plus the token scales once per launch and the score matrix grows with the pages,
# so traffic scales with the pages a rank holds.
TC_DRAM_BYTES_PER_PAGE = (272.316416e6 + 4.558080e6) / 2000
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


def configs_bench(args):
    """C0-C3 shapes of the reference's benchmarks (seeded synthetic data with their sizes and distributions),
    timed like the reference's harness: 5 warm-up calls, then 20 timed synchronous calls with host inputs
    and outputs; median and p95 in ms."""
    from maxsim_b200 import _api, cascade as casc, experimental as ex
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
        print(json.dumps({"configs": cfg, "op": op, "p50_ms": round(p50, 4), "p95_ms": round(p95, 4),
                          "reference_rtx4090_p50_ms": ref, "speedup_vs_rtx4090": None if ref is None else round(ref / p50, 2),
                          "note": note}), flush=True)

    rng = np.random.default_rng(SEED ^ 0x51A7)
    # C0 / C3: 4,096 docs of U[64, 192] tokens, query [4, 32, 128] from 4 target docs
    docs, off, cent = _clustered(rng, 4096, 64, 192)
    q = _queries(rng, cent, 4, 32)
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
    res = casc.residual_int4_to_device(casc.pack_residual_int4(docs, off)).prefix_data
    emit("C0", "int4 residual fused full scan", *timed(lambda: res.score_residual_batch(q)))
    emit("C0", "int4 residual candidates, M=512", *timed(lambda: res.score_residual_candidates_batch(q, cand)))
    for m in (512, 1024, 2048):
        emit("C3", f"int4-prefix cascade top-10, M={m}", *timed(lambda m=m: res.cascade_topk_batch(q, 10, m)))
    bres = casc.binary_residual_to_device(casc.pack_binary_residual_int4(docs, off))
    for m in (512, 1024, 2048):
        emit("C3", f"binary-prefix cascade top-10, M={m}",
             *timed(lambda m=m: casc.binary_cascade_topk(q, bres, 10, candidates=m, device="cuda")),
             note="binary sign prefix + per-token int4 residual (no reference counterpart)")
    del docs, tok, ten, res, bres
    # C1 / C2: 10,171 docs of U[400, 800] tokens, 256 queries x 20 tokens
    docs, off, cent = _clustered(rng, 10171, 400, 800)
    q256 = _queries(rng, cent, 256, 20)
    ids = [f"d{i}" for i in range(10171)]
    rr = Reranker(Index.from_embeddings(ids, docs, off, mode="int4"), device="cuda", int4_query="int8")
    emit("C1", "SDK search, tensor int4 + int8 query, 256 queries one by one",
         *timed(lambda: [rr.search(q256[i], k=10) for i in range(256)], reps=3, warm=1))
    h1 = rr.corpus.int4_packed.data
    emit("C1", "tensor int4 top-10, int8 query, 8 batches of 32",
         *timed(lambda: [h1.topk_batch_int8q(q256[i:i + 32], 10) for i in range(0, 256, 32)], reps=5, warm=2))
    del rr, h1
    for mode, label in (("binary", "binary (max_speed)"), ("binary_token_scale", "binary + fp16 token scale (balanced)")):
        rb = Reranker(Index.from_embeddings(ids, docs, off, mode=mode), device="cuda")
        emit("C2", f"SDK search, {label}, 256 queries one by one",
             *timed(lambda: [rb.search(q256[i], k=10) for i in range(256)], reps=3, warm=1))
        hb = rb.corpus.packed.data
        w = rng.uniform(0.5, 1.5, size=20).astype(np.float32)
        use_ts = mode == "binary_token_scale"
        for red, kw in (("maxsim", {}), ("weighted_maxsim", {"query_weights": w}), ("topk2", {}), ("topk4", {}),
                        ("smoothsim", {"temperature": 0.1})):
            emit("C2", f"{label} full scan, reducer {red}, 256 queries in one batch",
                 *timed(lambda red=red, kw=kw: hb.score_batch(q256, reducer=red, use_token_scale=use_ts, **kw), reps=5, warm=2))
        del rb, hb


def batch_sweep(args, torch, _lib, handle, queries, device):
    """One line per batch size: scan + top-k of the whole resident corpus, CUDA events on the launching
    stream, against both roofs (algorithmic HBM bytes and int8 tensor ops of that batch)."""
    hbm_peak, bf16_peak, peak_kind = _peaks()
    int8_peak = 2.0 * bf16_peak
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
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


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
# CPU baselines (oracle port of the reference kernel; test infrastructure)
# ---------------------------------------------------------------------------

def cpu_sample_rate(sample_pages: int, threads: int, queries_host, repeats: int = 1):
    """Seconds per 64-query batch over the full corpus, extrapolated from a page sample.

    The sample pages are generated with NumPy (same shape and distribution as
    the GPU corpus) and packed by the oracle; the timed call is the C
    restatement of the reference int8-query kernel.
    """
    import ctypes as C

    from oracle import reference_cpu as ref  # test infrastructure: CPU baseline only

    oracle = C.CDLL(str(REPO / "oracle" / "libmaxsim_oracle.so"))
    rng = np.random.default_rng(SEED + 3)
    cent = rng.standard_normal((sample_pages, DIM)).astype(np.float32)
    cent /= np.linalg.norm(cent, axis=1, keepdims=True)
    x = np.repeat(cent, PAGE_TOKENS, axis=0) + NOISE * rng.standard_normal((sample_pages * PAGE_TOKENS, DIM)).astype(
        np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    codes_h, _, _, scales_h = ref.pack_int4(x.astype(np.float32), "token")
    offs = (np.arange(sample_pages + 1, dtype=np.int64) * PAGE_TOKENS)
    q = np.ascontiguousarray(queries_host[:BATCH])
    qc, qs = ref.quantize_query_int8(q.reshape(-1, DIM))
    out = np.empty((BATCH, sample_pages), np.float32)
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        oracle.oracle_int4_int8q_scores(
            qc.ctypes.data_as(C.c_void_p), qs.ctypes.data_as(C.c_void_p), BATCH, QUERY_TOKENS, DIM,
            codes_h.ctypes.data_as(C.c_void_p), scales_h.ctypes.data_as(C.c_void_p), C.c_float(1.0),
            offs.ctypes.data_as(C.c_void_p), C.c_int64(sample_pages), None, C.c_int64(0),
            out.ctypes.data_as(C.c_void_p), threads)
        times.append(time.perf_counter() - t0)
    per_page = min(times) / sample_pages
    return per_page * NUM_PAGES, times


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
    ap.add_argument("--engine", type=int, default=0, help="0 auto, 1 SIMT, 2 tensor core")
    ap.add_argument("--pages", type=int, default=NUM_PAGES,
                    help="corpus pages (default: the C4 workload; smaller values are for profiling captures)")
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

    if args.configs:
        if rank == 0:
            torch.cuda.set_device(local_rank)
            configs_bench(args)
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

    queries, _ = make_queries(torch, device)
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

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        _oracle_ready()
        threads = os.cpu_count() or 1
        full_s, times = cpu_sample_rate(16, threads, host_q.view(-1, QUERY_TOKENS, DIM).numpy())
        cpu_baseline = {"value": BATCH / full_s, "unit": "queries/s", "cores": threads, "kind": "port",
                        "sample": f"64 queries x 24 tok vs 16 of 100,000 pages (C oracle restatement of the reference "
                                  f"int8-query kernel, {threads} OpenMP threads, {min(times):.2f} s), extrapolated "
                                  f"linearly to the full corpus"}

    hbm_peak, bf16_peak, peak_kind = _peaks()
    n_local = (page_hi - page_lo) * PAGE_TOKENS
    algo_bytes = n_local * (DIM // 2 + 4) + 8 * (page_hi - page_lo + 1) + BATCH * QUERY_TOKENS * DIM + BATCH * TOP_K * 12
    algo_ops = 2.0 * BATCH * QUERY_TOKENS * n_local * DIM
    achieved_gbs = algo_bytes / (kernel_ms * 1e-3) / 1e9
    achieved_tops = algo_ops / (kernel_ms * 1e-3) / 1e12
    int8_peak = 2.0 * bf16_peak
    hbm_time = algo_bytes / (hbm_peak * 1e9)
    tc_time = algo_ops / (int8_peak * 1e12)
    bound = "tensor" if tc_time > hbm_time else "hbm"
    if bound == "tensor":
        roof = {"bound": "tensor", "achieved": achieved_tops, "peak": int8_peak, "unit": "TOP/s",
                "frac": achieved_tops / int8_peak, "peak_note": f"int8 dense = 2 x bf16 {peak_kind} "
                                                               f"({bf16_peak} TF/s)"}
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
        "metric": "full-scan top-10 queries/s (per-token int4 x int8 query, 100k-page corpus)",
        "value": value,
        "unit": "queries/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8 x int4 (int32 accumulate, fp32 epilogue)",
        "data": "synthetic (seeded per-page centroid + noise, generated and packed on the GPU)",
        "config": {"workload": WORKLOAD if NUM_PAGES == 100_000 else f"profiling case: {NUM_PAGES} pages of the C4 distribution", "num_docs": NUM_PAGES, "num_tokens": NUM_PAGES * PAGE_TOKENS,
                   "batch": BATCH, "query_tokens": QUERY_TOKENS, "k": TOP_K,
                   "parallelism": f"document shards x{world} + NCCL all-gather merge",
                   "l2": f"corpus {NUM_PAGES * PAGE_TOKENS * (DIM // 2 + 4) / 1e9:.2f} GB vs 126 MB L2; no flush between steps",
                   "engine": ["auto", "simt", "tensor"][args.engine],
                   "step_ms_min": min(step_ms), "step_ms_max": max(step_ms)},
        "gpu_launches": int(launches),
        "e2e": {"value": BATCH * args.steps / e2e_s, "unit": "queries/s",
                "h2d_bytes_per_step": BATCH * QUERY_TOKENS * DIM * 4,
                "d2h_bytes_per_step": BATCH * TOP_K * 12 * (1 if world == 1 else 1),
                "api": "Reranker.search(int4_query='int8')" if world == 1
                else "ShardedReranker.search"},
        "roofline": roof,
        "cpu_baseline": cpu_baseline,
        "clocks": clocks,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    del searcher, handle
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args, torch, world, rank, local_rank):
    """Reference arm: CPU restatement of the reference int8-query kernel on all host cores.

    The reference has no CPU implementation of the int8-query path (only its
    CUDA kernel and NumPy test helpers), so the timed code is the oracle's C
    port of that kernel.  Nothing here touches the GPU.
    """
    if rank != 0:
        return
    _oracle_ready()
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(SEED + 4)
    qh = rng.standard_normal((NUM_QUERIES, QUERY_TOKENS, DIM)).astype(np.float32)
    qh /= np.linalg.norm(qh, axis=2, keepdims=True)
    sample = 8
    samples = []
    for i in range(args.warmup + args.steps):
        full_s, _ = cpu_sample_rate(sample, threads, qh[(i % 16) * BATCH:])
        if i >= args.warmup:
            samples.append(full_s)
    step_s = statistics.mean(samples)
    value = BATCH / step_s
    line = {
        "impl": "reference",
        "metric": "full-scan top-10 queries/s (per-token int4 x int8 query, 100k-page corpus)",
        "value": value, "unit": "queries/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8 x int4 (int32 accumulate, fp32 epilogue)", "data": "synthetic (same distribution as ours)",
        "config": {"workload": WORKLOAD, "num_docs": NUM_PAGES, "batch": BATCH, "query_tokens": QUERY_TOKENS,
                   "k": TOP_K},
        "cpu_baseline": {"value": value, "unit": "queries/s", "cores": threads, "kind": "port",
                         "sample": f"per step: 64 queries x 24 tok vs {sample} of 100,000 pages, extrapolated "
                                   "linearly; C restatement of the reference int8-query CUDA kernel "
                                   "(the reference has no CPU implementation of this path)"},
        "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
