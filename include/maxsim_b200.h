/*
 * maxsim_b200 -- C ABI of the B200-native compressed late-interaction scoring
 * library (libmaxsim_b200.so, sm_100a).
 *
 * This is the drop-in boundary for the reference's native extension module
 * `maxsim._maxsim_cuda` (reference: cpp/maxsim/cuda_extension.cu, pybind11
 * bindings at :3416-3513).  The reference binds two resident-handle classes,
 * CudaPackedDocs (binary signs, :1872-2675) and CudaInt4PackedDocs (int4 and
 * residual int4, :2677-3306), plus module functions.  Here one opaque handle
 * type `msb_docs` carries either format; every reference method maps to one
 * entry point below (the mapping is listed per function).  A ctypes binding
 * that reproduces the reference class surface is maxsim_b200/_maxsim_cuda.py.
 *
 * Conventions
 *   - Every function returns an int status (MSB_OK or an MSB_ERR_* code);
 *     msb_last_error() returns the message of the calling thread's last
 *     failure.  MSB_ERR_INVALID_ARGUMENT corresponds to the reference's
 *     std::invalid_argument (Python ValueError), MSB_ERR_CUDA to its
 *     std::runtime_error from check_cuda (Python RuntimeError).
 *   - Handles own all device memory they allocate; inputs are copied, so the
 *     caller keeps nothing alive.  A handle's scratch buffers grow
 *     monotonically and are reused across calls (reference :2350-2360), so a
 *     handle must not be used by two threads at once.
 *   - `*_device` entry points take device pointers (the query, outputs,
 *     candidates and the pointers in msb_score_opts) and enqueue work on
 *     `stream` (a cudaStream_t; NULL is the legacy default stream) without
 *     synchronising.  The other entry points take host pointers and return
 *     after the results are in host memory, like the reference methods.
 *   - No entry point falls back to the CPU.
 */
#ifndef MAXSIM_B200_H_
#define MAXSIM_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MSB_OK 0
#define MSB_ERR_INVALID_ARGUMENT 1
#define MSB_ERR_CUDA 2
#define MSB_ERR_NOT_SUPPORTED 3
#define MSB_ERR_INTERNAL 4

#define MSB_FORMAT_INT4 0   /* [N, dim/2] nibbles, even dim in the low nibble */
#define MSB_FORMAT_BINARY 1 /* [N, dim/8] sign bits, bit i of byte i/8, LSB first */

#define MSB_QUERY_F32 0 /* fp32 query tokens */
#define MSB_QUERY_I8 1  /* fp32 query tokens quantised on device to int8 per row */

#define MSB_REDUCER_MAXSIM 0
#define MSB_REDUCER_WEIGHTED_MAXSIM 1
#define MSB_REDUCER_TOPK2 2
#define MSB_REDUCER_TOPK4 3
#define MSB_REDUCER_SMOOTHSIM 4

typedef struct msb_docs msb_docs;

/* Per-call scoring options.  Zero-initialise and set what you need
 * (temperature must be > 0; 1.0 is the reference default). */
typedef struct msb_score_opts {
  int32_t reducer;            /* MSB_REDUCER_* */
  int32_t query_mode;         /* MSB_QUERY_*; int8 supports MSB_REDUCER_MAXSIM only */
  const float* weights;       /* weighted MaxSim: [weight_rows, query_tokens] */
  int32_t weight_rows;        /* 1 (shared) or batch */
  float temperature;          /* SmoothSim temperature, > 0 */
  int32_t use_residual;       /* handles with a residual stream: fused two-stream residual similarity */
  int32_t use_token_scale;    /* binary handles: apply the resident per-token scales */
  int32_t use_doc_scale;      /* binary handles: apply the resident per-document scales */
  float scale;                /* binary handles: scalar document scale (ignored with doc scales) */
  const float* doc_scale_override; /* binary handles: temporary [num_docs] scales, or NULL */
} msb_score_opts;

typedef struct msb_docs_info {
  int32_t format;
  int32_t dim;
  int64_t num_docs;
  int64_t num_tokens;
  int64_t packed_size;         /* bytes of the primary code array */
  float scale;                 /* int4 tensor scale (1.0 for per-token corpora) */
  float residual_scale;
  int32_t has_token_scale;
  int32_t has_doc_scale;
  int32_t has_residual;
  int32_t device;
  int64_t resident_bytes;      /* codes + offsets + scale vectors + residual stream */
  int64_t workspace_bytes;     /* current scratch capacity */
} msb_docs_info;

/* ---- library ----------------------------------------------------------- */
const char* msb_last_error(void);
int msb_version(void);
/* Kernels launched by this library since load (bench.py reports the delta). */
int64_t msb_launch_count(void);
/* Runtime knobs.  "engine": 0 auto, 1 SIMT only, 2 tensor-core only (errors
 * where unsupported).  "tc_int8_cache": 1 (default) lets the tensor-core engine
 * keep a resident int8 copy of an int4 corpus (128 B per token, built on first
 * use and counted in resident_bytes) and stream operand tiles from it with
 * TMA; 0 expands int4 rows per tile instead.  Sign-code (binary) corpora
 * always keep a +-1 int8 copy when the tensor-core engine scans them (MaxSim,
 * dim 128, scalar document scale), and use the SIMT engine when there is no
 * memory for it.  fp32 queries of up to 32 tokens run on the tensor-core
 * engine as three int8 digit planes of each row's 23-bit fixed-point value
 * (exact integer dots, one rounding), for MaxSim, weighted MaxSim, TopK2 /
 * TopK4 and SmoothSim.  The
 * fused residual stream (use_residual) runs there too, reading a second int8
 * copy of the residual codes (128 B per token, dropped when the residual is
 * replaced or cleared).  Candidate lists that name at least one document in
 * 16 are scored by a full tensor-core scan whose [batch, num_docs] scores
 * (workspace) are then gathered; shorter lists by the same scan over the
 * listed documents only, into the same kind of workspace.  "tc_f16_cache": 1
 * keeps an f16
 * copy instead (256 B per token, per-token-scale corpora) and runs kind::f16
 * MMAs whose fp32 accumulators hold the exact integer dots, so the epilogue
 * converts nothing; 0 (default) because its doubled MMA and operand traffic
 * made it slower.  "tc_row_replicas": 1 (default) copies a pass's query rows
 * (int8, at most 64) over the tensor memory's lane quarters.  "tc_fused_topk":
 * 1 selects the full-scan top-k inside the int8-query scan (bit-identical, 0 by
 * default: measured slower).  Unknown names return MSB_ERR_INVALID_ARGUMENT. */
int msb_set_option(const char* name, int64_t value);
int msb_get_option(const char* name, int64_t* value);

/* ---- resident corpus handles ------------------------------------------ */
/* CudaInt4PackedDocs(packed, offsets, dim, scale)  (reference :2679-2728) and
 * CudaPackedDocs(packed, offsets, dim)             (reference :1874-1918).
 * Host pointers; offsets [num_docs+1] must start at 0, be nondecreasing and
 * end at num_tokens.  `scale` is the int4 tensor scale (ignored for binary). */
int msb_docs_create(int32_t format, int32_t dim, const uint8_t* codes, int64_t num_tokens, const int64_t* offsets,
                    int64_t num_docs, float scale, msb_docs** out);
/* Same from device pointers (copied device to device on the current device). */
int msb_docs_create_device(int32_t format, int32_t dim, const uint8_t* codes, int64_t num_tokens,
                           const int64_t* offsets_device, const int64_t* offsets_host, int64_t num_docs, float scale,
                           msb_docs** out);
int msb_docs_destroy(msb_docs* docs);
int msb_docs_get_info(const msb_docs* docs, msb_docs_info* info);

/* set_token_scale_vector / clear_token_scale_vector (reference :1958-1973, :2749-2775).
 * require_positive=1 rejects values that are not finite and > 0 (int4 rule). */
int msb_docs_set_token_scales(msb_docs* docs, const float* scales, int64_t count, int32_t require_positive);
int msb_docs_set_token_scales_device(msb_docs* docs, const float* scales_device, int64_t count);
int msb_docs_clear_token_scales(msb_docs* docs);
/* set_scale_vector / clear_scale_vector (reference :1943-1956). */
int msb_docs_set_doc_scales(msb_docs* docs, const float* scales, int64_t count);
int msb_docs_clear_doc_scales(msb_docs* docs);
/* set_residual_int4 / clear_residual_int4 (reference :2777-2833).  codes are int4 [num_tokens, dim/2]
 * for both formats.  On a binary handle the residual completes a sign-bit prefix whose per-token
 * reconstruction scale is the handle's token scale vector (scale must be 1); that two-stream format has
 * no counterpart in the reference, whose residual cascade uses an int4 prefix. */
int msb_docs_set_residual(msb_docs* docs, const uint8_t* codes, int64_t num_tokens, float scale,
                          const float* token_scales);
int msb_docs_clear_residual(msb_docs* docs);

/* ---- streaming upload (load-to-GPU path) -------------------------------- */
/* Replaces the host side of Corpus.load + int4_to_device / residual_int4_to_device
 * (reference src/maxsim/sdk.py:331-400, experimental.py:271-305, cuda_extension.cu:2679-2773,
 * 2777-2831): the resident arrays are allocated at their final size and filled chunk by chunk
 * from host memory with asynchronous copies (pinned staging buffers overlap the copies with the
 * caller's decompression of the next chunk); token scales are validated on the device at the end
 * instead of by a host pass over every token.  No whole-corpus host copy is needed.
 *
 * msb_docs_create_for_upload takes the same arguments as msb_docs_create without the codes, plus
 * `flags`: MSB_UPLOAD_TOKEN_SCALES allocates a per-token scale vector, MSB_UPLOAD_RESIDUAL an int4
 * residual stream ([num_tokens, dim/2] codes and [num_tokens] scales).  Until msb_docs_upload_finish
 * succeeds, every scoring call on the handle fails with MSB_ERR_INVALID_ARGUMENT. */
#define MSB_UPLOAD_TOKEN_SCALES 1
#define MSB_UPLOAD_RESIDUAL 2
#define MSB_ARRAY_CODES 0                 /* [num_tokens, bytes per token] */
#define MSB_ARRAY_TOKEN_SCALES 1          /* [num_tokens] fp32 */
#define MSB_ARRAY_RESIDUAL_CODES 2        /* [num_tokens, dim/2] */
#define MSB_ARRAY_RESIDUAL_TOKEN_SCALES 3 /* [num_tokens] fp32 */
int msb_docs_create_for_upload(int32_t format, int32_t dim, int64_t num_tokens, const int64_t* offsets,
                               int64_t num_docs, float scale, int32_t flags, msb_docs** out);
/* Queues a copy of `bytes` host bytes into array `which` at byte offset `offset` on the handle's
 * stream and returns at once with a ticket.  The host buffer must stay unchanged until
 * msb_docs_upload_wait(ticket) returns (it is read asynchronously; pinned memory from
 * msb_pinned_alloc lets the copy overlap host work).  Ranges outside the array are rejected. */
int msb_docs_upload(msb_docs* docs, int32_t which, int64_t offset, const void* host, int64_t bytes,
                    int64_t* ticket);
int msb_docs_upload_wait(msb_docs* docs, int64_t ticket);
/* Waits for every queued copy, checks the arrays on the device (int4 codes hold no nibble 8, the
 * value -8; token scales are finite and > 0, with the messages of msb_docs_set_token_scales /
 * msb_docs_set_residual), records `residual_scale` (ignored without MSB_UPLOAD_RESIDUAL) and opens
 * the handle for scoring. */
int msb_docs_upload_finish(msb_docs* docs, float residual_scale);
/* Page-locked host staging buffers (cudaHostAlloc, portable across devices). */
int msb_pinned_alloc(int64_t bytes, void** out);
int msb_pinned_free(void* ptr);

/* ---- scoring (host buffers, synchronous) -------------------------------
 * maxsim_batch / score_batch / score_candidates_batch / score_residual_batch /
 * score_residual_candidates_batch / maxsim_batch_int8q
 * (reference :1975-2067, :2213-2230, :2835-2955, :2993-3006).
 * query [batch, query_tokens, dim] fp32; candidates NULL for all documents;
 * out [batch, num_candidates or num_docs]. */
int msb_docs_score(msb_docs* docs, const float* query, int32_t batch, int32_t query_tokens,
                   const msb_score_opts* opts, const int64_t* candidates, int64_t num_candidates, float* out);
/* topk_batch / topk_batch_int8q / topk_lut_batch (reference :2069-2109,
 * :2165-2211, :2232-2262, :2957-2991, :3008-3033): full scan then top-k with
 * ties to the lower document id.  out_scores/out_ids [batch, k]. */
int msb_docs_topk(msb_docs* docs, const float* query, int32_t batch, int32_t query_tokens, int32_t k,
                  const msb_score_opts* opts, float* out_scores, int64_t* out_ids);
/* Residual cascade (reference src/maxsim/cascade.py:294-417) entirely on the
 * device: prefix scan, per-row top-M, fused residual rescoring of each row's
 * candidates, final top-k with ties broken by candidate document id.  On a
 * binary handle with a residual stream the prefix is the sign scan scaled by the
 * per-token reconstruction scale. */
int msb_docs_cascade_topk(msb_docs* docs, const float* query, int32_t batch, int32_t query_tokens, int32_t k,
                          int32_t candidates, const msb_score_opts* opts, float* out_scores, int64_t* out_ids);

/* ---- scoring (device buffers, asynchronous on `stream`) --------------- */
int msb_docs_score_device(msb_docs* docs, const float* query, int32_t batch, int32_t query_tokens,
                          const msb_score_opts* opts, const int64_t* candidates, int64_t num_candidates, float* out,
                          void* stream);
int msb_docs_topk_device(msb_docs* docs, const float* query, int32_t batch, int32_t query_tokens, int32_t k,
                         const msb_score_opts* opts, float* out_scores, int64_t* out_ids, void* stream);

/* ---- free functions (device buffers) ----------------------------------- */
/* Row-wise top-k of scores [rows, ld] over the first `count` columns.  With
 * tie_ids ([count] or [rows, count] when tie_batched) the order is (score
 * desc, tie id asc) and out_ids holds tie ids; otherwise out_ids holds column
 * positions.  Used for the multi-GPU merge of per-shard top-k lists. */
int msb_topk_rows_device(const float* scores, int64_t ld, int32_t rows, int64_t count, int32_t k,
                         const int64_t* tie_ids, int32_t tie_batched, float* out_scores, int64_t* out_ids,
                         void* stream);
/* Merge of per-shard top-k lists after one all-gather (multi-GPU search; the
 * reference is single-GPU, so this replaces its host-side
 * `np.lexsort`-style top-k of src/maxsim/_api.py:732-735 over the union of
 * the shards' candidates).  `gathered` holds `world` blocks of
 * 16 * batch * k bytes in rank order: a rank's [batch, k] fp32 scores at byte
 * 0 of its block and its [batch, k] int64 local document ids at byte
 * 8 * batch * k, each row ordered (score desc, id asc); a local id of
 * INT64_MAX pads a shard with fewer than k documents.  Global id = local id +
 * first_doc[rank] ([world] int64, device).  Output [batch, k] in the
 * single-GPU order (score desc, global id asc).  world <= 1024. */
int msb_merge_shard_topk_device(const void* gathered, int32_t world, int32_t batch, int32_t k,
                                const int64_t* first_doc, float* out_scores, int64_t* out_ids, void* stream);
/* Kernel-formula int8 query quantisation (reference :1455-1492):
 * codes [rows, dim] int8, scales [rows] fp32. */
int msb_quantize_query_int8_device(const float* query, int64_t rows, int32_t dim, int8_t* codes, float* scales,
                                   void* stream);
/* Encoders bit-exact with the reference NumPy encoders
 * (src/maxsim/experimental.py:218-268, src/maxsim/_api.py:34-54).
 * per_token=1: token_scales [n] written; per_token=0: *tensor_scale written
 * (this variant synchronises `stream`). */
int msb_pack_int4_device(const float* x, int64_t n, int32_t dim, int32_t per_token, uint8_t* codes,
                         float* token_scales, float* tensor_scale, void* stream);
int msb_pack_signs_device(const float* x, int64_t n, int32_t dim, uint8_t* bits, float* mean_abs, void* stream);

/* ---- allocation-free variant ------------------------------------------- */
/* Bytes of the fixed device scratch used by msb_docs_topk_device_noalloc. */
#define MSB_NOALLOC_SCRATCH_BYTES (16u << 20) /* 16 MiB */
/* Full-scan top-k like msb_docs_topk_device (same arguments, options and
 * results), for callers that cannot call cudaMalloc: code that runs while a
 * framework's caching allocator owns all device memory, code inside a
 * memory-budgeted serving loop, or code that must not add driver allocations
 * (which synchronise the device) on a latency path.  It allocates nothing:
 * its scratch -- the [batch, num_docs] fp32 score matrix plus, for int8
 * queries, the quantised query rows -- lives in one fixed 16 MiB device
 * array inside this library, which every GPU that loads the library holds
 * until the process exits.  Calls whose scratch would exceed
 * MSB_NOALLOC_SCRATCH_BYTES (about batch * num_docs * 4 bytes) fail with
 * MSB_ERR_INVALID_ARGUMENT.  It always runs the CUDA-core scan engine.
 *   - The first call on each device looks up the scratch's device address
 *     (cudaGetSymbolAddress, which may load the library's device code on that
 *     device); make that first call before any stream capture.
 *   - All calls on a device share the one scratch array and it keeps the last
 *     call's contents.  Calls that overlap on the GPU (two streams, or two
 *     host threads) race on it: serialise them.
 * This entry point has no counterpart in the reference. */
int msb_docs_topk_device_noalloc(msb_docs* docs, const float* query, int32_t batch, int32_t query_tokens, int32_t k,
                                 const msb_score_opts* opts, float* out_scores, int64_t* out_ids, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MAXSIM_B200_H_ */
