// C ABI: resident corpus handles and the entry points declared in
// include/maxsim_b200.h.  Host-side validation reproduces the reference's
// argument errors (cpp/maxsim/cuda_extension.cu:1806-1824, :2690-2707,
// :2958-2966, :3224-3235); scoring routes to the tensor-core engine for
// dim-128 scans it supports and to the SIMT engine otherwise.
#include <atomic>
#include <cmath>
#include <cstring>
#include <initializer_list>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../include/maxsim_b200.h"
#include "common.cuh"

namespace msb {
void launch_simt_scan(const DocsView&, const QueryView&, const ReduceView&, const TargetsView&, bool, float*,
                      cudaStream_t);
void launch_quantize_rows(const float*, int64_t, int, int8_t*, float*, int32_t*, int32_t*, bool, cudaStream_t);
void launch_split_query_digits(const float*, int64_t, int32_t*, float*, const float*, int, int, cudaStream_t);
void launch_topk_rows(const float*, int64_t, int, int64_t, int, const int64_t*, bool, float*, int64_t*, cudaStream_t,
                      void* ws = nullptr, size_t ws_bytes = 0);
size_t topk_rows_workspace_bytes(int rows, int64_t T, int k);
void launch_merge_shard_topk(const void*, int, int, int, const int64_t*, float*, int64_t*, cudaStream_t);
void launch_gather_scores(const float*, int64_t, int, const int64_t*, int64_t, bool, float*, cudaStream_t);
void launch_pack_int4(const float*, int64_t, int, bool, uint8_t*, float*, float*, void*, cudaStream_t);
void launch_pack_signs(const float*, int64_t, int, uint8_t*, float*, cudaStream_t);
void launch_check_positive_finite(const float*, int64_t, unsigned int*, cudaStream_t);
void launch_check_int4_codes(const uint8_t*, int64_t, unsigned int*, cudaStream_t);
void launch_check_scale_range(const float*, int64_t, unsigned int*, cudaStream_t);
bool tc_scan_supported(const DocsView&, const QueryView&, const ReduceView&, const TargetsView&, bool residual);
void launch_tc_scan(const DocsView&, const QueryView&, const ReduceView&, const TargetsView&, float*, void* ws,
                    size_t ws_bytes, cudaStream_t, TopkFuse* fuse);
size_t tc_topk_cand_bytes(const QueryView&, int k);
size_t tc_scan_workspace_bytes(const DocsView&, const QueryView&, const TargetsView&);
size_t tc_candidate_units_bytes(const DocsView&, const QueryView&, const TargetsView&);
void launch_tc_scan_candidates(const DocsView&, const QueryView&, const ReduceView&, const TargetsView&, float* scores,
                               void* ws, void* units, size_t units_bytes, cudaStream_t);
bool tc_int8_cache_supported(const DocsView&);
bool popc_scan_supported(const DocsView&, const QueryView&, const ReduceView&, const TargetsView&, bool residual);
size_t popc_scan_workspace_bytes(const QueryView&);
void launch_popc_scan(const DocsView&, const QueryView&, const ReduceView&, const TargetsView&, float*, void* ws,
                      size_t ws_bytes, cudaStream_t);
void launch_expand_codes8(const uint8_t* codes, int64_t num_tokens, uint8_t* out, cudaStream_t);
void launch_expand_binary8(const uint8_t* codes, int64_t num_tokens, uint8_t* out, cudaStream_t);
void launch_expand_codes16(const uint8_t* codes, int64_t num_tokens, uint16_t* out, cudaStream_t);
void set_tc_row_replicas(int on);
int get_tc_row_replicas();

static std::atomic<int64_t> g_launches{0};
void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
static std::atomic<int> g_engine{0};  // 0 auto, 1 SIMT, 2 tensor core, 3 popcount (sign codes)
static std::atomic<int> g_tc_int8_cache{1};  // keep an int8-expanded copy of int4 corpora for the tc engine
static std::atomic<int> g_tc_f16_cache{0};   // keep an f16 copy instead (per-token scales): no conversion in the
                                             // epilogue, but twice the MMAs and operand bytes; measured slower
// Full-scan top-k selected inside the tensor-core scan (per-CTA lists + a merge kernel).  Off by default:
// bit-identical to the unfused path, but measured slower (the list insertions serialise the epilogue's
// document flush, and the unfused selection of a [B, D] score matrix costs well under 1 % of a scan).
static std::atomic<int> g_tc_fused_topk{0};
static std::atomic<uint64_t> g_corpus_serial{0};
}  // namespace msb

using namespace msb;

static thread_local std::string g_last_error;

namespace {

// Extra bytes after offsets and token scales: the tensor-core engine copies
// 16-byte-aligned supersets of these arrays with the bulk-copy engine.
constexpr size_t kTailPad = 64;

struct DeviceBuf {
  void* ptr = nullptr;
  size_t cap = 0;
  void ensure(size_t bytes, const char* what) {
    if (bytes <= cap) return;
    void* next = nullptr;
    check(cudaMalloc(&next, bytes), what);
    if (ptr) cudaFree(ptr);
    ptr = next;
    cap = bytes;
  }
  void release() {
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    cap = 0;
  }
  template <class T>
  T* as() const { return static_cast<T*>(ptr); }
};

// Page-locked host memory (cudaMallocHost), grown on demand.
struct PinnedBuf {
  void* ptr = nullptr;
  size_t cap = 0;
  void ensure(size_t bytes, const char* what) {
    if (bytes <= cap) return;
    void* next = nullptr;
    check(cudaMallocHost(&next, bytes), what);
    if (ptr) cudaFreeHost(ptr);
    ptr = next;
    cap = bytes;
  }
  void release() {
    if (ptr) cudaFreeHost(ptr);
    ptr = nullptr;
    cap = 0;
  }
};

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

template <class F>
int guarded(F&& f) {
  try {
    f();
    return MSB_OK;
  } catch (const InvalidArgument& e) {
    g_last_error = e.what();
    return MSB_ERR_INVALID_ARGUMENT;
  } catch (const NotSupported& e) {
    g_last_error = e.what();
    return MSB_ERR_NOT_SUPPORTED;
  } catch (const CudaFailure& e) {
    g_last_error = e.what();
    return MSB_ERR_CUDA;
  } catch (const std::bad_alloc&) {
    g_last_error = "host allocation failed";
    return MSB_ERR_INTERNAL;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return MSB_ERR_INTERNAL;
  }
}

void validate_offsets(const int64_t* off, int64_t num_docs, int64_t num_tokens) {
  if (num_docs < 0) throw InvalidArgument("offsets must contain at least [0, num_doc_tokens]");
  if (off[0] != 0) throw InvalidArgument("offsets must start at 0");
  if (off[num_docs] != num_tokens) throw InvalidArgument("offsets must end at num_doc_tokens");
  for (int64_t i = 1; i <= num_docs; ++i)
    if (off[i] < off[i - 1]) throw InvalidArgument("offsets must be monotonically nondecreasing");
}

}  // namespace

struct msb_docs {
  int format = 0;
  int dim = 0;
  int device = 0;
  int64_t num_docs = 0;
  int64_t num_tokens = 0;
  float scale = 1.0F;
  float residual_scale = 1.0F;
  bool has_token_scale = false;
  // Whether every finite token scale is below 2^104 in magnitude (the tensor-core scan's biased
  // accumulators stage s * 2^23): -1 until checked, on first use after the token scales change.
  int token_scale_small = -1;
  bool has_doc_scale = false;
  bool has_residual = false;
  cudaStream_t stream = nullptr;
  DeviceBuf codes, offsets, token_scale, doc_scale, residual_codes, residual_token_scale;
  // Workspace (grows monotonically, reused across calls).
  DeviceBuf w_query, w_qcodes, w_qwords, w_qscale, w_qsum, w_scores, w_cands, w_weights, w_top_s, w_top_i,
      w_override, w_fine, w_tc, w_popc,
      w_full,    // full-scan scores that candidate lists are gathered from
      w_units,   // work units of a candidate-list tensor-core scan
      w_select;  // per-chunk lists of a two-stage top-k over few long rows
  std::vector<int64_t> host_offsets;
  bool tc_used = false;  // the tensor-core engine ran since the last error check
  uint64_t serial = 0;   // unique corpus id for caches keyed on a corpus
  // int4 codes expanded once to int8 in the tensor-core scan's K order ([N, 128] bytes), so the scan
  // streams ready operand tiles with tiled TMA instead of expanding every tile for every query batch.
  DeviceBuf codes8;
  bool codes8_failed = false;  // allocation failed once: keep using the expanding scan
  // The same values as f16 ([N, 128], 256 B per token): tensor-core f16 operands whose fp32 accumulators
  // hold the exact integer dot, so the epilogue converts nothing.
  DeviceBuf codes16;
  bool codes16_failed = false;
  // The residual stream's int4 codes expanded like codes8, for the tensor-core residual scan; released
  // whenever the residual stream is replaced or cleared.
  DeviceBuf codes2_8;
  bool codes2_8_failed = false;
  // Streaming upload (msb_docs_create_for_upload .. msb_docs_upload_finish): scoring is refused while
  // open; each queued copy records an event in a small ring that its ticket names.
  static constexpr int kUploadEvents = 16;
  bool upload_open = false;
  int32_t upload_flags = 0;
  int64_t upload_serial = 0;
  cudaEvent_t upload_events[kUploadEvents] = {};
  DeviceBuf w_check;
  // Fused top-k: candidate blocks, and the corpus's first empty documents (score 0, never in a tile),
  // found once from the host offsets.
  DeviceBuf w_topk, empty_ids;
  int n_empty = -1;
  // Page-locked staging of the host-buffer entry points: the query in, the results and the tensor-core
  // error word out, so that a call makes one asynchronous copy each way and synchronises once.
  PinnedBuf pin_in, pin_out;

  size_t bytes_per_token() const { return format == kFormatInt4 ? dim / 2 : dim / 8; }
  int64_t resident_bytes() const {
    return static_cast<int64_t>(codes.cap + codes8.cap + codes16.cap + codes2_8.cap + offsets.cap + token_scale.cap +
                                doc_scale.cap + residual_codes.cap + residual_token_scale.cap);
  }
  int64_t workspace_bytes() const {
    return static_cast<int64_t>(w_query.cap + w_qcodes.cap + w_qwords.cap + w_qscale.cap + w_qsum.cap +
                                w_scores.cap + w_cands.cap + w_weights.cap + w_top_s.cap + w_top_i.cap +
                                w_override.cap + w_fine.cap + w_tc.cap + w_check.cap + w_full.cap +
                                w_popc.cap + w_topk.cap + w_units.cap + w_select.cap);
  }
  ~msb_docs() {
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    DeviceBuf* all[] = {&codes,   &offsets,  &token_scale, &doc_scale, &residual_codes, &residual_token_scale,
                        &w_query, &w_qcodes, &w_qwords,    &w_qscale,  &w_qsum,         &w_scores,
                        &w_cands, &w_weights, &w_top_s,    &w_top_i,   &w_override,     &w_fine,
                        &w_tc,    &codes8,   &codes16,   &w_check,        &codes2_8,  &w_full, &w_popc, &w_topk, &empty_ids,
                        &w_units, &w_select};
    for (DeviceBuf* b : all) b->release();
    pin_in.release();
    pin_out.release();
    for (cudaEvent_t& e : upload_events)
      if (e) cudaEventDestroy(e);
    if (stream) cudaStreamDestroy(stream);
    if (prev >= 0) cudaSetDevice(prev);
  }
};

namespace {

// Device entry points run on the caller's stream as given (NULL = the legacy default stream).
cudaStream_t pick_stream(msb_docs*, void* s) { return static_cast<cudaStream_t>(s); }

struct Resolved {
  DocsView docs;
  ReduceView red;
  bool residual;
  int mode;
};

// Validate options against the handle; weights/override are device pointers.
Resolved resolve(msb_docs* h, const msb_score_opts* o, int batch, int qtok, const float* d_weights,
                 const float* d_override) {
  if (!o) throw InvalidArgument("options must not be NULL");
  if (o->reducer < kMaxSim || o->reducer > kSmooth)
    throw InvalidArgument("reducer must be one of 'maxsim', 'weighted_maxsim', 'topk2', 'topk4', or 'smoothsim'");
  if (!(o->temperature > 0.0F) || !std::isfinite(o->temperature))
    throw InvalidArgument("temperature must be finite and > 0");
  if (o->reducer == kWeighted) {
    if (!o->weights) throw InvalidArgument("query_weights are required for reducer='weighted_maxsim'");
    if (o->weight_rows != 1 && o->weight_rows != batch)
      throw InvalidArgument("query_weights must have shape [query_tokens] or [batch, query_tokens]");
  } else if (o->weights) {
    throw InvalidArgument("query_weights are only valid for reducer='weighted_maxsim'");
  }
  if (o->query_mode != kQueryF32 && o->query_mode != kQueryI8) throw InvalidArgument("unknown query mode");
  if (o->query_mode == kQueryI8 && o->reducer != kMaxSim)
    throw InvalidArgument("int8 queries support reducer='maxsim' only");
  Resolved r{};
  DocsView& d = r.docs;
  d.codes = h->codes.as<uint8_t>();
  d.offsets = h->offsets.as<int64_t>();
  d.host_offsets = h->host_offsets.data();
  d.corpus_id = h->serial;
  d.num_docs = h->num_docs;
  d.num_tokens = h->num_tokens;
  d.dim = h->dim;
  d.format = h->format;
  r.residual = o->use_residual != 0;
  if (h->format == kFormatInt4) {
    d.token_scale = h->has_token_scale ? h->token_scale.as<float>() : nullptr;
    d.scale = h->scale;
    if (r.residual) {
      if (!h->has_residual)
        throw InvalidArgument("residual int4 data was requested but is not loaded on this CUDA handle");
      if (o->query_mode != kQueryF32) throw InvalidArgument("residual scoring takes fp32 queries");
      d.codes2 = h->residual_codes.as<uint8_t>();
      d.token_scale2 = h->residual_token_scale.as<float>();
      d.scale2 = h->residual_scale;
    }
  } else if (r.residual) {
    // sign-bit prefix scaled by its per-token reconstruction scale + per-token int4 residual
    if (!h->has_residual)
      throw InvalidArgument("residual int4 data was requested but is not loaded on this CUDA handle");
    if (!h->has_token_scale)
      throw InvalidArgument("residual scoring on a binary handle needs the prefix token scale vector");
    if (o->query_mode != kQueryF32) throw InvalidArgument("residual scoring takes fp32 queries");
    if (o->use_doc_scale || d_override)
      throw InvalidArgument("document scales do not apply to residual scoring");
    d.token_scale = h->token_scale.as<float>();
    d.codes2 = h->residual_codes.as<uint8_t>();
    d.token_scale2 = h->residual_token_scale.as<float>();
    d.scale2 = h->residual_scale;
    d.scale = 1.0F;
  } else {
    if (o->use_token_scale) {
      if (!h->has_token_scale)
        throw InvalidArgument("token scale vector was requested but is not loaded on this CUDA handle");
      d.token_scale = h->token_scale.as<float>();
    }
    if (d_override) {
      if (o->use_doc_scale) throw InvalidArgument("scale_vector_override and use_scale_vector cannot both be set");
      d.doc_scale = d_override;
    } else if (o->use_doc_scale) {
      if (!h->has_doc_scale)
        throw InvalidArgument("scale vector was requested but is not loaded on this CUDA handle");
      d.doc_scale = h->doc_scale.as<float>();
    }
    d.scale = o->scale;
  }
  r.red.reducer = o->reducer;
  r.red.weights = d_weights;
  r.red.weights_batched = (o->reducer == kWeighted && o->weight_rows == batch && batch > 1) ? 1 : 0;
  r.red.temperature = o->temperature;
  r.mode = o->query_mode;
  (void)qtok;
  return r;
}

void run_scan(msb_docs* h, const Resolved& r, const float* d_query, int batch, int qtok, const TargetsView& tg,
              float* d_out, cudaStream_t stream, TopkFuse* fuse = nullptr);

// Candidate lists (shared or per row) that name at least one document in 16 are scored faster by a full
// tensor-core scan whose scores are then gathered: per (document, query) that scan costs a few percent
// of the SIMT rescoring of a candidate.  Returns false (nothing done) when the list is shorter, the SIMT
// engine is forced, or the tensor-core engine does not support the full scan.  (If a binary corpus or
// the residual stream cannot get its int8 copy, the full scan runs on the SIMT engine: correct, slower.)
// A [batch, num_docs] score scratch (w_full) for a candidate-list scan; false when the device has no
// memory for it (the lists are then rescored on the SIMT engine).
bool candidate_scratch(msb_docs* h, int batch) {
  const size_t bytes = sizeof(float) * static_cast<size_t>(batch) * h->num_docs;
  if (bytes <= h->w_full.cap) return true;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  h->w_full.release();
  h->w_full.ptr = p;
  h->w_full.cap = bytes;
  return true;
}

bool scan_targets_via_full_scan(msb_docs* h, const Resolved& r, const float* d_query, int batch, int qtok,
                                const TargetsView& tg, float* d_out, cudaStream_t stream) {
  if (!tg.ids || g_engine.load() == 1 || tg.count * 16 < h->num_docs || batch <= 0 || qtok <= 0) return false;
  QueryView qv{};
  qv.f32 = d_query;
  qv.batch = batch;
  qv.qtok = qtok;
  qv.mode = r.mode;
  if (!tc_scan_supported(r.docs, qv, r.red, TargetsView{}, r.residual)) return false;
  // no room for the full score matrix: rescore the list instead (the shorter output of the SIMT engine)
  if (!candidate_scratch(h, batch)) return false;
  run_scan(h, r, d_query, batch, qtok, TargetsView{}, h->w_full.as<float>(), stream);
  launch_gather_scores(h->w_full.as<float>(), h->num_docs, batch, tg.ids, tg.count, tg.per_row != 0, d_out, stream);
  return true;
}

// Whether the handle's token scales are all below 2^104 in magnitude (non-finite values aside): a
// device check, run once after the scales change.
int token_scales_small(msb_docs* h, const float* d_scales, cudaStream_t stream) {
  if (h->token_scale_small < 0) {
    h->w_check.ensure(8 * sizeof(unsigned int), "cudaMalloc scale range flag");
    unsigned int* flag = static_cast<unsigned int*>(h->w_check.ptr) + 4;
    check(cudaMemsetAsync(flag, 0, sizeof(unsigned int), stream), "clear scale range flag");
    launch_check_scale_range(d_scales, h->num_tokens, flag, stream);
    unsigned int big = 0;
    check(cudaMemcpyAsync(&big, flag, sizeof(big), cudaMemcpyDeviceToHost, stream), "read scale range flag");
    check(cudaStreamSynchronize(stream), "synchronize scale range check");
    h->token_scale_small = big == 0 ? 1 : 0;
  }
  return h->token_scale_small;
}

// Run one scan into d_out [B, T].  d_query is a device pointer.  With `fuse`, a tensor-core full scan may
// select the top-k itself (fuse->done); otherwise the scores land in d_out.
void run_scan(msb_docs* h, const Resolved& r, const float* d_query, int batch, int qtok, const TargetsView& tg,
              float* d_out, cudaStream_t stream, TopkFuse* fuse) {
  const int64_t T = tg.ids ? tg.count : h->num_docs;
  if (batch == 0 || T == 0) return;
  if (qtok == 0) {
    check(cudaMemsetAsync(d_out, 0, sizeof(float) * static_cast<size_t>(batch) * T, stream), "zero scores");
    return;
  }
  if (scan_targets_via_full_scan(h, r, d_query, batch, qtok, tg, d_out, stream)) return;
  QueryView qv{};
  qv.f32 = d_query;
  qv.batch = batch;
  qv.qtok = qtok;
  qv.mode = r.mode;
  // (the popcount engine scans sign codes; a residual stream, as in a cascade's rescoring, takes the
  // automatic route)
  const int engine = g_engine.load() == 3 && r.residual ? 0 : g_engine.load();
  if (engine == 3) {
    // AND + popcount over the sign codes (forced; see popc_scan.cu)
    if (!popc_scan_supported(r.docs, qv, r.red, tg, r.residual))
      throw NotSupported("the popcount engine does not support this scan");
    const int64_t rows = static_cast<int64_t>(batch) * qtok;
    if (r.mode == kQueryI8) {
      h->w_qcodes.ensure(static_cast<size_t>(rows) * h->dim, "cudaMalloc int8 query codes");
      h->w_qwords.ensure(static_cast<size_t>(rows) * h->dim, "cudaMalloc int8 query words");
      h->w_qscale.ensure(static_cast<size_t>(rows) * sizeof(float), "cudaMalloc int8 query scales");
      h->w_qsum.ensure(static_cast<size_t>(rows) * sizeof(int32_t), "cudaMalloc int8 query sums");
      launch_quantize_rows(d_query, rows, h->dim, h->w_qcodes.as<int8_t>(), h->w_qscale.as<float>(),
                           h->w_qsum.as<int32_t>(), h->w_qwords.as<int32_t>(), false, stream);
      qv.i8 = h->w_qcodes.as<int8_t>();
      qv.row_scale = h->w_qscale.as<float>();
    }
    const size_t ws = popc_scan_workspace_bytes(qv);
    h->w_popc.ensure(ws, "cudaMalloc popcount scan workspace");
    launch_popc_scan(r.docs, qv, r.red, tg, d_out, h->w_popc.ptr, h->w_popc.cap, stream);
    return;
  }
  const bool tc_ok = tc_scan_supported(r.docs, qv, r.red, tg, r.residual);
  if (engine == 2 && !tc_ok) throw NotSupported("the tensor-core engine does not support this scan");
  bool use_tc = tc_ok && engine != 1;
  DocsView dv = r.docs;
  if (use_tc) {
    // Resident operand copies for the tensor-core engine, made once per handle: an f16 copy (option), or
    // the int8 copy (int4 expanded, or +-1 for sign codes).  int4 corpora fall back to expanding per
    // tile when there is no memory for a copy; binary corpora fall back to the SIMT engine.
    const bool binary = h->format == kFormatBinary;
    // TopK and SmoothSim kernels read the int8 copy
    const bool topk = r.red.reducer == kTopK2 || r.red.reducer == kTopK4 || r.red.reducer == kSmooth;
    if (!binary && !r.residual && !topk && g_tc_f16_cache.load() && !h->codes16_failed && dv.token_scale &&
        tc_int8_cache_supported(dv)) {
      if (!h->codes16.ptr) {
        const size_t bytes = static_cast<size_t>(h->num_tokens) * 256;
        void* p = nullptr;
        if (cudaMalloc(&p, bytes) != cudaSuccess) {
          (void)cudaGetLastError();  // not enough memory for the f16 copy: use the int8 copy
          h->codes16_failed = true;
        } else {
          h->codes16.ptr = p;
          h->codes16.cap = bytes;
          launch_expand_codes16(h->codes.as<uint8_t>(), h->num_tokens, static_cast<uint16_t*>(h->codes16.ptr),
                                stream);
        }
      }
      if (h->codes16.ptr) dv.codes16 = static_cast<const uint16_t*>(h->codes16.ptr);
    }
    if (!dv.codes16 && (binary || r.residual || topk || g_tc_int8_cache.load()) && !h->codes8_failed &&
        tc_int8_cache_supported(dv)) {
      if (!h->codes8.ptr) {
        const size_t bytes = static_cast<size_t>(h->num_tokens) * 128;
        void* p = nullptr;
        if (cudaMalloc(&p, bytes) != cudaSuccess) {
          (void)cudaGetLastError();  // not enough memory for the copy
          h->codes8_failed = true;
        } else {
          h->codes8.ptr = p;
          h->codes8.cap = bytes;
          if (binary) launch_expand_binary8(h->codes.as<uint8_t>(), h->num_tokens, h->codes8.as<uint8_t>(), stream);
          else launch_expand_codes8(h->codes.as<uint8_t>(), h->num_tokens, h->codes8.as<uint8_t>(), stream);
        }
      }
      if (h->codes8.ptr) dv.codes8 = h->codes8.as<uint8_t>();
    }
    if ((binary || topk) && !dv.codes8) {
      if (engine == 2) throw NotSupported("no device memory for the tensor-core engine's int8 copy of the codes");
      use_tc = false;
    }
    if (r.residual) {
      // the fused residual stream reads int8 copies of both streams; without them, the SIMT engine
      if (dv.codes8 && !h->codes2_8.ptr && !h->codes2_8_failed) {
        const size_t bytes = static_cast<size_t>(h->num_tokens) * 128;
        void* p = nullptr;
        if (cudaMalloc(&p, bytes) != cudaSuccess) {
          (void)cudaGetLastError();
          h->codes2_8_failed = true;
        } else {
          h->codes2_8.ptr = p;
          h->codes2_8.cap = bytes;
          launch_expand_codes8(h->residual_codes.as<uint8_t>(), h->num_tokens, h->codes2_8.as<uint8_t>(), stream);
        }
      }
      if (h->codes2_8.ptr) dv.codes2_8 = h->codes2_8.as<uint8_t>();
      if (!dv.codes8 || !dv.codes2_8) {
        if (engine == 2) throw NotSupported("no device memory for the tensor-core engine's int8 copies of the streams");
        use_tc = false;
      }
    }
  }
  if (use_tc && tg.ids && !candidate_scratch(h, batch)) {
    // candidate lists score into a [B, D] scratch; without memory for it, the SIMT engine
    if (engine == 2) throw NotSupported("no device memory for the tensor-core candidate scan's score matrix");
    use_tc = false;
  }
  if (use_tc && dv.token_scale) dv.token_scale_small = token_scales_small(h, dv.token_scale, stream);
  const int64_t rows = static_cast<int64_t>(batch) * qtok;
  if (r.mode == kQueryI8) {
    h->w_qcodes.ensure(static_cast<size_t>(rows) * h->dim, "cudaMalloc int8 query codes");
    h->w_qwords.ensure(static_cast<size_t>(rows) * h->dim, "cudaMalloc int8 query words");
    h->w_qscale.ensure(static_cast<size_t>(rows) * sizeof(float), "cudaMalloc int8 query scales");
    h->w_qsum.ensure(static_cast<size_t>(rows) * sizeof(int32_t), "cudaMalloc int8 query sums");
    // words in the order the chosen dot reads: nibble order for int4 codes and for the tensor-core
    // engine's int8 copies, natural order for the SIMT sign-code dot
    launch_quantize_rows(d_query, rows, h->dim, h->w_qcodes.as<int8_t>(), h->w_qscale.as<float>(),
                         h->w_qsum.as<int32_t>(), h->w_qwords.as<int32_t>(), h->format == kFormatInt4 || use_tc,
                         stream);
    qv.i8 = h->w_qcodes.as<int8_t>();
    qv.i8_words = h->w_qwords.as<int32_t>();
    qv.row_scale = h->w_qscale.as<float>();
    qv.row_sum = h->w_qsum.as<int32_t>();
  }
  if (use_tc) {
    if (r.mode == kQueryF32) {
      // fp32 queries: three int8 digit planes and a power-of-two scale per row
      h->w_qwords.ensure(static_cast<size_t>(rows) * 3 * h->dim, "cudaMalloc query digit planes");
      h->w_qscale.ensure(static_cast<size_t>(rows) * sizeof(float), "cudaMalloc query digit scales");
      const bool weighted = r.red.reducer == kWeighted;
      launch_split_query_digits(d_query, rows, h->w_qwords.as<int32_t>(), h->w_qscale.as<float>(),
                                weighted ? r.red.weights : nullptr, qtok, weighted ? r.red.weights_batched : 0,
                                stream);
      qv.i8_words = h->w_qwords.as<int32_t>();
      qv.row_scale = h->w_qscale.as<float>();
    }
    const size_t ws = tc_scan_workspace_bytes(dv, qv, TargetsView{});
    h->w_tc.ensure(ws > 0 ? ws : 16, "cudaMalloc tensor-core scan workspace");
    if (tg.ids) {
      // Candidate lists shorter than a sixteenth of the corpus: each listed document is a work unit of
      // the same scan, scored into the [B, D] scratch at its position and gathered
      h->w_units.ensure(tc_candidate_units_bytes(dv, qv, tg), "cudaMalloc candidate work units");
      launch_tc_scan_candidates(dv, qv, r.red, tg, h->w_full.as<float>(), h->w_tc.ptr, h->w_units.ptr,
                                h->w_units.cap, stream);
      launch_gather_scores(h->w_full.as<float>(), h->num_docs, batch, tg.ids, tg.count, tg.per_row != 0, d_out,
                           stream);
    } else {
      launch_tc_scan(dv, qv, r.red, tg, d_out, h->w_tc.ptr, h->w_tc.cap, stream, fuse);
    }
    h->tc_used = true;
    return;
  }
  launch_simt_scan(r.docs, qv, r.red, tg, r.residual, d_out, stream);
}

// Top-k of `rows` full score rows with the handle's selection workspace (a few long rows are selected in
// chunks by several blocks each, then merged).
void topk_full_rows(msb_docs* h, const float* scores, int rows, int k, float* out_s, int64_t* out_id, cudaStream_t s) {
  const size_t ws = topk_rows_workspace_bytes(rows, h->num_docs, k);
  if (ws) h->w_select.ensure(ws, "cudaMalloc top-k selection workspace");
  launch_topk_rows(scores, h->num_docs, rows, h->num_docs, k, nullptr, false, out_s, out_id, s, ws ? h->w_select.ptr : nullptr,
                   ws ? h->w_select.cap : 0);
}

// Fused top-k set-up for a full-scan top-k (k <= 4096): candidate workspace and the empty-document list.
bool prepare_fused_topk(msb_docs* h, int batch, int k, float* out_s, int64_t* out_i, TopkFuse* f) {
  if (!g_tc_fused_topk.load() || k > 4096 || batch <= 0) return false;
  if (h->n_empty < 0) {
    std::vector<int64_t> ids;
    for (int64_t d = 0; d < h->num_docs && ids.size() < 4096; ++d)
      if (h->host_offsets[d + 1] == h->host_offsets[d]) ids.push_back(d);
    if (!ids.empty()) {
      h->empty_ids.ensure(sizeof(int64_t) * ids.size(), "cudaMalloc empty document list");
      check(cudaMemcpy(h->empty_ids.ptr, ids.data(), sizeof(int64_t) * ids.size(), cudaMemcpyHostToDevice),
            "upload empty document list");
    }
    h->n_empty = static_cast<int>(ids.size());
  }
  QueryView qv{};
  qv.batch = batch;
  const size_t bytes = tc_topk_cand_bytes(qv, k);
  h->w_topk.ensure(bytes, "cudaMalloc fused top-k candidates");
  *f = TopkFuse{};
  f->k = k;
  f->cand = h->w_topk.ptr;
  f->cand_bytes = h->w_topk.cap;
  f->empty_ids = h->empty_ids.as<int64_t>();
  f->n_empty = h->n_empty;
  f->out_s = out_s;
  f->out_i = out_i;
  return true;
}

// After a synchronising host-buffer call: surface a bounded-wait timeout of the
// tensor-core kernel (its first 4 workspace bytes) as a CUDA error.
void check_tc_flag(msb_docs* h, cudaStream_t s) {
  if (!h->tc_used) return;
  h->tc_used = false;
  int flag = 0;
  check(cudaMemcpyAsync(&flag, h->w_tc.ptr, sizeof(int), cudaMemcpyDeviceToHost, s), "read tc error flag");
  check(cudaStreamSynchronize(s), "synchronize tc error flag");
  if (flag != 0)
    throw CudaFailure("tensor-core scan aborted: a pipeline wait timed out (code " + std::to_string(flag) + ")");
}

void check_query(msb_docs* h, const void* q, int batch, int qtok) {
  if (batch < 0 || qtok < 0) throw InvalidArgument("query must have shape [batch, query_tokens, dim]");
  if (!q && static_cast<int64_t>(batch) * qtok > 0) throw InvalidArgument("query pointer is NULL");
  if (h && h->upload_open) throw InvalidArgument("the corpus upload has not finished (msb_docs_upload_finish)");
}

// The *_device entry points dereference their pointers in kernels: a pageable host pointer handed to
// one would fault the GPU, so it is refused here, before anything is enqueued.  Device, managed and
// pinned (mapped, unified-address) host memory are accessible from the device.
void require_device_accessible(const void* p, const char* what) {
  if (!p) return;
  cudaPointerAttributes attr{};
  const cudaError_t e = cudaPointerGetAttributes(&attr, p);
  if (e != cudaSuccess) {
    cudaGetLastError();  // clear the non-sticky error
    throw InvalidArgument(std::string(what) + " is not a CUDA pointer");
  }
  if (attr.type == cudaMemoryTypeUnregistered)
    throw InvalidArgument(std::string(what) + " must be device memory on a *_device call (got a host pointer)");
}

void require_device_opts(const msb_score_opts* o) {
  if (!o) return;
  if (o->reducer == kWeighted) require_device_accessible(o->weights, "opts.weights");
  require_device_accessible(o->doc_scale_override, "opts.doc_scale_override");
}

void check_candidates(msb_docs* h, const int64_t* c, int64_t m) {
  for (int64_t i = 0; i < m; ++i)
    if (c[i] < 0 || c[i] >= h->num_docs)
      throw InvalidArgument("candidate_indices entries must be between 0 and num_docs - 1");
}

// Copy host weights/override to device scratch; returns device pointers.
void stage_host_options(msb_docs* h, const msb_score_opts* o, int batch, int qtok, cudaStream_t s,
                        const float** d_w, const float** d_ov) {
  *d_w = nullptr;
  *d_ov = nullptr;
  if (o && o->reducer == kWeighted && o->weights) {
    const int rows = o->weight_rows == batch ? batch : 1;
    const size_t bytes = sizeof(float) * static_cast<size_t>(rows) * qtok;
    if (bytes) {
      h->w_weights.ensure(bytes, "cudaMalloc reducer query-weight cache");
      check(cudaMemcpyAsync(h->w_weights.ptr, o->weights, bytes, cudaMemcpyHostToDevice, s), "copy query weights");
      *d_w = h->w_weights.as<float>();
    } else {
      *d_w = reinterpret_cast<const float*>(o->weights);  // never dereferenced
    }
  }
  if (o && o->doc_scale_override) {
    const size_t bytes = sizeof(float) * static_cast<size_t>(h->num_docs);
    h->w_override.ensure(bytes > 0 ? bytes : 4, "cudaMalloc reducer scale-vector cache");
    check(cudaMemcpyAsync(h->w_override.ptr, o->doc_scale_override, bytes, cudaMemcpyHostToDevice, s),
          "copy scale-vector override");
    *d_ov = h->w_override.as<float>();
  }
}

// Host inputs and outputs up to this size go through the handle's page-locked staging buffers.
constexpr size_t kPinnedMax = size_t{8} << 20;

const float* stage_query(msb_docs* h, const float* q, int batch, int qtok, cudaStream_t s) {
  const size_t bytes = sizeof(float) * static_cast<size_t>(batch) * qtok * h->dim;
  if (!bytes) return nullptr;
  h->w_query.ensure(bytes, "cudaMalloc resident query cache");
  const void* src = q;
  if (bytes <= kPinnedMax) {
    // every host-buffer call ends with a stream synchronisation, so the staging buffer is free again
    h->pin_in.ensure(bytes, "cudaMallocHost query staging");
    std::memcpy(h->pin_in.ptr, q, bytes);
    src = h->pin_in.ptr;
  }
  check(cudaMemcpyAsync(h->w_query.ptr, src, bytes, cudaMemcpyHostToDevice, s), "copy query to device");
  return h->w_query.as<float>();
}

// Results of a host-buffer call: device -> caller copies, the tensor-core error word, one synchronisation.
struct HostCopy {
  void* dst;
  const void* src;
  size_t bytes;
};
void finish_host_call(msb_docs* h, cudaStream_t s, std::initializer_list<HostCopy> copies, const char* what) {
  size_t total = 16;  // the error word first
  for (const HostCopy& c : copies) total += (c.bytes + 15) & ~size_t{15};
  if (total > kPinnedMax) {
    for (const HostCopy& c : copies)
      check(cudaMemcpyAsync(c.dst, c.src, c.bytes, cudaMemcpyDeviceToHost, s), what);
    check(cudaStreamSynchronize(s), what);
    check_tc_flag(h, s);
    return;
  }
  h->pin_out.ensure(total, "cudaMallocHost result staging");
  unsigned char* pin = static_cast<unsigned char*>(h->pin_out.ptr);
  const bool flag = h->tc_used;
  if (flag) check(cudaMemcpyAsync(pin, h->w_tc.ptr, sizeof(int), cudaMemcpyDeviceToHost, s), "read tc error flag");
  size_t off = 16;
  for (const HostCopy& c : copies) {
    check(cudaMemcpyAsync(pin + off, c.src, c.bytes, cudaMemcpyDeviceToHost, s), what);
    off += (c.bytes + 15) & ~size_t{15};
  }
  check(cudaStreamSynchronize(s), what);
  if (flag) {
    h->tc_used = false;
    int code = 0;
    std::memcpy(&code, pin, sizeof(int));
    if (code != 0)
      throw CudaFailure("tensor-core scan aborted: a pipeline wait timed out (code " + std::to_string(code) + ")");
  }
  off = 16;
  for (const HostCopy& c : copies) {
    std::memcpy(c.dst, pin + off, c.bytes);
    off += (c.bytes + 15) & ~size_t{15};
  }
}

msb_docs* create_common(int32_t format, int32_t dim, int64_t num_tokens, const int64_t* offsets_host,
                        int64_t num_docs) {
  if (format != kFormatInt4 && format != kFormatBinary) throw InvalidArgument("unknown format");
  if (format == kFormatInt4 && (dim <= 0 || dim % 2 != 0)) throw InvalidArgument("dim must be positive and divisible by 2");
  if (dim <= 0 || dim % 8 != 0) throw InvalidArgument("dim must be positive and divisible by 8");
  if (num_tokens < 0) throw InvalidArgument("packed must have shape [num_doc_tokens, bytes]");
  if (!offsets_host || num_docs < 1) throw InvalidArgument("offsets must contain at least [0, num_doc_tokens]");
  if (num_docs > 0x7FFFFFFF) throw NotSupported("more than 2^31 - 1 documents per handle");
  validate_offsets(offsets_host, num_docs, num_tokens);
  auto* h = new msb_docs();
  h->serial = g_corpus_serial.fetch_add(1) + 1;
  h->format = format;
  h->dim = dim;
  h->num_docs = num_docs;
  h->num_tokens = num_tokens;
  cudaGetDevice(&h->device);
  check(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking), "create handle stream");
  h->host_offsets.assign(offsets_host, offsets_host + num_docs + 1);
  return h;
}

}  // namespace

extern "C" {

const char* msb_last_error(void) { return g_last_error.c_str(); }
int msb_version(void) { return 1; }
int64_t msb_launch_count(void) { return g_launches.load(); }

int msb_set_option(const char* name, int64_t value) {
  return guarded([&] {
    if (!name) throw InvalidArgument("option name is NULL");
    if (std::strcmp(name, "engine") == 0) {
      if (value < 0 || value > 3)
        throw InvalidArgument("engine must be 0 (auto), 1 (SIMT), 2 (tensor core) or 3 (popcount, sign codes)");
      g_engine.store(static_cast<int>(value));
      return;
    }
    if (std::strcmp(name, "tc_int8_cache") == 0) {
      if (value != 0 && value != 1) throw InvalidArgument("tc_int8_cache must be 0 or 1");
      g_tc_int8_cache.store(static_cast<int>(value));
      return;
    }
    if (std::strcmp(name, "tc_f16_cache") == 0) {
      if (value != 0 && value != 1) throw InvalidArgument("tc_f16_cache must be 0 or 1");
      g_tc_f16_cache.store(static_cast<int>(value));
      return;
    }
    if (std::strcmp(name, "tc_fused_topk") == 0) {
      if (value != 0 && value != 1) throw InvalidArgument("tc_fused_topk must be 0 or 1");
      g_tc_fused_topk.store(static_cast<int>(value));
      return;
    }
    if (std::strcmp(name, "tc_row_replicas") == 0) {
      if (value != 0 && value != 1) throw InvalidArgument("tc_row_replicas must be 0 or 1");
      set_tc_row_replicas(static_cast<int>(value));
      return;
    }
    throw InvalidArgument(std::string("unknown option: ") + name);
  });
}

int msb_get_option(const char* name, int64_t* value) {
  return guarded([&] {
    if (!name || !value) throw InvalidArgument("NULL argument");
    if (std::strcmp(name, "engine") == 0) {
      *value = g_engine.load();
      return;
    }
    if (std::strcmp(name, "tc_int8_cache") == 0) {
      *value = g_tc_int8_cache.load();
      return;
    }
    if (std::strcmp(name, "tc_f16_cache") == 0) {
      *value = g_tc_f16_cache.load();
      return;
    }
    if (std::strcmp(name, "tc_fused_topk") == 0) {
      *value = g_tc_fused_topk.load();
      return;
    }
    if (std::strcmp(name, "tc_row_replicas") == 0) {
      *value = get_tc_row_replicas();
      return;
    }
    throw InvalidArgument(std::string("unknown option: ") + name);
  });
}

int msb_docs_create(int32_t format, int32_t dim, const uint8_t* codes, int64_t num_tokens, const int64_t* offsets,
                    int64_t num_docs, float scale, msb_docs** out) {
  return guarded([&] {
    if (!out) throw InvalidArgument("out is NULL");
    *out = nullptr;
    if (format == kFormatInt4 && (!(scale > 0.0F) || !std::isfinite(scale)))
      throw InvalidArgument("scale must be finite and > 0");
    msb_docs* h = create_common(format, dim, num_tokens, offsets, num_docs);
    try {
      h->scale = format == kFormatInt4 ? scale : 1.0F;
      const size_t cbytes = h->bytes_per_token() * static_cast<size_t>(num_tokens);
      if (cbytes) {
        if (!codes) throw InvalidArgument("packed pointer is NULL");
        h->codes.ensure(cbytes, "cudaMalloc packed docs");
        check(cudaMemcpyAsync(h->codes.ptr, codes, cbytes, cudaMemcpyHostToDevice, h->stream),
              "copy packed docs to device");
      }
      h->offsets.ensure(sizeof(int64_t) * (num_docs + 1) + kTailPad, "cudaMalloc offsets");
      check(cudaMemcpyAsync(h->offsets.ptr, offsets, sizeof(int64_t) * (num_docs + 1), cudaMemcpyHostToDevice,
                            h->stream),
            "copy offsets to device");
      check(cudaStreamSynchronize(h->stream), "synchronize upload");
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
  });
}

int msb_docs_create_device(int32_t format, int32_t dim, const uint8_t* codes, int64_t num_tokens,
                           const int64_t* offsets_device, const int64_t* offsets_host, int64_t num_docs, float scale,
                           msb_docs** out) {
  return guarded([&] {
    if (!out) throw InvalidArgument("out is NULL");
    *out = nullptr;
    if (format == kFormatInt4 && (!(scale > 0.0F) || !std::isfinite(scale)))
      throw InvalidArgument("scale must be finite and > 0");
    msb_docs* h = create_common(format, dim, num_tokens, offsets_host, num_docs);
    try {
      h->scale = format == kFormatInt4 ? scale : 1.0F;
      const size_t cbytes = h->bytes_per_token() * static_cast<size_t>(num_tokens);
      if (cbytes) {
        h->codes.ensure(cbytes, "cudaMalloc packed docs");
        check(cudaMemcpyAsync(h->codes.ptr, codes, cbytes, cudaMemcpyDeviceToDevice, h->stream), "copy packed docs");
      }
      h->offsets.ensure(sizeof(int64_t) * (num_docs + 1) + kTailPad, "cudaMalloc offsets");
      const void* src = offsets_device ? static_cast<const void*>(offsets_device) : offsets_host;
      check(cudaMemcpyAsync(h->offsets.ptr, src, sizeof(int64_t) * (num_docs + 1), cudaMemcpyDefault, h->stream),
            "copy offsets");
      check(cudaStreamSynchronize(h->stream), "synchronize upload");
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
  });
}

int msb_docs_destroy(msb_docs* docs) {
  return guarded([&] { delete docs; });
}

int msb_docs_get_info(const msb_docs* h, msb_docs_info* info) {
  return guarded([&] {
    if (!h || !info) throw InvalidArgument("NULL argument");
    info->format = h->format;
    info->dim = h->dim;
    info->num_docs = h->num_docs;
    info->num_tokens = h->num_tokens;
    info->packed_size = static_cast<int64_t>(h->bytes_per_token()) * h->num_tokens;
    info->scale = h->scale;
    info->residual_scale = h->residual_scale;
    info->has_token_scale = h->has_token_scale;
    info->has_doc_scale = h->has_doc_scale;
    info->has_residual = h->has_residual;
    info->device = h->device;
    info->resident_bytes = h->resident_bytes();
    info->workspace_bytes = h->workspace_bytes();
  });
}

int msb_docs_set_token_scales(msb_docs* h, const float* scales, int64_t count, int32_t require_positive) {
  return guarded([&] {
    if (!h) throw InvalidArgument("handle is NULL");
    if (count != h->num_tokens) throw InvalidArgument("token scale vector must have shape [num_doc_tokens]");
    if (require_positive)
      for (int64_t i = 0; i < count; ++i)
        if (!(scales[i] > 0.0F) || !std::isfinite(scales[i]))
          throw InvalidArgument("token scales must be finite and > 0");
    DeviceGuard g(h->device);
    const size_t bytes = sizeof(float) * static_cast<size_t>(count);
    h->token_scale.ensure(bytes + kTailPad, "cudaMalloc resident token scale vector");
    if (bytes) {
      check(cudaMemcpyAsync(h->token_scale.ptr, scales, bytes, cudaMemcpyHostToDevice, h->stream),
            "copy token scale vector to device");
      check(cudaStreamSynchronize(h->stream), "synchronize token scale upload");
    }
    h->has_token_scale = true;
    h->token_scale_small = -1;
  });
}

int msb_docs_set_token_scales_device(msb_docs* h, const float* scales, int64_t count) {
  return guarded([&] {
    if (!h) throw InvalidArgument("handle is NULL");
    if (count != h->num_tokens) throw InvalidArgument("token scale vector must have shape [num_doc_tokens]");
    DeviceGuard g(h->device);
    const size_t bytes = sizeof(float) * static_cast<size_t>(count);
    h->token_scale.ensure(bytes + kTailPad, "cudaMalloc resident token scale vector");
    if (bytes) {
      check(cudaMemcpyAsync(h->token_scale.ptr, scales, bytes, cudaMemcpyDeviceToDevice, h->stream),
            "copy token scale vector");
      check(cudaStreamSynchronize(h->stream), "synchronize token scale upload");
    }
    h->has_token_scale = true;
    h->token_scale_small = -1;
  });
}

int msb_docs_clear_token_scales(msb_docs* h) {
  return guarded([&] {
    if (!h) throw InvalidArgument("handle is NULL");
    h->has_token_scale = false;
  });
}

int msb_docs_set_doc_scales(msb_docs* h, const float* scales, int64_t count) {
  return guarded([&] {
    if (!h) throw InvalidArgument("handle is NULL");
    if (count != h->num_docs) throw InvalidArgument("scale vector must have shape [num_docs]");
    DeviceGuard g(h->device);
    const size_t bytes = sizeof(float) * static_cast<size_t>(count);
    h->doc_scale.ensure(bytes, "cudaMalloc resident scale vector");
    check(cudaMemcpyAsync(h->doc_scale.ptr, scales, bytes, cudaMemcpyHostToDevice, h->stream),
          "copy scale vector to device");
    check(cudaStreamSynchronize(h->stream), "synchronize scale upload");
    h->has_doc_scale = true;
  });
}

int msb_docs_clear_doc_scales(msb_docs* h) {
  return guarded([&] {
    if (!h) throw InvalidArgument("handle is NULL");
    h->has_doc_scale = false;
  });
}

int msb_docs_set_residual(msb_docs* h, const uint8_t* codes, int64_t num_tokens, float scale,
                          const float* token_scales) {
  return guarded([&] {
    if (!h) throw InvalidArgument("handle is NULL");
    if (num_tokens != h->num_tokens)
      throw InvalidArgument("residual packed data must have shape [num_doc_tokens, dim / 2]");
    if (h->format == kFormatBinary && scale != 1.0F)
      throw InvalidArgument("a binary handle's residual stream uses per-token scales only (scale must be 1)");
    if (!(scale > 0.0F) || !std::isfinite(scale)) throw InvalidArgument("residual scale must be finite and > 0");
    for (int64_t i = 0; i < num_tokens; ++i)
      if (!(token_scales[i] > 0.0F) || !std::isfinite(token_scales[i]))
        throw InvalidArgument("residual token scales must be finite and > 0");
    DeviceGuard g(h->device);
    const size_t cbytes = static_cast<size_t>(h->dim / 2) * static_cast<size_t>(num_tokens);  // int4 residual
    const size_t sbytes = sizeof(float) * static_cast<size_t>(num_tokens);
    h->residual_codes.ensure(cbytes > 0 ? cbytes : 4, "cudaMalloc resident int4 residual data");
    h->residual_token_scale.ensure(sbytes + kTailPad, "cudaMalloc resident int4 residual token scales");
    if (cbytes)
      check(cudaMemcpyAsync(h->residual_codes.ptr, codes, cbytes, cudaMemcpyHostToDevice, h->stream),
            "copy int4 residual data to device");
    if (sbytes)
      check(cudaMemcpyAsync(h->residual_token_scale.ptr, token_scales, sbytes, cudaMemcpyHostToDevice, h->stream),
            "copy int4 residual token scales to device");
    check(cudaStreamSynchronize(h->stream), "synchronize residual upload");
    h->residual_scale = scale;
    h->codes2_8.release();  // the int8 copy of the previous residual stream
    h->codes2_8_failed = false;
    h->has_residual = true;
  });
}

int msb_docs_create_for_upload(int32_t format, int32_t dim, int64_t num_tokens, const int64_t* offsets,
                               int64_t num_docs, float scale, int32_t flags, msb_docs** out) {
  return guarded([&] {
    if (!out) throw InvalidArgument("out is NULL");
    *out = nullptr;
    if (format == kFormatInt4 && (!(scale > 0.0F) || !std::isfinite(scale)))
      throw InvalidArgument("scale must be finite and > 0");
    if (flags & ~(MSB_UPLOAD_TOKEN_SCALES | MSB_UPLOAD_RESIDUAL)) throw InvalidArgument("unknown upload flags");
    msb_docs* h = create_common(format, dim, num_tokens, offsets, num_docs);
    try {
      h->scale = format == kFormatInt4 ? scale : 1.0F;
      const size_t n = static_cast<size_t>(num_tokens);
      const size_t cbytes = h->bytes_per_token() * n;
      if (cbytes) h->codes.ensure(cbytes, "cudaMalloc packed docs");
      h->offsets.ensure(sizeof(int64_t) * (num_docs + 1) + kTailPad, "cudaMalloc offsets");
      check(cudaMemcpyAsync(h->offsets.ptr, offsets, sizeof(int64_t) * (num_docs + 1), cudaMemcpyHostToDevice,
                            h->stream),
            "copy offsets to device");
      if (flags & MSB_UPLOAD_TOKEN_SCALES)
        h->token_scale.ensure(sizeof(float) * n + kTailPad, "cudaMalloc resident token scale vector");
      if (flags & MSB_UPLOAD_RESIDUAL) {
        const size_t rbytes = static_cast<size_t>(dim / 2) * n;
        h->residual_codes.ensure(rbytes > 0 ? rbytes : 4, "cudaMalloc resident int4 residual data");
        h->residual_token_scale.ensure(sizeof(float) * n + kTailPad, "cudaMalloc resident int4 residual token scales");
      }
      for (cudaEvent_t& e : h->upload_events)
        check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "create upload event");
      check(cudaStreamSynchronize(h->stream), "synchronize upload setup");
      h->upload_flags = flags;
      h->upload_open = true;
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
  });
}

int msb_docs_upload(msb_docs* h, int32_t which, int64_t offset, const void* host, int64_t bytes, int64_t* ticket) {
  return guarded([&] {
    if (!h) throw InvalidArgument("handle is NULL");
    if (!h->upload_open) throw InvalidArgument("the handle is not open for upload (msb_docs_create_for_upload)");
    if (offset < 0 || bytes < 0) throw InvalidArgument("upload offset and size must be nonnegative");
    if (bytes > 0 && !host) throw InvalidArgument("host pointer is NULL");
    const int64_t n = h->num_tokens;
    unsigned char* base = nullptr;
    int64_t size = 0;
    switch (which) {
      case MSB_ARRAY_CODES:
        base = static_cast<unsigned char*>(h->codes.ptr);
        size = static_cast<int64_t>(h->bytes_per_token()) * n;
        break;
      case MSB_ARRAY_TOKEN_SCALES:
        if (!(h->upload_flags & MSB_UPLOAD_TOKEN_SCALES)) throw InvalidArgument("the handle has no token scale upload");
        base = static_cast<unsigned char*>(h->token_scale.ptr);
        size = 4 * n;
        break;
      case MSB_ARRAY_RESIDUAL_CODES:
        if (!(h->upload_flags & MSB_UPLOAD_RESIDUAL)) throw InvalidArgument("the handle has no residual upload");
        base = static_cast<unsigned char*>(h->residual_codes.ptr);
        size = static_cast<int64_t>(h->dim / 2) * n;
        break;
      case MSB_ARRAY_RESIDUAL_TOKEN_SCALES:
        if (!(h->upload_flags & MSB_UPLOAD_RESIDUAL)) throw InvalidArgument("the handle has no residual upload");
        base = static_cast<unsigned char*>(h->residual_token_scale.ptr);
        size = 4 * n;
        break;
      default:
        throw InvalidArgument("unknown upload array");
    }
    if (offset > size || bytes > size - offset) throw InvalidArgument("upload range exceeds the array");
    DeviceGuard g(h->device);
    if (bytes > 0)
      check(cudaMemcpyAsync(base + offset, host, static_cast<size_t>(bytes), cudaMemcpyHostToDevice, h->stream),
            "upload chunk to device");
    const int64_t t = ++h->upload_serial;
    check(cudaEventRecord(h->upload_events[t % msb_docs::kUploadEvents], h->stream), "record upload event");
    if (ticket) *ticket = t;
  });
}

int msb_docs_upload_wait(msb_docs* h, int64_t ticket) {
  return guarded([&] {
    if (!h) throw InvalidArgument("handle is NULL");
    if (ticket <= 0 || ticket > h->upload_serial) throw InvalidArgument("unknown upload ticket");
    DeviceGuard g(h->device);
    // A slot reused by a later copy on the same stream completes after this ticket's copy.
    check(cudaEventSynchronize(h->upload_events[ticket % msb_docs::kUploadEvents]), "wait for upload");
  });
}

int msb_docs_upload_finish(msb_docs* h, float residual_scale) {
  return guarded([&] {
    if (!h) throw InvalidArgument("handle is NULL");
    if (!h->upload_open) throw InvalidArgument("the handle is not open for upload (msb_docs_create_for_upload)");
    const bool residual = (h->upload_flags & MSB_UPLOAD_RESIDUAL) != 0;
    if (residual) {
      if (h->format == kFormatBinary && residual_scale != 1.0F)
        throw InvalidArgument("a binary handle's residual stream uses per-token scales only (scale must be 1)");
      if (!(residual_scale > 0.0F) || !std::isfinite(residual_scale))
        throw InvalidArgument("residual scale must be finite and > 0");
    }
    DeviceGuard g(h->device);
    h->w_check.ensure(4 * sizeof(unsigned int), "cudaMalloc upload check flags");
    unsigned int* bad = static_cast<unsigned int*>(h->w_check.ptr);
    check(cudaMemsetAsync(bad, 0, 4 * sizeof(unsigned int), h->stream), "clear upload check flags");
    const int64_t rbytes = static_cast<int64_t>(h->dim / 2) * h->num_tokens;
    if (h->format == kFormatInt4) launch_check_int4_codes(static_cast<const uint8_t*>(h->codes.ptr), rbytes, bad, h->stream);
    if (h->upload_flags & MSB_UPLOAD_TOKEN_SCALES)
      launch_check_positive_finite(static_cast<const float*>(h->token_scale.ptr), h->num_tokens, bad + 1, h->stream);
    if (residual) {
      launch_check_int4_codes(static_cast<const uint8_t*>(h->residual_codes.ptr), rbytes, bad + 2, h->stream);
      launch_check_positive_finite(static_cast<const float*>(h->residual_token_scale.ptr), h->num_tokens, bad + 3,
                                   h->stream);
    }
    unsigned int flags[4] = {0, 0, 0, 0};
    check(cudaMemcpyAsync(flags, bad, sizeof(flags), cudaMemcpyDeviceToHost, h->stream), "read upload check flags");
    check(cudaStreamSynchronize(h->stream), "synchronize upload");
    if (flags[0]) throw InvalidArgument("int4 codes must be symmetric int4 values in [-7, 7]");
    if (flags[1]) throw InvalidArgument("token scales must be finite and > 0");
    if (flags[2]) throw InvalidArgument("residual int4 codes must be symmetric int4 values in [-7, 7]");
    if (flags[3]) throw InvalidArgument("residual token scales must be finite and > 0");
    h->has_token_scale = (h->upload_flags & MSB_UPLOAD_TOKEN_SCALES) != 0;
    h->token_scale_small = -1;
    if (residual) {
      h->residual_scale = residual_scale;
      h->codes2_8.release();  // the int8 copy of the previous residual stream
      h->codes2_8_failed = false;
      h->has_residual = true;
    }
    h->upload_open = false;
  });
}

int msb_pinned_alloc(int64_t bytes, void** out) {
  return guarded([&] {
    if (!out) throw InvalidArgument("out is NULL");
    *out = nullptr;
    if (bytes <= 0) throw InvalidArgument("staging buffer size must be > 0");
    check(cudaHostAlloc(out, static_cast<size_t>(bytes), cudaHostAllocPortable), "cudaHostAlloc staging buffer");
  });
}

int msb_pinned_free(void* ptr) {
  return guarded([&] {
    if (ptr) check(cudaFreeHost(ptr), "cudaFreeHost staging buffer");
  });
}

int msb_docs_clear_residual(msb_docs* h) {
  return guarded([&] {
    if (!h) throw InvalidArgument("handle is NULL");
    h->codes2_8.release();  // the int8 copy of the previous residual stream
    h->codes2_8_failed = false;
    h->has_residual = false;
  });
}

int msb_docs_score(msb_docs* h, const float* query, int32_t batch, int32_t qtok, const msb_score_opts* opts,
                   const int64_t* candidates, int64_t num_candidates, float* out) {
  return guarded([&] {
    if (!h) throw InvalidArgument("handle is NULL");
    check_query(h, query, batch, qtok);
    if (candidates) check_candidates(h, candidates, num_candidates);
    DeviceGuard g(h->device);
    cudaStream_t s = h->stream;
    const float *d_w, *d_ov;
    stage_host_options(h, opts, batch, qtok, s, &d_w, &d_ov);
    Resolved r = resolve(h, opts, batch, qtok, d_w, d_ov);
    const int64_t T = candidates ? num_candidates : h->num_docs;
    if (batch == 0 || T == 0) return;
    const float* d_q = stage_query(h, query, batch, qtok, s);
    TargetsView tg{};
    if (candidates) {
      h->w_cands.ensure(sizeof(int64_t) * T, "cudaMalloc reducer candidate cache");
      check(cudaMemcpyAsync(h->w_cands.ptr, candidates, sizeof(int64_t) * T, cudaMemcpyHostToDevice, s),
            "copy reducer candidates to device");
      tg.ids = h->w_cands.as<int64_t>();
      tg.count = T;
    }
    const size_t obytes = sizeof(float) * static_cast<size_t>(batch) * T;
    h->w_scores.ensure(obytes, "cudaMalloc resident score cache");
    run_scan(h, r, d_q, batch, qtok, tg, h->w_scores.as<float>(), s);
    finish_host_call(h, s, {{out, h->w_scores.ptr, obytes}}, "copy scores to host");
  });
}

int msb_docs_topk(msb_docs* h, const float* query, int32_t batch, int32_t qtok, int32_t k, const msb_score_opts* opts,
                  float* out_scores, int64_t* out_ids) {
  return guarded([&] {
    if (!h) throw InvalidArgument("handle is NULL");
    if (k < 1 || k > h->num_docs) throw InvalidArgument("k must be between 1 and num_docs");
    check_query(h, query, batch, qtok);
    DeviceGuard g(h->device);
    cudaStream_t s = h->stream;
    const float *d_w, *d_ov;
    stage_host_options(h, opts, batch, qtok, s, &d_w, &d_ov);
    Resolved r = resolve(h, opts, batch, qtok, d_w, d_ov);
    if (batch == 0) return;
    const float* d_q = stage_query(h, query, batch, qtok, s);
    h->w_scores.ensure(sizeof(float) * static_cast<size_t>(batch) * h->num_docs, "cudaMalloc full score cache");
    h->w_top_s.ensure(sizeof(float) * static_cast<size_t>(batch) * k, "cudaMalloc top score cache");
    h->w_top_i.ensure(sizeof(int64_t) * static_cast<size_t>(batch) * k, "cudaMalloc top index cache");
    TargetsView tg{};
    TopkFuse fuse{};
    const bool try_fuse = prepare_fused_topk(h, batch, k, h->w_top_s.as<float>(), h->w_top_i.as<int64_t>(), &fuse);
    run_scan(h, r, d_q, batch, qtok, tg, h->w_scores.as<float>(), s, try_fuse ? &fuse : nullptr);
    if (!fuse.done) topk_full_rows(h, h->w_scores.as<float>(), batch, k, h->w_top_s.as<float>(), h->w_top_i.as<int64_t>(), s);
    finish_host_call(h, s,
                     {{out_scores, h->w_top_s.ptr, sizeof(float) * static_cast<size_t>(batch) * k},
                      {out_ids, h->w_top_i.ptr, sizeof(int64_t) * static_cast<size_t>(batch) * k}},
                     "copy top-k to host");
  });
}

int msb_docs_cascade_topk(msb_docs* h, const float* query, int32_t batch, int32_t qtok, int32_t k, int32_t m,
                          const msb_score_opts* opts, float* out_scores, int64_t* out_ids) {
  return guarded([&] {
    if (!h) throw InvalidArgument("handle is NULL");
    if (k < 1 || k > m || m > h->num_docs)
      throw InvalidArgument("cascade sizes must satisfy 1 <= k <= candidates <= num_docs");
    if (!h->has_residual || !h->has_token_scale)
      throw InvalidArgument("the cascade requires per-token prefix scales and residual int4 data");
    check_query(h, query, batch, qtok);
    DeviceGuard g(h->device);
    cudaStream_t s = h->stream;
    const float *d_w, *d_ov;
    stage_host_options(h, opts, batch, qtok, s, &d_w, &d_ov);
    msb_score_opts prefix_opts = *opts;
    prefix_opts.use_residual = 0;
    prefix_opts.query_mode = kQueryF32;
    if (h->format == kFormatBinary) {
      // binary prefix: sign scan scaled by the per-token reconstruction scale
      prefix_opts.use_token_scale = 1;
      prefix_opts.use_doc_scale = 0;
      prefix_opts.scale = 1.0F;
      prefix_opts.doc_scale_override = nullptr;
    }
    Resolved rp = resolve(h, &prefix_opts, batch, qtok, d_w, d_ov);
    msb_score_opts fine_opts = prefix_opts;
    fine_opts.use_residual = 1;
    Resolved rf = resolve(h, &fine_opts, batch, qtok, d_w, d_ov);
    if (batch == 0) return;
    const float* d_q = stage_query(h, query, batch, qtok, s);
    const size_t B = static_cast<size_t>(batch);
    h->w_top_s.ensure(sizeof(float) * B * k, "cudaMalloc top score cache");
    h->w_top_i.ensure(sizeof(int64_t) * B * k, "cudaMalloc top index cache");
    if (m == h->num_docs) {
      h->w_scores.ensure(sizeof(float) * B * h->num_docs, "cudaMalloc full score cache");
      run_scan(h, rf, d_q, batch, qtok, TargetsView{}, h->w_scores.as<float>(), s);
      topk_full_rows(h, h->w_scores.as<float>(), batch, k, h->w_top_s.as<float>(), h->w_top_i.as<int64_t>(), s);
    } else {
      h->w_scores.ensure(sizeof(float) * B * h->num_docs, "cudaMalloc coarse score cache");
      h->w_cands.ensure(sizeof(int64_t) * B * m, "cudaMalloc cascade candidate cache");
      h->w_fine.ensure(sizeof(float) * B * m * 2, "cudaMalloc cascade fine score cache");
      run_scan(h, rp, d_q, batch, qtok, TargetsView{}, h->w_scores.as<float>(), s);
      // Per-row top-M of the prefix scores (values land in the second half of w_fine).
      float* top_m_scores = h->w_fine.as<float>() + B * m;
      topk_full_rows(h, h->w_scores.as<float>(), batch, m, top_m_scores, h->w_cands.as<int64_t>(), s);
      TargetsView tg{};
      tg.ids = h->w_cands.as<int64_t>();
      tg.count = m;
      tg.per_row = 1;
      // Rescoring of per-row candidate lists: from the full tensor-core residual scan when the lists are
      // long enough, else from a tensor-core scan of the listed documents (or the SIMT engine).
      run_scan(h, rf, d_q, batch, qtok, tg, h->w_fine.as<float>(), s);
      launch_topk_rows(h->w_fine.as<float>(), m, batch, m, k, h->w_cands.as<int64_t>(), true,
                       h->w_top_s.as<float>(), h->w_top_i.as<int64_t>(), s);
    }
    finish_host_call(h, s, {{out_scores, h->w_top_s.ptr, sizeof(float) * B * k},
                            {out_ids, h->w_top_i.ptr, sizeof(int64_t) * B * k}},
                     "copy cascade top-k to host");
  });
}

int msb_docs_score_device(msb_docs* h, const float* query, int32_t batch, int32_t qtok, const msb_score_opts* opts,
                          const int64_t* candidates, int64_t num_candidates, float* out, void* stream) {
  return guarded([&] {
    if (!h) throw InvalidArgument("handle is NULL");
    check_query(h, query, batch, qtok);
    DeviceGuard g(h->device);
    if (static_cast<int64_t>(batch) * qtok > 0) require_device_accessible(query, "query");
    require_device_accessible(candidates, "candidates");
    require_device_accessible(out, "out");
    require_device_opts(opts);
    cudaStream_t s = pick_stream(h, stream);
    Resolved r = resolve(h, opts, batch, qtok, opts ? opts->weights : nullptr, opts ? opts->doc_scale_override : nullptr);
    TargetsView tg{};
    if (candidates) {
      tg.ids = candidates;
      tg.count = num_candidates;
    }
    run_scan(h, r, query, batch, qtok, tg, out, s);
  });
}

int msb_docs_topk_device(msb_docs* h, const float* query, int32_t batch, int32_t qtok, int32_t k,
                         const msb_score_opts* opts, float* out_scores, int64_t* out_ids, void* stream) {
  return guarded([&] {
    if (!h) throw InvalidArgument("handle is NULL");
    if (k < 1 || k > h->num_docs) throw InvalidArgument("k must be between 1 and num_docs");
    check_query(h, query, batch, qtok);
    DeviceGuard g(h->device);
    if (static_cast<int64_t>(batch) * qtok > 0) require_device_accessible(query, "query");
    require_device_accessible(out_scores, "out_scores");
    require_device_accessible(out_ids, "out_ids");
    require_device_opts(opts);
    cudaStream_t s = pick_stream(h, stream);
    Resolved r = resolve(h, opts, batch, qtok, opts ? opts->weights : nullptr, opts ? opts->doc_scale_override : nullptr);
    if (batch == 0) return;
    h->w_scores.ensure(sizeof(float) * static_cast<size_t>(batch) * h->num_docs, "cudaMalloc full score cache");
    TopkFuse fuse{};
    const bool try_fuse = prepare_fused_topk(h, batch, k, out_scores, out_ids, &fuse);
    run_scan(h, r, query, batch, qtok, TargetsView{}, h->w_scores.as<float>(), s, try_fuse ? &fuse : nullptr);
    if (!fuse.done) topk_full_rows(h, h->w_scores.as<float>(), batch, k, out_scores, out_ids, s);
  });
}

int msb_topk_rows_device(const float* scores, int64_t ld, int32_t rows, int64_t count, int32_t k,
                         const int64_t* tie_ids, int32_t tie_batched, float* out_scores, int64_t* out_ids,
                         void* stream) {
  return guarded([&] {
    if (ld < count) throw InvalidArgument("ld must be >= count");
    launch_topk_rows(scores, ld, rows, count, k, tie_ids, tie_batched != 0, out_scores, out_ids,
                     static_cast<cudaStream_t>(stream));
  });
}

int msb_merge_shard_topk_device(const void* gathered, int32_t world, int32_t batch, int32_t k,
                                const int64_t* first_doc, float* out_scores, int64_t* out_ids, void* stream) {
  return guarded([&] {
    if (!gathered || !first_doc || !out_scores || !out_ids) throw InvalidArgument("NULL argument");
    launch_merge_shard_topk(gathered, world, batch, k, first_doc, out_scores, out_ids,
                            static_cast<cudaStream_t>(stream));
  });
}

int msb_quantize_query_int8_device(const float* query, int64_t rows, int32_t dim, int8_t* codes, float* scales,
                                   void* stream) {
  return guarded([&] {
    if (dim <= 0 || dim % 8 != 0) throw InvalidArgument("dim must be positive and divisible by 8");
    launch_quantize_rows(query, rows, dim, codes, scales, nullptr, nullptr, false, static_cast<cudaStream_t>(stream));
  });
}

int msb_pack_int4_device(const float* x, int64_t n, int32_t dim, int32_t per_token, uint8_t* codes,
                         float* token_scales, float* tensor_scale, void* stream) {
  return guarded([&] {
    if (dim <= 0 || dim % 8 != 0) throw InvalidArgument("dim must be positive and divisible by 8");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (per_token) {
      if (!token_scales) throw InvalidArgument("token_scales is NULL");
      launch_pack_int4(x, n, dim, true, codes, token_scales, nullptr, nullptr, s);
      return;
    }
    void* scratch = nullptr;
    check(cudaMalloc(&scratch, 16), "cudaMalloc absmax scratch");
    try {
      launch_pack_int4(x, n, dim, false, codes, nullptr, tensor_scale, scratch, s);
    } catch (...) {
      cudaFree(scratch);
      throw;
    }
    cudaFree(scratch);
  });
}

int msb_pack_signs_device(const float* x, int64_t n, int32_t dim, uint8_t* bits, float* mean_abs, void* stream) {
  return guarded([&] {
    if (dim <= 0 || dim % 8 != 0) throw InvalidArgument("dim must be positive and divisible by 8");
    launch_pack_signs(x, n, dim, bits, mean_abs, static_cast<cudaStream_t>(stream));
  });
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free full-scan top-k (msb_docs_topk_device_noalloc)
// ---------------------------------------------------------------------------
// Fixed scratch for callers that cannot allocate device memory: the score
// matrix and the int8 query rows of one call.  Each device that loads the
// library holds it until the process exits; all calls on a device share it.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MSB_NOALLOC_SCRATCH_BYTES];

namespace {

// In host code `g_noalloc_scratch` names a host-side stand-in, not device
// memory, so kernels are given the device address looked up here: once per
// device, with that device current (the caller's DeviceGuard makes it so).
unsigned char* noalloc_scratch_on_current_device() {
  static std::mutex mu;
  static std::vector<void*> addr;
  int dev = 0;
  check(cudaGetDevice(&dev), "get device");
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= static_cast<int>(addr.size())) addr.resize(static_cast<size_t>(dev) + 1, nullptr);
  if (!addr[dev]) {
    void* p = nullptr;
    check(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress of the no-alloc scratch");
    addr[dev] = p;
  }
  return static_cast<unsigned char*>(addr[dev]);
}

constexpr size_t round256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

}  // namespace

extern "C" int msb_docs_topk_device_noalloc(msb_docs* h, const float* query, int32_t batch, int32_t qtok, int32_t k,
                                            const msb_score_opts* opts, float* out_scores, int64_t* out_ids,
                                            void* stream) {
  return guarded([&] {
    if (!h) throw InvalidArgument("handle is NULL");
    if (k < 1 || k > h->num_docs) throw InvalidArgument("k must be between 1 and num_docs");
    check_query(h, query, batch, qtok);
    DeviceGuard g(h->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // Pointers the kernels dereference must be device-accessible: checked on every call (host queries).
    if (static_cast<int64_t>(batch) * qtok > 0) require_device_accessible(query, "query");
    require_device_accessible(out_scores, "out_scores");
    require_device_accessible(out_ids, "out_ids");
    require_device_opts(opts);
    Resolved r = resolve(h, opts, batch, qtok, opts ? opts->weights : nullptr, opts ? opts->doc_scale_override : nullptr);
    if (batch == 0) return;
    // Scratch layout: scores [batch, num_docs] fp32, then (int8 queries) codes,
    // scan-order words, scales and code sums of the batch * qtok query rows.
    constexpr size_t cap = MSB_NOALLOC_SCRATCH_BYTES;
    const int64_t rows = static_cast<int64_t>(batch) * qtok;
    const bool fits = h->num_docs <= static_cast<int64_t>(cap / sizeof(float) / static_cast<size_t>(batch)) &&
                      rows <= static_cast<int64_t>(cap / static_cast<size_t>(h->dim));
    size_t need = fits ? round256(sizeof(float) * static_cast<size_t>(batch) * h->num_docs) : cap + 1;
    const size_t codes_at = need;
    const size_t words_at = codes_at + round256(static_cast<size_t>(rows) * h->dim);
    const size_t scales_at = words_at + round256(static_cast<size_t>(rows) * h->dim);
    const size_t sums_at = scales_at + round256(static_cast<size_t>(rows) * sizeof(float));
    if (fits && r.mode == kQueryI8) need = sums_at + round256(static_cast<size_t>(rows) * sizeof(int32_t));
    if (need > cap)
      throw InvalidArgument("msb_docs_topk_device_noalloc: batch " + std::to_string(batch) + " x " +
                            std::to_string(h->num_docs) + " documents (" + std::to_string(qtok) +
                            " query tokens) needs more than its fixed scratch of " + std::to_string(cap) +
                            " bytes; use msb_docs_topk_device or a smaller batch");
    unsigned char* base = noalloc_scratch_on_current_device();
    float* scores = reinterpret_cast<float*>(base);
    if (qtok == 0) {
      check(cudaMemsetAsync(scores, 0, sizeof(float) * static_cast<size_t>(batch) * h->num_docs, s), "zero scores");
    } else {
      QueryView qv{};
      qv.f32 = query;
      qv.batch = batch;
      qv.qtok = qtok;
      qv.mode = r.mode;
      if (r.mode == kQueryI8) {
        qv.i8 = reinterpret_cast<const int8_t*>(base + codes_at);
        qv.i8_words = reinterpret_cast<const int32_t*>(base + words_at);
        qv.row_scale = reinterpret_cast<const float*>(base + scales_at);
        qv.row_sum = reinterpret_cast<const int32_t*>(base + sums_at);
        launch_quantize_rows(query, rows, h->dim, reinterpret_cast<int8_t*>(base + codes_at),
                             reinterpret_cast<float*>(base + scales_at), reinterpret_cast<int32_t*>(base + sums_at),
                             reinterpret_cast<int32_t*>(base + words_at), h->format == kFormatInt4, s);
      }
      // Every score is written by the scan, so nothing in the scratch needs clearing.
      launch_simt_scan(r.docs, qv, r.red, TargetsView{}, r.residual, scores, s);
    }
    launch_topk_rows(scores, h->num_docs, batch, h->num_docs, k, nullptr, false, out_scores, out_ids, s);
  });
}
