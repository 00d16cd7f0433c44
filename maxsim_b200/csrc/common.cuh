// Shared device/host definitions for the maxsim_b200 CUDA library (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

namespace msb {

// ---------------------------------------------------------------------------
// Formats, query modes and reducers (names follow the reference SDK).
// ---------------------------------------------------------------------------
enum DocFormat : int { kFormatInt4 = 0, kFormatBinary = 1 };
enum QueryMode : int { kQueryF32 = 0, kQueryI8 = 1 };
enum Reducer : int { kMaxSim = 0, kWeighted = 1, kTopK2 = 2, kTopK4 = 3, kSmooth = 4 };

constexpr float kLowest = -3.402823466e+38F;

// Error raised by host-side validation; mapped to MSB_ERR_INVALID_ARGUMENT.
struct InvalidArgument : std::runtime_error {
  explicit InvalidArgument(const std::string& m) : std::runtime_error(m) {}
};
struct NotSupported : std::runtime_error {
  explicit NotSupported(const std::string& m) : std::runtime_error(m) {}
};
// CUDA failure; mapped to MSB_ERR_CUDA.
struct CudaFailure : std::runtime_error {
  explicit CudaFailure(const std::string& m) : std::runtime_error(m) {}
};

inline void check(cudaError_t st, const char* what) {
  if (st != cudaSuccess) throw CudaFailure(std::string(what) + ": " + cudaGetErrorString(st));
}

// Counts every kernel this library launches (reported by bench.py as
// gpu_launches; the driver cross-checks it against its own evidence).
void count_launch(int n = 1);

// ---------------------------------------------------------------------------
// Device-side description of one resident corpus and one scan request.
// ---------------------------------------------------------------------------
struct DocsView {
  const uint8_t* codes;        // [N, bytes_per_token]: int4 nibbles (dim/2 B) or sign bits (dim/8 B)
  const float* token_scale;    // [N] or nullptr
  const uint8_t* codes2;       // residual int4 stream [N, dim/2] or nullptr
  const float* token_scale2;   // residual token scales [N]
  const int64_t* offsets;      // [D + 1]
  const float* doc_scale;      // [D] or nullptr (binary scale vector)
  const int64_t* host_offsets;  // host copy of offsets (work partitioning)
  uint64_t corpus_id;          // unique per resident corpus (keys host-side caches)
  const uint8_t* codes8;       // int4 codes expanded to int8 in scan K order [N, 128], or nullptr
  const uint16_t* codes16;     // the same as f16 values [N, 128], or nullptr (tensor-core f16 operands)
  const uint8_t* codes2_8;     // the residual stream expanded to int8 like codes8, or nullptr
  int64_t num_docs;
  int64_t num_tokens;
  int dim;
  int format;
  float scale;                 // int4 tensor scale or binary scalar doc scale
  float scale2;                // residual tensor scale
  int token_scale_small;       // every finite token scale is below 2^104 in magnitude (s * 2^23 is exact)
};

struct QueryView {
  const float* f32;            // [B, Q, dim]
  const int8_t* i8;            // [B*Q, dim] natural order (int8 mode)
  const int32_t* i8_words;     // [B*Q, dim/4] packed words in scan order (int8 mode)
  const float* row_scale;      // [B*Q] (int8 mode)
  const int32_t* row_sum;      // [B*Q] sum of codes (binary int8 mode)
  int batch;
  int qtok;
  int mode;
};

struct ReduceView {
  int reducer;
  const float* weights;        // [Q] or [B, Q] (weighted MaxSim)
  int weights_batched;
  float temperature;
};

struct TargetsView {
  const int64_t* ids;          // [T] shared list, or [B, T] per-row lists, or nullptr (all docs)
  int64_t count;               // T
  int per_row;                 // ids is [B, T]
};

// Fused per-query top-k of a tensor-core full scan: each CTA keeps the k best documents of every query in
// shared memory and writes them as one candidate block; a merge kernel forms the final [B, k].
struct TopkFuse {
  int k;                        // top-k per query row
  void* cand;                   // candidate blocks, 16 * B * k bytes each (device workspace)
  size_t cand_bytes;
  const int64_t* empty_ids;     // the corpus's first empty documents (score 0, never in a tile), device
  int n_empty;                  // how many of them (at most k are used)
  float* out_s;                 // [B, k] results (device)
  int64_t* out_i;
  bool done;                    // set when the fused path ran (otherwise the caller selects from scores)
};

// ---------------------------------------------------------------------------
// Small device helpers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t float_to_ordered(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ordered_to_float(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(u);
}

}  // namespace msb
