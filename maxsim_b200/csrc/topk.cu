// Row-wise top-k selection: score descending, ties to the lower id.
//
// Tie policy of the reference: cpp/maxsim/cuda_extension.cu:1629-1692 and
// src/maxsim/_api.py:732-735 (lexsort by (-score, id)); with explicit tie ids
// it is src/maxsim/cascade.py:436-453 (ties broken by candidate doc id).
//
// Two paths, one block of 1024 threads per row:
//   * small rows (T <= kSortCap): bitonic sort of (ordered key, tie id) in
//     shared memory -- used for candidate lists, shard merges and short rows;
//   * long rows: 4-pass 8-bit radix select of the k-th largest ordered key,
//     then collection of everything above it plus the lowest-index ties, and
//     a bitonic sort of the k survivors.
#include <algorithm>

#include "common.cuh"

namespace msb {

constexpr int kTopkThreads = 1024;
constexpr int kSortCap = 4096;

// Sort (composite descending, then payload) pairs held in shared memory.
__device__ void bitonic_sort_desc(uint64_t* key, uint32_t* pos, int n_pow2) {
  for (int size = 2; size <= n_pow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < n_pow2; i += blockDim.x) {
        int partner = i ^ stride;
        if (partner > i) {
          bool descending = (i & size) == 0;
          uint64_t a = key[i], b = key[partner];
          bool swap = descending ? (a < b) : (a > b);
          if (swap) {
            key[i] = b;
            key[partner] = a;
            uint32_t t = pos[i];
            pos[i] = pos[partner];
            pos[partner] = t;
          }
        }
      }
      __syncthreads();
    }
  }
}

__device__ __forceinline__ uint64_t composite(uint32_t okey, uint32_t tie) {
  return (static_cast<uint64_t>(okey) << 32) | static_cast<uint64_t>(0xFFFFFFFFu - tie);
}

__global__ void __launch_bounds__(kTopkThreads) topk_sort_kernel(const float* __restrict__ scores, int64_t ld,
                                                                  int64_t T, int k, const int64_t* __restrict__ tie_ids,
                                                                  int tie_batched, float* __restrict__ out_s,
                                                                  int64_t* __restrict__ out_id) {
  extern __shared__ unsigned char smem_raw[];
  int n = 1;
  while (n < T) n <<= 1;
  uint64_t* key = reinterpret_cast<uint64_t*>(smem_raw);
  uint32_t* pos = reinterpret_cast<uint32_t*>(key + n);
  const int row = blockIdx.x;
  const float* s = scores + static_cast<int64_t>(row) * ld;
  const int64_t* tie = tie_ids ? tie_ids + (tie_batched ? static_cast<int64_t>(row) * T : 0) : nullptr;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    if (i < T) {
      uint32_t t = tie ? static_cast<uint32_t>(tie[i]) : static_cast<uint32_t>(i);
      key[i] = composite(float_to_ordered(s[i]), t);
      pos[i] = static_cast<uint32_t>(i);
    } else {
      key[i] = 0;
      pos[i] = 0xFFFFFFFFu;
    }
  }
  __syncthreads();
  bitonic_sort_desc(key, pos, n);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    uint32_t p = pos[i];
    out_s[static_cast<int64_t>(row) * k + i] = s[p];
    out_id[static_cast<int64_t>(row) * k + i] = tie ? tie[p] : static_cast<int64_t>(p);
  }
}

// Block (row, c) selects the top k of targets [c * chunk, min(T, (c + 1) * chunk)) of its row.  One chunk per
// row (chunk >= T): the row's top-k into out_s / out_id.  Several chunks: each block writes its sorted list,
// with global target ids, as block c of `blocks` (16 * rows * k bytes per chunk: [rows, k] scores, then
// [rows, k] int64 ids), the layout merge_shard_topk_kernel merges.
__global__ void __launch_bounds__(kTopkThreads) topk_select_kernel(const float* __restrict__ scores, int64_t ld,
                                                                    int64_t T, int k, float* __restrict__ out_s,
                                                                    int64_t* __restrict__ out_id, int64_t chunk,
                                                                    unsigned char* __restrict__ blocks) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix, s_mask, s_remaining, s_taken, s_ties_taken;
  __shared__ uint32_t warp_count[kTopkThreads / 32];
  int n = 1;
  while (n < k) n <<= 1;
  uint64_t* key = reinterpret_cast<uint64_t*>(smem_raw);
  uint32_t* pos = reinterpret_cast<uint32_t*>(key + n);
  const int row = blockIdx.x;
  const int64_t start = static_cast<int64_t>(blockIdx.y) * chunk;
  const float* s = scores + static_cast<int64_t>(row) * ld + start;
  T = T - start < chunk ? T - start : chunk;  // this block's targets (at least k: the host sizes chunks)
  if (blocks) {
    const int64_t rows = gridDim.x;
    out_s = reinterpret_cast<float*>(blocks + static_cast<int64_t>(blockIdx.y) * 16 * rows * k);
    out_id = reinterpret_cast<int64_t*>(blocks + static_cast<int64_t>(blockIdx.y) * 16 * rows * k + 8 * rows * k);
  }

  if (threadIdx.x == 0) {
    s_prefix = 0;
    s_mask = 0;
    s_remaining = static_cast<uint32_t>(k);
    s_taken = 0;
    s_ties_taken = 0;
  }
  __syncthreads();
  // Radix select of the k-th largest ordered key, most significant byte first.
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
    for (int64_t i = threadIdx.x; i < T; i += blockDim.x) {
      uint32_t kk = float_to_ordered(s[i]);
      if ((kk & mask) == prefix) atomicAdd(&hist[(kk >> shift) & 0xFFu], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t need = s_remaining, acc = 0;
      int digit = 255;
      for (; digit > 0; --digit) {
        if (acc + hist[digit] >= need) break;
        acc += hist[digit];
      }
      s_prefix = prefix | (static_cast<uint32_t>(digit) << shift);
      s_mask = mask | (0xFFu << shift);
      s_remaining = need - acc;
    }
    __syncthreads();
  }
  const uint32_t kth = s_prefix;          // exact k-th largest ordered key
  const uint32_t ties_needed = s_remaining;  // how many elements equal to kth to keep
  // Collect strictly greater keys (at most k - ties_needed of them).
  for (int64_t i = threadIdx.x; i < T; i += blockDim.x) {
    uint32_t kk = float_to_ordered(s[i]);
    if (kk > kth) {
      uint32_t slot = atomicAdd(&s_taken, 1u);
      key[slot] = composite(kk, static_cast<uint32_t>(i));
      pos[slot] = static_cast<uint32_t>(i);
    }
  }
  __syncthreads();
  // Ties: keep the lowest indices, scanning chunks in index order.
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t base = 0; base < T; base += blockDim.x) {
    if (s_ties_taken >= ties_needed) break;
    const int64_t i = base + threadIdx.x;
    const bool tie = i < T && float_to_ordered(s[i]) == kth;
    const uint32_t ballot = __ballot_sync(0xFFFFFFFFu, tie);
    if (lane == 0) warp_count[warp] = __popc(ballot);
    __syncthreads();
    if (tie) {
      uint32_t before = s_ties_taken;
      for (int w = 0; w < warp; ++w) before += warp_count[w];
      before += __popc(ballot & ((1u << lane) - 1u));
      if (before < ties_needed) {
        uint32_t slot = s_taken + (before - s_ties_taken);
        key[slot] = composite(kth, static_cast<uint32_t>(i));
        pos[slot] = static_cast<uint32_t>(i);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t total = 0;
      for (int w = 0; w < kTopkThreads / 32; ++w) total += warp_count[w];
      uint32_t got = total < ties_needed - s_ties_taken ? total : ties_needed - s_ties_taken;
      s_taken += got;
      s_ties_taken += got;
    }
    __syncthreads();
  }
  for (int i = k + threadIdx.x; i < n; i += blockDim.x) {
    key[i] = 0;
    pos[i] = 0xFFFFFFFFu;
  }
  __syncthreads();
  bitonic_sort_desc(key, pos, n);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    uint32_t p = pos[i];
    out_s[static_cast<int64_t>(row) * k + i] = s[p];
    out_id[static_cast<int64_t>(row) * k + i] = start + static_cast<int64_t>(p);
  }
}

static int next_pow2(int64_t v) {
  int n = 1;
  while (n < v) n <<= 1;
  return n;
}

void launch_merge_shard_topk(const void* gathered, int world, int batch, int k, const int64_t* first_doc, float* out_s,
                             int64_t* out_id, cudaStream_t stream);

// Rows shorter than this are selected by one block each: below it the selection's fixed per-pass costs,
// not the row's length, set a block's time, and a second launch would only add to them.
constexpr int64_t kChunkedSelectMin = 32768;

// Chunks per row of a two-stage selection (1: one block per row), given the workspace it may use.
int select_chunks(int rows, int64_t T, int k, size_t ws_bytes) {
  if (T < kChunkedSelectMin) return 1;
  int64_t c = (T + 2047) / 2048;                              // about 2,048 targets a block
  c = std::min<int64_t>(c, std::max<int64_t>(1, 296 / rows));  // enough blocks for the SMs, no more
  c = std::min<int64_t>(c, std::min<int64_t>(64, T / k));
  // every chunk, the last one included, holds at least k targets; the lists fit the workspace
  while (c > 1 && (T - (c - 1) * ((T + c - 1) / c) < k || static_cast<size_t>(c) * 16 * rows * k > ws_bytes)) --c;
  return static_cast<int>(c);
}

size_t topk_rows_workspace_bytes(int rows, int64_t T, int k) {
  return T < kChunkedSelectMin ? 0 : static_cast<size_t>(64) * 16 * rows * k;
}

void launch_topk_rows(const float* scores, int64_t ld, int rows, int64_t T, int k, const int64_t* tie_ids,
                      bool tie_batched, float* out_s, int64_t* out_id, cudaStream_t stream, void* ws,
                      size_t ws_bytes) {
  if (rows <= 0) return;
  if (k < 1 || k > T) throw InvalidArgument("k must be between 1 and the number of targets");
  if (T > 0xFFFFFFF0LL) throw NotSupported("top-k rows longer than 2^32 - 16 are not supported");
  if (T <= kSortCap) {
    const size_t smem = static_cast<size_t>(next_pow2(T)) * (sizeof(uint64_t) + sizeof(uint32_t));
    topk_sort_kernel<<<rows, kTopkThreads, smem, stream>>>(scores, ld, T, k, tie_ids, tie_batched ? 1 : 0, out_s,
                                                            out_id);
    count_launch();
    check(cudaGetLastError(), "launch top-k sort kernel");
    return;
  }
  if (tie_ids) throw NotSupported("explicit tie ids are supported for rows of at most 4096 targets");
  if (k > 8192) throw NotSupported("k above 8192 is not supported for long rows");
  const size_t smem = static_cast<size_t>(next_pow2(k)) * (sizeof(uint64_t) + sizeof(uint32_t));
  if (smem > 48 * 1024) {
    check(cudaFuncSetAttribute(topk_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem)),
          "raise top-k shared memory limit");
  }
  // Few long rows: chunks of a row selected by separate blocks (rows x chunks), then merged
  const int chunks = ws ? select_chunks(rows, T, k, ws_bytes) : 1;
  if (chunks > 1) {
    const int64_t chunk = (T + chunks - 1) / chunks;
    topk_select_kernel<<<dim3(rows, chunks), kTopkThreads, smem, stream>>>(scores, ld, T, k, nullptr, nullptr, chunk,
                                                                             static_cast<unsigned char*>(ws));
    count_launch();
    check(cudaGetLastError(), "launch chunked top-k select kernel");
    launch_merge_shard_topk(ws, chunks, rows, k, nullptr, out_s, out_id, stream);
    return;
  }
  topk_select_kernel<<<rows, kTopkThreads, smem, stream>>>(scores, ld, T, k, out_s, out_id, T, nullptr);
  count_launch();
  check(cudaGetLastError(), "launch top-k select kernel");
}

// Merge of per-shard top-k lists (multi-GPU search).  `gathered` holds `world` blocks of 16 * batch * k
// bytes, one per rank in rank order, as one all-gather leaves them: the rank's [batch, k] fp32 scores at
// byte 0 of its block and its [batch, k] int64 local document ids at byte 8 * batch * k.  Each rank's
// row is ordered (score desc, id asc); global id = local id + first_doc[rank] (a local id of INT64_MAX
// pads a shard holding fewer than k documents and stays INT64_MAX).  One warp per query row repeats k
// times: every lane offers the best head among its ranks (lane, lane + 32, ...), a butterfly reduction
// picks the winner in the single-GPU order (ordered score key desc, global id asc), and the winning
// rank advances.  Shards are disjoint, so the result equals the top-k of the whole corpus.  first_doc may
// be null (the blocks already hold global ids: the fused top-k of the tensor-core scan).
constexpr int kMergeWarps = 4;
constexpr int kMergeMaxWorld = 1024;
__global__ void __launch_bounds__(kMergeWarps * 32) merge_shard_topk_kernel(
    const unsigned char* __restrict__ gathered, int world, int batch, int k, const int64_t* __restrict__ first_doc,
    float* __restrict__ out_s, int64_t* __restrict__ out_id) {
  __shared__ int pos_all[kMergeWarps][kMergeMaxWorld];
  const int wib = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kMergeWarps + wib;
  if (row >= batch) return;
  int* pos = pos_all[wib];
  for (int r = lane; r < world; r += 32) pos[r] = 0;
  __syncwarp();
  const size_t blk = 16ull * static_cast<size_t>(batch) * k;
  const size_t row_off = static_cast<size_t>(row) * k;
  auto head = [&](int r, uint32_t& key, int64_t& gid) {
    const int p = pos[r];
    const unsigned char* b = gathered + static_cast<size_t>(r) * blk;
    key = float_to_ordered(reinterpret_cast<const float*>(b)[row_off + p]);
    const int64_t lid = reinterpret_cast<const int64_t*>(b + 8ull * batch * k)[row_off + p];
    gid = lid == INT64_MAX ? INT64_MAX : lid + (first_doc ? first_doc[r] : 0);
  };
  for (int j = 0; j < k; ++j) {
    bool have = false;
    uint32_t bk = 0;
    int64_t bg = INT64_MAX;
    int br = -1;
    for (int r = lane; r < world; r += 32) {
      if (pos[r] >= k) continue;
      uint32_t key;
      int64_t gid;
      head(r, key, gid);
      if (!have || key > bk || (key == bk && gid < bg)) {
        have = true;
        bk = key;
        bg = gid;
        br = r;
      }
    }
#pragma unroll
    for (int delta = 16; delta > 0; delta >>= 1) {
      const int oh = __shfl_xor_sync(0xFFFFFFFFu, have ? 1 : 0, delta);
      const uint32_t ok = __shfl_xor_sync(0xFFFFFFFFu, bk, delta);
      const int64_t og = __shfl_xor_sync(0xFFFFFFFFu, bg, delta);
      const int orr = __shfl_xor_sync(0xFFFFFFFFu, br, delta);
      if (oh && (!have || ok > bk || (ok == bk && (og < bg || (og == bg && orr < br))))) {
        have = true;
        bk = ok;
        bg = og;
        br = orr;
      }
    }
    // every lane now holds the winner (ties between lanes resolved by rank, identically everywhere)
    if (lane == 0) {
      out_s[row_off + j] = have ? ordered_to_float(bk) : -INFINITY;
      out_id[row_off + j] = bg;
    }
    if (have && lane == (br & 31)) ++pos[br];
    __syncwarp();
  }
}

void launch_merge_shard_topk(const void* gathered, int world, int batch, int k, const int64_t* first_doc,
                             float* out_s, int64_t* out_id, cudaStream_t stream) {
  if (world < 1 || world > kMergeMaxWorld) throw InvalidArgument("world must be between 1 and 1024");
  if (k < 1) throw InvalidArgument("k must be >= 1");
  if (batch < 0) throw InvalidArgument("batch must be >= 0");
  if (batch == 0) return;
  const int blocks = (batch + kMergeWarps - 1) / kMergeWarps;
  merge_shard_topk_kernel<<<blocks, kMergeWarps * 32, 0, stream>>>(static_cast<const unsigned char*>(gathered), world,
                                                                   batch, k, first_doc, out_s, out_id);
  count_launch();
  check(cudaGetLastError(), "launch shard merge kernel");
}

// out[b, j] = scores[b, ids[j]] (shared list) or scores[b, ids[b * count + j]] (per-row lists): the scores
// of candidate lists read out of a full scan.
__global__ void gather_scores_kernel(const float* __restrict__ scores, int64_t ld, int rows,
                                     const int64_t* __restrict__ ids, int64_t count, int per_row,
                                     float* __restrict__ out) {
  const int64_t n = static_cast<int64_t>(rows) * count;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < n;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t b = e / count, j = e - b * count;
    out[e] = scores[b * ld + ids[per_row ? e : j]];
  }
}

// The empty documents' candidate block of a fused top-k: every query row gets the first min(k, n_empty)
// empty documents with score 0 (they never appear in a tile), the rest (-inf, INT64_MAX).
__global__ void empty_block_kernel(unsigned char* __restrict__ blk, int batch, int k, const int64_t* __restrict__ ids,
                                   int n_empty) {
  const int64_t n = static_cast<int64_t>(batch) * k;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < n;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(e % k);
    reinterpret_cast<float*>(blk)[e] = j < n_empty ? 0.0F : -INFINITY;
    reinterpret_cast<int64_t*>(blk + 8ull * n)[e] = j < n_empty ? ids[j] : INT64_MAX;
  }
}

void launch_empty_block(void* blk, int batch, int k, const int64_t* ids, int n_empty, cudaStream_t stream) {
  const int64_t n = static_cast<int64_t>(batch) * k;
  if (n == 0) return;
  empty_block_kernel<<<static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 1024)), 256, 0, stream>>>(
      static_cast<unsigned char*>(blk), batch, k, ids, n_empty);
  count_launch();
  check(cudaGetLastError(), "launch empty-document block kernel");
}

void launch_gather_scores(const float* scores, int64_t ld, int rows, const int64_t* ids, int64_t count, bool per_row,
                          float* out, cudaStream_t stream) {
  const int64_t n = static_cast<int64_t>(rows) * count;
  if (n <= 0) return;
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148LL * 8));
  gather_scores_kernel<<<blocks, 256, 0, stream>>>(scores, ld, rows, ids, count, per_row ? 1 : 0, out);
  count_launch();
  check(cudaGetLastError(), "launch candidate score gather kernel");
}

}  // namespace msb
