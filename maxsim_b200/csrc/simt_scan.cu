// SIMT scan engine: every format x query mode x reducer, any dim (dim % 8 == 0).
//
// This engine is the general path: odd dims, queries of more than 32 tokens
// with fp32 values, SmoothSim (and TopK of the residual streams), candidate
// lists naming fewer than one document in 16.  Dim-128 MaxSim, weighted
// MaxSim and TopK full scans (int8 queries, fp32 queries as digit planes, the
// fused residual streams), and the longer candidate lists gathered from them,
// run on the tcgen05 engine (tc_scan.cu).
//
// Semantics follow the reference kernels:
//   int4 fp32     cpp/maxsim/cuda_extension.cu:1268-1323 and :757-844
//   int4 int8     cpp/maxsim/cuda_extension.cu:1494-1627 (exact int32 dot,
//                 per-token scale applied before the maximum)
//   binary fp32   cpp/maxsim/cuda_extension.cu:237-250, :297-352
//   binary int8   cpp/maxsim/cuda_extension.cu:1365-1449 (sum of +-q)
//   residual      cpp/maxsim/cuda_extension.cu:1045-1137
//   reducers      cpp/maxsim/cuda_extension.cu:477-653
// Layout of the work: one 128-thread block per (target, batch row); block
// index = target * B + row so the B blocks that read one document run
// back-to-back and share it through L2.  Warps own query rows, lanes stride
// the document's tokens, lanes merge with shuffles, and the per-row values
// are summed in query-row order by one thread (deterministic).
#include "common.cuh"

namespace msb {

// ---------------------------------------------------------------------------
// Reducer policies
// ---------------------------------------------------------------------------
template <int R>
struct Red;

template <>
struct Red<kMaxSim> {
  struct S { float best; int count; };
  static constexpr bool kScaleFirst = false;
  __device__ static S init() { return {kLowest, 0}; }
  __device__ static void add(S& s, float v, float) {
    s.best = (s.count == 0 || v > s.best) ? v : s.best;
    ++s.count;
  }
  __device__ static S merge(S a, S b, float) {
    if (a.count == 0) return b;
    if (b.count == 0) return a;
    a.best = b.best > a.best ? b.best : a.best;
    a.count += b.count;
    return a;
  }
  __device__ static S shfl(S s, int delta) {
    s.best = __shfl_down_sync(0xFFFFFFFFu, s.best, delta);
    s.count = __shfl_down_sync(0xFFFFFFFFu, s.count, delta);
    return s;
  }
  __device__ static float finish(S s, float w, float) { return s.count == 0 ? 0.0F : s.best * w; }
};

template <>
struct Red<kWeighted> : Red<kMaxSim> {};

template <int K>
struct RedTopK {
  struct S { float v[K]; int count; };
  static constexpr bool kScaleFirst = false;
  __device__ static S init() {
    S s;
#pragma unroll
    for (int i = 0; i < K; ++i) s.v[i] = kLowest;
    s.count = 0;
    return s;
  }
  __device__ static void add(S& s, float x, float) {
    // Insertion into a descending register list with fixed indices.
#pragma unroll
    for (int i = 0; i < K; ++i) {
      float cur = s.v[i];
      bool take = x > cur;
      s.v[i] = take ? x : cur;
      x = take ? cur : x;
    }
    s.count = s.count < K ? s.count + 1 : K;
  }
  __device__ static S merge(S a, S b, float t) {
#pragma unroll
    for (int i = 0; i < K; ++i)
      if (i < b.count) add(a, b.v[i], t);
    return a;
  }
  __device__ static S shfl(S s, int delta) {
#pragma unroll
    for (int i = 0; i < K; ++i) s.v[i] = __shfl_down_sync(0xFFFFFFFFu, s.v[i], delta);
    s.count = __shfl_down_sync(0xFFFFFFFFu, s.count, delta);
    return s;
  }
  __device__ static float finish(S s, float, float) {
    if (s.count == 0) return 0.0F;
    float total = 0.0F;
#pragma unroll
    for (int i = 0; i < K; ++i)
      if (i < s.count) total += s.v[i];
    return total / static_cast<float>(s.count);
  }
};
template <>
struct Red<kTopK2> : RedTopK<2> {};
template <>
struct Red<kTopK4> : RedTopK<4> {};

template <>
struct Red<kSmooth> {
  // Online log-sum-exp: maximum and sum of exp((v - max) / t).
  struct S { float m; float sum; };
  static constexpr bool kScaleFirst = true;
  __device__ static S init() { return {kLowest, 0.0F}; }
  __device__ static void add(S& s, float v, float t) {
    if (s.sum == 0.0F) { s.m = v; s.sum = 1.0F; return; }
    if (v == s.m) {
      s.sum += 1.0F;
    } else if (v < s.m) {
      s.sum += expf((v - s.m) / t);
    } else {
      s.sum = s.sum * expf((s.m - v) / t) + 1.0F;
      s.m = v;
    }
  }
  __device__ static S merge(S a, S b, float t) {
    if (a.sum == 0.0F) return b;
    if (b.sum == 0.0F) return a;
    if (a.m == b.m) {
      a.sum += b.sum;
    } else if (b.m < a.m) {
      a.sum += b.sum * expf((b.m - a.m) / t);
    } else {
      a.sum = a.sum * expf((a.m - b.m) / t) + b.sum;
      a.m = b.m;
    }
    return a;
  }
  __device__ static S shfl(S s, int delta) {
    s.m = __shfl_down_sync(0xFFFFFFFFu, s.m, delta);
    s.sum = __shfl_down_sync(0xFFFFFFFFu, s.sum, delta);
    return s;
  }
  __device__ static float finish(S s, float, float t) { return s.sum == 0.0F ? 0.0F : s.m + t * logf(s.sum); }
};

// ---------------------------------------------------------------------------
// Per-token dot products
// ---------------------------------------------------------------------------
// int4 nibbles -> fp32 dot in dimension order.
__device__ __forceinline__ float dot_int4_f32(const float* __restrict__ q, const uint8_t* __restrict__ row,
                                              int dim) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(row);
  float acc = 0.0F;
  for (int i = 0; i < dim / 8; ++i) {
    uint32_t word = __ldg(w + i);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int nib = static_cast<int>((word >> (4 * j)) & 0xFu);
      nib = nib >= 8 ? nib - 16 : nib;
      acc = fmaf(static_cast<float>(nib), __ldg(q + 8 * i + j), acc);
    }
  }
  return acc;
}

// Sign-extend the four low (or high) nibbles of a word into four int8 lanes.
__device__ __forceinline__ int32_t nibbles_lo_s8(uint32_t w) {
  return static_cast<int32_t>((w & 0x0F0F0F0Fu) | ((w & 0x08080808u) * 0x1Eu));
}
__device__ __forceinline__ int32_t nibbles_hi_s8(uint32_t w) { return nibbles_lo_s8(w >> 4); }

// int4 x int8: query words are stored pair-wise per 8 dims: word 2i holds the
// even dims 8i,8i+2,8i+4,8i+6 and word 2i+1 the odd dims (nibble order).
__device__ __forceinline__ int dot_int4_i8(const int32_t* __restrict__ qw, const uint8_t* __restrict__ row,
                                           int dim) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(row);
  int acc = 0;
  for (int i = 0; i < dim / 8; ++i) {
    uint32_t word = __ldg(w + i);
    acc = __dp4a(nibbles_lo_s8(word), __ldg(qw + 2 * i), acc);
    acc = __dp4a(nibbles_hi_s8(word), __ldg(qw + 2 * i + 1), acc);
  }
  return acc;
}

// Binary x fp32: sum of +-q in dimension order.
__device__ __forceinline__ float dot_bin_f32(const float* __restrict__ q, const uint8_t* __restrict__ row,
                                             int dim) {
  float acc = 0.0F;
  for (int i = 0; i < dim / 8; ++i) {
    uint32_t byte = __ldg(row + i);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float v = __ldg(q + 8 * i + j);
      acc += ((byte >> j) & 1u) ? v : -v;
    }
  }
  return acc;
}

// Spread the 4 bits of a nibble into the low bit of 4 bytes.
__device__ __forceinline__ int32_t spread_nibble(uint32_t n) {
  return static_cast<int32_t>((n * 0x00204081u) & 0x01010101u);
}

// Binary x int8: 2 * (sum of q over set bits) - sum(q); words in dim order.
__device__ __forceinline__ int dot_bin_i8(const int32_t* __restrict__ qw, int32_t qsum,
                                          const uint8_t* __restrict__ row, int dim) {
  int acc = 0;
  for (int i = 0; i < dim / 8; ++i) {
    uint32_t byte = __ldg(row + i);
    acc = __dp4a(spread_nibble(byte & 0xFu), __ldg(qw + 2 * i), acc);
    acc = __dp4a(spread_nibble(byte >> 4), __ldg(qw + 2 * i + 1), acc);
  }
  return 2 * acc - qsum;
}

// Format selector for the kernel template.
// kKindResidual: int4 prefix + int4 residual; kKindResidualBinary: sign-bit prefix (scaled by its per-token
// reconstruction scale) + int4 residual.
enum ScanKind : int { kKindInt4 = 0, kKindBinary = 1, kKindResidual = 2, kKindResidualBinary = 3 };

template <int Kind, int Mode, int R>
__global__ void __launch_bounds__(128) simt_scan_kernel(DocsView docs, QueryView qv, ReduceView red,
                                                        TargetsView tg, float* __restrict__ out) {
  using P = Red<R>;
  extern __shared__ float row_value[];  // [Q]
  const int B = qv.batch;
  const int Q = qv.qtok;
  const int64_t blk = blockIdx.x;
  const int b = static_cast<int>(blk % B);
  const int64_t j = blk / B;
  const int64_t T = tg.ids ? tg.count : docs.num_docs;
  const int64_t d = tg.ids ? (tg.per_row ? tg.ids[static_cast<int64_t>(b) * T + j] : tg.ids[j]) : j;
  const int64_t start = docs.offsets[d];
  const int64_t end = docs.offsets[d + 1];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int dim = docs.dim;

  float doc_scale = 1.0F;
  if (Kind == kKindInt4) doc_scale = docs.scale;
  if (Kind == kKindBinary) doc_scale = docs.doc_scale ? docs.doc_scale[d] : docs.scale;

  const int bytes_per_token = (Kind == kKindBinary || Kind == kKindResidualBinary) ? dim / 8 : dim / 2;
  for (int r = warp; r < Q; r += 4) {
    const int64_t row = static_cast<int64_t>(b) * Q + r;
    typename P::S st = P::init();
    for (int64_t t = start + lane; t < end; t += 32) {
      const uint8_t* code = docs.codes + t * bytes_per_token;
      float sim;
      if (Kind == kKindResidual) {
        const float* qf = qv.f32 + row * dim;
        float d1 = dot_int4_f32(qf, code, dim);
        float d2 = dot_int4_f32(qf, docs.codes2 + t * bytes_per_token, dim);
        float s1 = docs.token_scale ? docs.token_scale[t] : 1.0F;
        sim = d1 * docs.scale * s1 + d2 * docs.scale2 * docs.token_scale2[t];
      } else if (Kind == kKindResidualBinary) {
        const float* qf = qv.f32 + row * dim;
        const float d1 = dot_bin_f32(qf, code, dim);                                     // sum of +-q
        const float d2 = dot_int4_f32(qf, docs.codes2 + t * static_cast<int64_t>(dim / 2), dim);
        sim = d1 * docs.token_scale[t] + d2 * docs.scale2 * docs.token_scale2[t];
      } else {
        if (Mode == kQueryI8) {
          const int32_t* qw = qv.i8_words + row * (dim / 4);
          int idot = (Kind == kKindInt4) ? dot_int4_i8(qw, code, dim) : dot_bin_i8(qw, qv.row_sum[row], code, dim);
          sim = static_cast<float>(idot);
        } else {
          const float* qf = qv.f32 + row * dim;
          sim = (Kind == kKindInt4) ? dot_int4_f32(qf, code, dim) : dot_bin_f32(qf, code, dim);
        }
        if (docs.token_scale) sim *= docs.token_scale[t];
        if (P::kScaleFirst) sim *= doc_scale;
      }
      P::add(st, sim, red.temperature);
    }
#pragma unroll
    for (int delta = 16; delta > 0; delta >>= 1) {
      typename P::S other = P::shfl(st, delta);
      if (lane < delta) st = P::merge(st, other, red.temperature);
    }
    if (lane == 0) {
      float w = 1.0F;
      if (R == kWeighted) w = red.weights[(red.weights_batched ? static_cast<int64_t>(b) * Q : 0) + r];
      if (Mode == kQueryI8) w = qv.row_scale[row];
      row_value[r] = P::finish(st, w, red.temperature);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float acc = 0.0F;
    for (int r = 0; r < Q; ++r) acc += row_value[r];
    if (!P::kScaleFirst && Kind != kKindResidual && Kind != kKindResidualBinary) acc *= doc_scale;
    out[static_cast<int64_t>(b) * T + j] = acc;
  }
}

// ---------------------------------------------------------------------------
// Binary codes x fp32 queries at dim 128: nibble tables.  The sign dot of one query row with one token is
// sum over the 32 nibbles p of L[p][n_p], where L[p][v] = sum_{j<4} (bit j of v ? +q : -q)[4p + j] and n_p
// is the token's nibble p (dims 4p..4p+3: bits of byte (4p)/8, LSB first).  A block builds the tables of
// its query's rows once in shared memory (2 KB per row) and scans kLutDocs documents with them: 32
// conflict-free table reads and adds per (row, token) instead of 128 loads, selects and adds.  Each
// thread loads a token's 16 code bytes once per group of kLutRows query rows.  The per-row sum order is
// nibble-wise (the reference adds dims in order), within the fp32 paths' tolerance.
// ---------------------------------------------------------------------------
constexpr int kLutDocs = 16;
constexpr int kLutRows = 8;
constexpr int kLutMaxQ = 48;

template <int R>
__global__ void __launch_bounds__(128) bin_lut_scan_kernel(DocsView docs, QueryView qv, ReduceView red,
                                                           TargetsView tg, float* __restrict__ out) {
  using P = Red<R>;
  using S = typename P::S;
  extern __shared__ __align__(16) float lut_smem[];
  const int Q = qv.qtok;
  float* lut = lut_smem;                  // [Q][32][16]
  float* row_value = lut + Q * 512;       // [Q]
  S* part = reinterpret_cast<S*>(row_value + ((Q + 3) & ~3));  // [4 warps][kLutRows]
  const int b = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t T = tg.ids ? tg.count : docs.num_docs;
  for (int e = threadIdx.x; e < Q * 512; e += blockDim.x) {
    const int r = e >> 9, pos = (e >> 4) & 31, v = e & 15;
    const float* qr = qv.f32 + (static_cast<int64_t>(b) * Q + r) * 128 + 4 * pos;
    float acc = 0.0F;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc += ((v >> j) & 1) ? qr[j] : -qr[j];
    lut[e] = acc;
  }
  __syncthreads();
  const int64_t j_end = min(T, static_cast<int64_t>(blockIdx.x + 1) * kLutDocs);
  for (int64_t j = static_cast<int64_t>(blockIdx.x) * kLutDocs; j < j_end; ++j) {
    const int64_t d = tg.ids ? (tg.per_row ? tg.ids[static_cast<int64_t>(b) * T + j] : tg.ids[j]) : j;
    const int64_t start = docs.offsets[d];
    const int64_t end = docs.offsets[d + 1];
    const float doc_scale = docs.doc_scale ? docs.doc_scale[d] : docs.scale;
    for (int r0 = 0; r0 < Q; r0 += kLutRows) {
      S st[kLutRows];
#pragma unroll
      for (int g = 0; g < kLutRows; ++g) st[g] = P::init();
      for (int64_t t = start + threadIdx.x; t < end; t += blockDim.x) {
        const uint4 c = __ldg(reinterpret_cast<const uint4*>(docs.codes + t * 16));
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
        const float ts = docs.token_scale ? docs.token_scale[t] : 1.0F;
#pragma unroll
        for (int g = 0; g < kLutRows; ++g) {
          if (r0 + g < Q) {
            const float* L = lut + (r0 + g) * 512;
            float s0 = 0.0F, s1 = 0.0F;
#pragma unroll
            for (int pos = 0; pos < 32; pos += 2) {
              s0 += L[16 * pos + ((w[pos >> 3] >> (4 * (pos & 7))) & 15u)];
              s1 += L[16 * (pos + 1) + ((w[pos >> 3] >> (4 * ((pos + 1) & 7))) & 15u)];
            }
            float sim = s0 + s1;
            if (docs.token_scale) sim *= ts;
            if (P::kScaleFirst) sim *= doc_scale;
            P::add(st[g], sim, red.temperature);
          }
        }
      }
#pragma unroll
      for (int g = 0; g < kLutRows; ++g) {
#pragma unroll
        for (int delta = 16; delta > 0; delta >>= 1) {
          const S other = P::shfl(st[g], delta);
          if (lane < delta) st[g] = P::merge(st[g], other, red.temperature);
        }
        if (lane == 0) part[warp * kLutRows + g] = st[g];
      }
      __syncthreads();
      if (threadIdx.x < kLutRows && r0 + threadIdx.x < Q) {
        const int r = r0 + threadIdx.x;
        S acc = part[threadIdx.x];
        for (int w2 = 1; w2 < 4; ++w2) acc = P::merge(acc, part[w2 * kLutRows + threadIdx.x], red.temperature);
        float wt = 1.0F;
        if (R == kWeighted) wt = red.weights[(red.weights_batched ? static_cast<int64_t>(b) * Q : 0) + r];
        row_value[r] = P::finish(acc, wt, red.temperature);
      }
      __syncthreads();
    }
    if (threadIdx.x == 0) {
      float acc = 0.0F;
      for (int r = 0; r < Q; ++r) acc += row_value[r];
      if (!P::kScaleFirst) acc *= doc_scale;
      out[static_cast<int64_t>(b) * T + j] = acc;
    }
    __syncthreads();
  }
}

template <int R>
static void launch_bin_lut(const DocsView& docs, const QueryView& qv, const ReduceView& red, const TargetsView& tg,
                           float* out, cudaStream_t stream) {
  const int64_t T = tg.ids ? tg.count : docs.num_docs;
  const int64_t gx = (T + kLutDocs - 1) / kLutDocs;
  if (gx == 0 || qv.batch == 0) return;
  const int Q = qv.qtok;
  const size_t smem = sizeof(float) * (static_cast<size_t>(Q) * 512 + ((Q + 3) & ~3)) +
                      sizeof(typename Red<R>::S) * 4 * kLutRows;
  // a per-device function attribute: set on every launch (cheap), so every device a process uses has it
  check(cudaFuncSetAttribute(bin_lut_scan_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)),
        "set binary table scan shared memory");
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(qv.batch));
  bin_lut_scan_kernel<R><<<grid, 128, smem, stream>>>(docs, qv, red, tg, out);
  count_launch();
  check(cudaGetLastError(), "launch binary table scan kernel");
}

// ---------------------------------------------------------------------------
// int4 codes (and the int4 residual stream) x fp32 queries at dim 128: register-blocked rows.
// One warp per (target, query): its lanes stride the document's tokens, RG query rows at a time.  A
// lane converts the 8 nibbles of a code word to floats once (exactly: the bits 0x4B000000 | (nibble ^ 8)
// are the float 2^23 + value + 8) and feeds them to the RG rows' FMA chains, the group's query values
// staged in shared memory and read as broadcasts.  Each row's chain runs over the dims in order like
// dot_int4_f32, so the values are bit-identical to the general kernel's.  The warp merges its lanes with
// shuffles and lane 0 adds the row values in row order.  Single-warp blocks (tens of thousands for a
// full scan) let the block scheduler balance documents of different lengths across the SMs.
// ---------------------------------------------------------------------------
template <int R, bool kRes, int RG>
__global__ void __launch_bounds__(32) int4_rows_scan_kernel(DocsView docs, QueryView qv, ReduceView red,
                                                            TargetsView tg, float* __restrict__ out) {
  using P = Red<R>;
  using S = typename P::S;
  __shared__ __align__(16) float qs[RG * 128];
  const int Q = qv.qtok;
  const int lane = threadIdx.x;
  const int b = blockIdx.y;
  const int64_t j = blockIdx.x;
  const int64_t T = tg.ids ? tg.count : docs.num_docs;
  const int64_t d = tg.ids ? (tg.per_row ? tg.ids[static_cast<int64_t>(b) * T + j] : tg.ids[j]) : j;
  const int64_t start = docs.offsets[d];
  const int64_t end = docs.offsets[d + 1];
  const float4* qsrc = reinterpret_cast<const float4*>(qv.f32 + static_cast<int64_t>(b) * Q * 128);
  float total = 0.0F;
  for (int r0 = 0; r0 < Q; r0 += RG) {
    __syncwarp();  // the previous group's readers are done
#pragma unroll
    for (int e = lane; e < RG * 32; e += 32) {
      const int r = r0 + (e >> 5);
      reinterpret_cast<float4*>(qs)[e] = r < Q ? __ldg(qsrc + static_cast<int64_t>(r0) * 32 + e) : make_float4(0, 0, 0, 0);
    }
    __syncwarp();
    S st[RG];
#pragma unroll
    for (int g = 0; g < RG; ++g) st[g] = P::init();
    for (int64_t t = start + lane; t < end; t += 32) {
      float dot[2][RG];
#pragma unroll
      for (int pass = 0; pass < (kRes ? 2 : 1); ++pass) {
        const uint4* src = reinterpret_cast<const uint4*>((pass == 0 ? docs.codes : docs.codes2) + t * 64);
        float acc[RG];
#pragma unroll
        for (int g = 0; g < RG; ++g) acc[g] = 0.0F;
#pragma unroll
        for (int v4 = 0; v4 < 4; ++v4) {
          const uint4 cv = __ldg(src + v4);
          const uint32_t wv[4] = {cv.x ^ 0x88888888u, cv.y ^ 0x88888888u, cv.z ^ 0x88888888u, cv.w ^ 0x88888888u};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int word = 4 * v4 + k;  // dims 8 word .. 8 word + 7; nibble n is dim 8 word + n
            float val[8];
#pragma unroll
            for (int n = 0; n < 8; ++n)
              val[n] = __int_as_float(static_cast<int>(((wv[k] >> (4 * n)) & 15u) | 0x4B000000u)) - 8388616.0F;
#pragma unroll
            for (int g = 0; g < RG; ++g) {
              const float4 qa = *reinterpret_cast<const float4*>(qs + g * 128 + 8 * word);
              const float4 qb = *reinterpret_cast<const float4*>(qs + g * 128 + 8 * word + 4);
              acc[g] = fmaf(val[0], qa.x, acc[g]);
              acc[g] = fmaf(val[1], qa.y, acc[g]);
              acc[g] = fmaf(val[2], qa.z, acc[g]);
              acc[g] = fmaf(val[3], qa.w, acc[g]);
              acc[g] = fmaf(val[4], qb.x, acc[g]);
              acc[g] = fmaf(val[5], qb.y, acc[g]);
              acc[g] = fmaf(val[6], qb.z, acc[g]);
              acc[g] = fmaf(val[7], qb.w, acc[g]);
            }
          }
        }
#pragma unroll
        for (int g = 0; g < RG; ++g) dot[pass][g] = acc[g];
      }
      const float ts = docs.token_scale ? docs.token_scale[t] : 1.0F;
      const float ts2 = kRes ? docs.token_scale2[t] : 0.0F;
#pragma unroll
      for (int g = 0; g < RG; ++g) {
        float sim;
        if (kRes) {
          sim = dot[0][g] * docs.scale * ts + dot[1][g] * docs.scale2 * ts2;
        } else {
          sim = dot[0][g];
          if (docs.token_scale) sim *= ts;
          if (P::kScaleFirst) sim *= docs.scale;
        }
        P::add(st[g], sim, red.temperature);
      }
    }
#pragma unroll
    for (int g = 0; g < RG; ++g) {
#pragma unroll
      for (int delta = 16; delta > 0; delta >>= 1) {
        const S other = P::shfl(st[g], delta);
        if (lane < delta) st[g] = P::merge(st[g], other, red.temperature);
      }
      const int r = r0 + g;
      if (r < Q) {
        float wt = 1.0F;
        if (R == kWeighted) wt = red.weights[(red.weights_batched ? static_cast<int64_t>(b) * Q : 0) + r];
        total += P::finish(st[g], wt, red.temperature);  // lane 0's value is the row's; rows in order
      }
    }
  }
  if (lane == 0) {
    if (!kRes && !P::kScaleFirst) total *= docs.scale;
    out[static_cast<int64_t>(b) * T + j] = total;
  }
}

template <int R, bool kRes>
static void launch_int4_lut(const DocsView& docs, const QueryView& qv, const ReduceView& red, const TargetsView& tg,
                            float* out, cudaStream_t stream) {
  // 16-row groups where the reducer state is one value and one stream is read; 8 for the top-k and smooth
  // states and for the two residual streams (whose 16-row form does not fit in registers)
  constexpr int RG = (!kRes && (R == kMaxSim || R == kWeighted)) ? 16 : 8;
  const int64_t T = tg.ids ? tg.count : docs.num_docs;
  if (T == 0 || qv.batch == 0) return;
  if (T > 0x7FFFFFFFLL) throw InvalidArgument("too many targets for one scan");
  dim3 grid(static_cast<unsigned>(T), static_cast<unsigned>(qv.batch));
  int4_rows_scan_kernel<R, kRes, RG><<<grid, 32, 0, stream>>>(docs, qv, red, tg, out);
  count_launch();
  check(cudaGetLastError(), "launch int4 row-blocked scan kernel");
}

template <bool kRes>
static void launch_int4_lut_reducer(const DocsView& docs, const QueryView& qv, const ReduceView& red,
                                    const TargetsView& tg, float* out, cudaStream_t stream) {
  switch (red.reducer) {
    case kMaxSim: launch_int4_lut<kMaxSim, kRes>(docs, qv, red, tg, out, stream); break;
    case kWeighted: launch_int4_lut<kWeighted, kRes>(docs, qv, red, tg, out, stream); break;
    case kTopK2: launch_int4_lut<kTopK2, kRes>(docs, qv, red, tg, out, stream); break;
    case kTopK4: launch_int4_lut<kTopK4, kRes>(docs, qv, red, tg, out, stream); break;
    case kSmooth: launch_int4_lut<kSmooth, kRes>(docs, qv, red, tg, out, stream); break;
    default: throw InvalidArgument("unknown reducer");
  }
}

template <int Kind, int Mode>
static void launch_kind_mode(const DocsView& docs, const QueryView& qv, const ReduceView& red, const TargetsView& tg,
                             float* out, cudaStream_t stream) {
  const int64_t T = tg.ids ? tg.count : docs.num_docs;
  const int64_t blocks = T * qv.batch;
  if (blocks == 0) return;
  if (blocks > 0x7FFFFFFFLL) throw InvalidArgument("scan grid too large (targets x batch exceeds 2^31)");
  const size_t smem = sizeof(float) * static_cast<size_t>(qv.qtok);
  if (smem > 48 * 1024) throw NotSupported("query_tokens above 12288 are not supported");
  dim3 grid(static_cast<unsigned>(blocks));
  switch (red.reducer) {
    case kMaxSim: simt_scan_kernel<Kind, Mode, kMaxSim><<<grid, 128, smem, stream>>>(docs, qv, red, tg, out); break;
    case kWeighted: simt_scan_kernel<Kind, Mode, kWeighted><<<grid, 128, smem, stream>>>(docs, qv, red, tg, out); break;
    case kTopK2: simt_scan_kernel<Kind, Mode, kTopK2><<<grid, 128, smem, stream>>>(docs, qv, red, tg, out); break;
    case kTopK4: simt_scan_kernel<Kind, Mode, kTopK4><<<grid, 128, smem, stream>>>(docs, qv, red, tg, out); break;
    case kSmooth: simt_scan_kernel<Kind, Mode, kSmooth><<<grid, 128, smem, stream>>>(docs, qv, red, tg, out); break;
    default: throw InvalidArgument("unknown reducer");
  }
  count_launch();
  check(cudaGetLastError(), "launch SIMT scan kernel");
}

void launch_simt_scan(const DocsView& docs, const QueryView& qv, const ReduceView& red, const TargetsView& tg,
                      bool residual, float* out, cudaStream_t stream) {
  // (int4 row-blocked scan: dim 128; the query is read as float4, so a caller's device pointer must be
  // 16-byte aligned; codes are the handle's own allocations)
  const bool i4_lut = docs.dim == 128 && qv.qtok >= 1 && qv.batch <= 65535 &&
                      (reinterpret_cast<uintptr_t>(qv.f32) & 15) == 0;
  if (residual) {
    if (qv.mode != kQueryF32) throw InvalidArgument("residual scoring takes fp32 queries");
    if (docs.format == kFormatBinary) launch_kind_mode<kKindResidualBinary, kQueryF32>(docs, qv, red, tg, out, stream);
    else if (i4_lut) launch_int4_lut_reducer<true>(docs, qv, red, tg, out, stream);
    else launch_kind_mode<kKindResidual, kQueryF32>(docs, qv, red, tg, out, stream);
    return;
  }
  if (qv.mode == kQueryI8 && red.reducer != kMaxSim)
    throw InvalidArgument("int8 queries support reducer='maxsim' only");
  if (docs.format == kFormatInt4) {
    if (qv.mode == kQueryI8) launch_kind_mode<kKindInt4, kQueryI8>(docs, qv, red, tg, out, stream);
    else if (i4_lut) launch_int4_lut_reducer<false>(docs, qv, red, tg, out, stream);
    else launch_kind_mode<kKindInt4, kQueryF32>(docs, qv, red, tg, out, stream);
  } else if (qv.mode == kQueryF32 && docs.dim == 128 && qv.qtok >= 1 && qv.qtok <= kLutMaxQ && qv.batch <= 65535) {
    switch (red.reducer) {
      case kMaxSim: launch_bin_lut<kMaxSim>(docs, qv, red, tg, out, stream); break;
      case kWeighted: launch_bin_lut<kWeighted>(docs, qv, red, tg, out, stream); break;
      case kTopK2: launch_bin_lut<kTopK2>(docs, qv, red, tg, out, stream); break;
      case kTopK4: launch_bin_lut<kTopK4>(docs, qv, red, tg, out, stream); break;
      case kSmooth: launch_bin_lut<kSmooth>(docs, qv, red, tg, out, stream); break;
      default: throw InvalidArgument("unknown reducer");
    }
  } else {
    if (qv.mode == kQueryI8) launch_kind_mode<kKindBinary, kQueryI8>(docs, qv, red, tg, out, stream);
    else launch_kind_mode<kKindBinary, kQueryF32>(docs, qv, red, tg, out, stream);
  }
}

// ---------------------------------------------------------------------------
// Query quantisation (kernel formula of cpp/maxsim/cuda_extension.cu:1455-1492)
// ---------------------------------------------------------------------------
// One warp per row.  Emits natural-order int8 codes, the per-row scale, the
// code sum (binary identity) and packed words in the order the chosen dot
// product consumes: nibble order (even dims, odd dims per 8) for int4 docs or
// natural order for binary docs.
__global__ void quantize_rows_kernel(const float* __restrict__ q, int64_t rows, int dim, int8_t* __restrict__ codes,
                                     float* __restrict__ scales, int32_t* __restrict__ sums,
                                     int32_t* __restrict__ words, int nibble_order) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* x = q + row * dim;
  float m = 0.0F;
  for (int i = lane; i < dim; i += 32) m = fmaxf(m, fabsf(x[i]));
#pragma unroll
  for (int delta = 16; delta > 0; delta >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, delta));
  const float s = (m == 0.0F) ? 1.0F : __fdiv_rn(m, 127.0F);
  const float inv = __fdiv_rn(1.0F, s);
  int partial = 0;
  int8_t* c = codes + row * dim;
  for (int i = lane; i < dim; i += 32) {
    int v = __float2int_rn(__fmul_rn(x[i], inv));
    v = v > 127 ? 127 : (v < -127 ? -127 : v);
    c[i] = static_cast<int8_t>(v);
    partial += v;
  }
#pragma unroll
  for (int delta = 16; delta > 0; delta >>= 1) partial += __shfl_xor_sync(0xFFFFFFFFu, partial, delta);
  if (lane == 0) {
    scales[row] = s;
    if (sums) sums[row] = partial;
  }
  __syncwarp();
  if (words) {
    int32_t* w = words + row * (dim / 4);
    for (int g = lane; g < dim / 8; g += 32) {
      uint32_t a = 0, bword = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        int i0 = nibble_order ? 8 * g + 2 * k : 8 * g + k;
        int i1 = nibble_order ? 8 * g + 2 * k + 1 : 8 * g + 4 + k;
        a |= (static_cast<uint32_t>(static_cast<uint8_t>(c[i0]))) << (8 * k);
        bword |= (static_cast<uint32_t>(static_cast<uint8_t>(c[i1]))) << (8 * k);
      }
      w[2 * g] = static_cast<int32_t>(a);
      w[2 * g + 1] = static_cast<int32_t>(bword);
    }
  }
}

void launch_quantize_rows(const float* q, int64_t rows, int dim, int8_t* codes, float* scales, int32_t* sums,
                          int32_t* words, bool nibble_order, cudaStream_t stream) {
  if (rows <= 0) return;
  const int64_t threads = rows * 32;
  const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
  quantize_rows_kernel<<<blocks, 256, 0, stream>>>(q, rows, dim, codes, scales, sums, words, nibble_order ? 1 : 0);
  count_launch();
  check(cudaGetLastError(), "launch query quantisation kernel");
}

}  // namespace msb
