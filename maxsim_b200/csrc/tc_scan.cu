// Tensor-core (tcgen05) MaxSim scan for dim-128 corpora: int8 queries, and fp32 queries as int8 digit
// planes.
//
// D[query row, token] = sum_k A[row, k] * B[token, k] runs on the 5th-gen
// tensor cores (tcgen05.mma kind::i8, int32 accumulators in TMEM); the
// CUDA cores do the part the tensor core cannot: per-token scale before the
// maximum, the segmented (per document) maximum over ragged token ranges, and
// the sum over a query's rows.  Semantics are the reference kernel's
// (cpp/maxsim/cuda_extension.cu:1507-1627): exact int32 dot, fl(float(dot) *
// s_t), maximum per query row, doc += fl(best * qscale) in row order, * scale.
//
// Layout of the work
//   * A query tile is 128 TMEM lanes = floor(128 / Q) whole queries (Q rows
//     each); query rows are int8, K permuted to the nibble order of the codes.
//   * A work unit is (pair of query tiles, contiguous document range).  Each
//     token tile is loaded and expanded once and multiplied against both
//     query tiles, so loads, expansion and pipeline hand-offs are shared by
//     two 128 x 128 products.  Document ranges are token quantiles of the
//     corpus, 2 x SM-count of them, ordered range-major, so every CTA gets the
//     same number of equal-sized units and the CTAs working on one range run
//     together and share its codes through L2.
//   * Candidate lists: a list naming at least one document in 16 is read out of a
//     full scan; a shorter one gets one unit per (listed document, query-tile
//     pair), built on the device (candidate_units_kernel), and the same kernel
//     scores the listed documents into a [B, D] scratch that is gathered.
//   * Persistent CTAs (one per SM), 12 warps: warps 0-7 epilogue (query tile
//     warp / 4, TMEM lane quarter warp % 4), warp 8 TMEM allocation and MMA
//     issue (one thread), warps 9-10 expanders, warp 11 loader.  Fewer
//     producer warps leave more issue slots to the epilogue and allow up to
//     168 registers per thread.
//   * Operand tiles.  By default the int4 corpus is expanded once into a
//     resident int8 copy in the scan's K order (128 B per token, built by
//     expand_codes8_kernel on first use), and the loader fills each B stage
//     with one tiled TMA load (cp.async.bulk.tensor.2d, 128 rows x 128 bytes,
//     128-byte swizzle: the UMMA layout) while expander warps only stage the
//     tile metadata (token scales, document ends).  Without the copy (option
//     "tc_int8_cache" 0, or no memory for it) the loader copies raw int4 rows
//     into a 6-deep ring and the two expander warps take alternate tiles, each
//     writing 16 x every code (the nibble moved to the top of its byte, three
//     logic operations per four bytes of codes) in the swizzled layout, in a
//     chunk order that keeps their shared loads and stores free of bank
//     conflicts; the epilogue divides the 16 x dot accumulators back exactly.
//   * TMEM holds two token-tile buffers x two query tiles x 128 columns.  One
//     commit per token tile both frees its shared-memory stage and hands the
//     accumulators to the epilogue, which returns them as soon as the tile's
//     last columns are in registers.  The first K step overwrites, the other
//     three accumulate, so an accumulator holds the exact int32 dot (below
//     2^24: conversion to float is exact); one FMUL applies the token scale
//     and three-input max reduces.  The epilogue reads TMEM with 16x256b
//     loads, so each thread holds two rows x 16 columns per 64-column chunk
//     and reads its 16 token scales with four 16-byte loads from a permuted
//     layout; a row's maximum is completed with two butterfly shuffles when a
//     document ends, and tiles without document ends skip the walk.
//
// Variants (template parameters of tc_scan_kernel)
//   * kDigits: fp32 query rows as three int8 digit planes of their 23-bit fixed-point values, on four
//     TMEM lanes per row; the epilogue combines the planes' exact dots before the token scale.  Weighted
//     MaxSim folds the weights into the rows' power-of-two scales.
//   * Sign-code corpora read a resident +-1 int8 copy through the same TMA path.
//   * kTwin: passes with one query tile let the two epilogue groups take two document ranges in turn.
//   * kRep: one tile of at most 64 (32) int8 query rows is copied two (four) times over the TMEM lane
//     quarters, and each epilogue warp takes a 64- (32-) column slice of every token tile.
//   * kRes: the fused two-stream residual (int4 or sign-code prefix + int4 residual), two accumulators
//     per query tile.
//   * kTopK: the TopK2 / TopK4 reducers, per-thread lists merged across a row's four threads.
//   * kSmooth: the SmoothSim reducer, a running log-sum-exp per thread merged across a row's four threads.
//
// Every mbarrier wait is bounded (%globaltimer); on timeout the kernel raises
// an error flag, drains, frees its TMEM and returns.
#include <cuda.h>
#include <cuda_fp16.h>  // CUtensorMap (the encoder is fetched through cudaGetDriverEntryPoint)

#include <algorithm>
#include <atomic>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace msb {
namespace tc {

constexpr int kTileN = 128;       // tokens per tile (MMA N)
constexpr int kG = 2;             // query tiles per unit, sharing every expanded token tile
constexpr int kMeta = 8;          // tile metadata ring (scales, document ends), released by the epilogue
constexpr int kRaw = 6;           // raw-code ring filled by bulk copies
constexpr int kAccBufs = 2;       // token-tile accumulator buffers (each kG x 128 TMEM columns)
constexpr int kEpiWarps = 8;      // warp w: query tile w / 4 of the pair, TMEM lane quarter w % 4
constexpr int kXWarps = 2;        // expanders (two tokens per thread per tile)
constexpr int kMmaWarp = kEpiWarps;            // warp 8
constexpr int kXWarp0 = kMmaWarp + 1;          // warps 9..10
constexpr int kLoadWarp = kXWarp0 + kXWarps;   // warp 11
constexpr int kThreads = (kLoadWarp + 1) * 32; // 384 = 12 warps
constexpr int kSegGroup = 8;      // finished documents per epilogue flush
constexpr int kMaxRangeDocs = 512;
constexpr uint32_t kTmemCols = kAccBufs * kG * kTileN;        // 512
constexpr uint64_t kTimeoutNs = 4000000000ull;                // 4 s per wait
// Biased accumulators (int8 queries, per-token scales): one extra K = 32 MMA of two constant 0x7F
// operands opens every accumulator at kBiasValue = 32 * 127 * 127, so a finished accumulator holds
// dot + kBiasValue in (0, 2^23): read as a float it is the subnormal (dot + kBiasValue) * 2^-149, which
// one fused multiply-add maps exactly to dot * 2^-23 (see bias_scale2).
constexpr int kBiasBytes = 128 * 32;
constexpr int32_t kBiasValue = 32 * 127 * 127;  // 516,128 > |dot| <= 127 * 7 * 128 = 113,792
// Operand tiles expanded in shared memory hold 16 x the int4 codes (see the expanders), so accumulators
// hold 16 x the dot; their bias is 32 * 255 * 255 (unsigned 0xFF operands) > 16 * 127 * 8 * 128.
constexpr int32_t kBiasValue16 = 32 * 255 * 255;  // 2,080,800; 16 * dot + kBiasValue16 < 2^22

struct Unit {
  int64_t d_lo, d_hi;    // documents [d_lo, d_hi), at most kMaxRangeDocs
  int64_t tok_lo, tok_hi;
  int32_t qpair;         // query tiles kG * qpair .. kG * qpair + kG - 1
  int32_t pad;
};

struct Params {
  const uint8_t* codes;
  const float* token_scale;   // nullptr: tensor scale (integer maximum)
  const int64_t* offsets;
  const int32_t* qwords;      // [B*Q, 32] nibble-order int8 words
  const float* qscale;        // [B*Q]
  const Unit* units;
  int num_units;
  int num_items;              // work items: units, or (twin mode) pairs of units
  int batch;
  int qtok;
  int qpt;                    // queries per tile
  float scale;                // tensor scale applied to the document score (1 for the residual stream)
  const float* token_scale2;  // residual stream (kRes): per-token scales of the second stream
  float res_scale1;           // residual stream: the prefix's and the residual's scalar scales
  float res_scale2;
  int64_t num_docs;           // output row stride
  float* out;                 // [B, num_docs]
  int* error;                 // set to a non-zero code on timeout
  float smooth_scale;         // SmoothSim: the document scale applied to every value before the reduction
  float temperature;          // SmoothSim: the temperature (> 0)
  int topk_k;                 // fused top-k: k (0: write the score matrix instead)
  unsigned char* cand;        // fused top-k: candidate blocks [gridDim * groups][16 * batch * k bytes]
};

// Shared-memory layout (bytes, from a 1024-aligned base).
constexpr int kATileBytes = 128 * 128;                 // 16 KB
constexpr int kBTileBytes = kTileN * 128;              // 16 KB
constexpr int kRawCodeBytes = kTileN * 64;             // 8 KB
constexpr int kRawScaleFloats = kTileN + 4;            // aligned superset of the tile's scales
constexpr int kUoffEntries = kMaxRangeDocs + 4;
// Token scales in the order the epilogue threads consume them: column c = 64h + 8j + 2t + b is held by
// threads with t % 4 = t at index h * 80 + t * 20 + 2j + b, so each thread reads its 16 scales of a
// 64-column chunk with four conflict-free 16-byte loads (the 20-float stride spreads the four
// threads' blocks over distinct banks).
__host__ __device__ constexpr int scale_slot(int col) {
  return (col >> 6) * 80 + ((col & 7) >> 1) * 20 + ((col & 63) >> 3) * 2 + (col & 1);
}
struct StageMeta {
  float scale[160];
  int16_t seg_end[kTileN];   // exclusive end column of each document ending in the tile
  int32_t seg_doc[kTileN];
  int32_t nseg;
  int32_t valid;             // valid columns
};
constexpr int kMetaBytes = ((sizeof(StageMeta) + 127) / 128) * 128;
constexpr int kRowBytes = kSegGroup * kG * 128 * 4;    // [group][query tile][row]
// Shared-memory layout (bytes, from a 1024-aligned base).  When operand tiles arrive by TMA from the
// resident int8 copy (kPre), the raw ring carries only token scales, and the bytes the expanding path
// uses for raw int4 rows hold more B stages instead: a deeper operand prefetch for passes that are
// bound by DRAM latency (few query tiles, so little work per tile).
// With f16 operands (kF16, from the resident f16 copy) each operand tile is twice as large (two 128-byte
// swizzled K halves of 64 values) and the query tiles are single-buffered to keep 4 B stages.
// With the residual stream (kRes) each B stage holds two operand tiles (prefix, then residual), the raw
// ring two scale vectors, and a second scale array per meta slot sits after the meta ring.
// With biased accumulators (kBias) a 4 KB constant operand follows the B ring, which has one stage less.
template <bool kPre, bool kF16 = false, bool kRes = false, bool kBias = false>
struct Layout {
  static constexpr int stages = (kF16 || kRes) ? 4 : (kPre ? (kBias ? 7 : 8) : 4);  // B ring, freed by the MMA commit
  static constexpr int a_tile = kF16 ? 2 * kATileBytes : kATileBytes;
  static constexpr int b_tile = (kF16 || kRes) ? 2 * kBTileBytes : kBTileBytes;
  static constexpr int a_bufs = (kF16 || kRes) ? 1 : 2;
  static constexpr int raw_code_bytes = kPre ? 0 : kRawCodeBytes;
  static constexpr int raw_scale_bytes = kRawScaleFloats * 4;  // one vector (16-byte multiple)
  static constexpr int raw_bytes = ((raw_code_bytes + (kRes ? 2 : 1) * raw_scale_bytes + 127) / 128) * 128;
  static constexpr int off_a = 0;                        // [a_bufs][kG] query tiles
  static constexpr int off_b = off_a + a_bufs * kG * a_tile;
  static constexpr int off_bias = off_b + stages * b_tile;  // kBias: 128 rows x 32 bytes of 0x7F
  static constexpr int off_raw = off_bias + (kBias ? kBiasBytes : 0);
  static constexpr int off_meta = off_raw + kRaw * raw_bytes;
  static constexpr int off_scale2 = off_meta + kMeta * kMetaBytes;  // [kMeta][160] (kRes)
  static constexpr int off_uoff = off_scale2 + (kRes ? kMeta * 160 * 4 : 0);
  static constexpr int off_row = off_uoff + 2 * kUoffEntries * 8;
  static constexpr int off_bar = off_row + kRowBytes + 128;  // + per-group doc ids
  static constexpr int num_bars = 2 * stages + 2 * kMeta + 2 * kRaw + kAccBufs + 10;
  // fused top-k lists (fp32 score + int32 document per entry) in what the 227 KB leave, at most 8 KB
  static constexpr int off_topk = ((off_bar + num_bars * 8 + 64) + 15) / 16 * 16;
  static constexpr int topk_room = (227 * 1024 - 1024 - off_topk) / 16 * 16;
  static constexpr int topk_bytes = topk_room < 8192 ? topk_room : 8192;
  static constexpr int bytes = off_topk + topk_bytes + 1024;  // + alignment slack
  static constexpr int bytes_plain = off_topk + 1024;         // without the lists (no fused top-k)
  static_assert(bytes <= 227 * 1024 && topk_bytes >= 0, "shared memory budget");
  static_assert(off_b % 1024 == 0 && b_tile % 1024 == 0 && a_tile % 1024 == 0, "128-byte-swizzled operand tiles");
  static_assert(off_uoff % 16 == 0 && off_raw % 16 == 0 && raw_bytes % 16 == 0 && raw_scale_bytes % 16 == 0,
                "bulk-copy alignment");
};

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)  // suspend up to ~1 ms per try
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: false on timeout (after raising the error flag and abort bit).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int code) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  // The loader and expander warps (codes < 20 or >= 40) back off so their waiting does not take issue
  // slots from the epilogue warps; the MMA warp (20-29) and the epilogue (30-39) rely on try_wait's own
  // suspension, so they resume as soon as the phase completes.
  const bool backoff = code < 20 || code >= 40;
  uint32_t sleep_ns = 32;
  for (uint32_t it = 0;; ++it) {
    if (mbar_try(bar, parity)) return true;
    if (backoff) {
      __nanosleep(sleep_ns);
      if (sleep_ns < 256) sleep_ns <<= 1;
    }
    if ((it & 7u) == 7u) {
      if (*abort_flag) return false;
      if (global_ns() - t0 > kTimeoutNs) {
        *abort_flag = 1;
        atomicExch(err, code);
        return false;
      }
    }
  }
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  // K-major, no swizzle: 8-row x 16-byte core matrices; LBO between core
  // matrices along K, SBO between 8-row groups; version 1 (bits 46-47).
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);  // SWIZZLE_128B
}
// K-major, no swizzle (layout type 0): the constant bias operand, 128 rows x 32 bytes in 8-row x 16-byte
// core matrices, LBO 128 bytes between the two K core matrices, SBO 256 bytes between 8-row groups.
// Every byte is 0x7F, so the product does not depend on how rows map to addresses inside the 4 KB.
__device__ __forceinline__ uint64_t umma_desc_plain(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(128u >> 4) << 16) |
         (static_cast<uint64_t>(256u >> 4) << 32) | (1ull << 46);
}
// Two biased accumulators of adjacent columns (as float bits: subnormals (dot + kBiasValue) * 2^-149)
// to fl(dot * s) for their token scales, given as s * 2^23: the packed FMA forms
// (dot + kBiasValue) * 2^-23 - kBiasValue * 2^-23 = dot * 2^-23 exactly (|dot| < 2^17; subnormal
// inputs are kept, no flush to zero), and the packed product dot * 2^-23 * (s * 2^23) is rounded once,
// to the same float as fl(float(dot) * s).  Two instructions per two values, both on the FMA pipe.
// kX16: accumulators of 16 * dot + kBiasValue16: (16 dot + kBiasValue16) * 2^-27 - kBiasValue16 * 2^-27
// is the same dot * 2^-23, exactly.
template <bool kX16 = false>
__device__ __forceinline__ void bias_scale2(uint32_t& x0, uint32_t& x1, float2 s23) {
  // -bias * 2^-23 (or 2^-27), exact
  constexpr float kNeg = kX16 ? -static_cast<float>(kBiasValue16) / 134217728.0F
                              : -static_cast<float>(kBiasValue) / 8388608.0F;
  constexpr float kMul = kX16 ? 0x1p122F : 0x1p126F;
  const float2 v = __fmul2_rn(__ffma2_rn(make_float2(__uint_as_float(x0), __uint_as_float(x1)),
                                         make_float2(kMul, kMul), make_float2(kNeg, kNeg)),
                              s23);
  x0 = __float_as_uint(v.x);
  x1 = __float_as_uint(v.y);
}
// Two biased accumulators (as above) to dot * 2^-23, exactly, as a float pair.
template <bool kX16 = false>
__device__ __forceinline__ float2 bias_unscale2(uint32_t x0, uint32_t x1) {
  constexpr float kNeg = kX16 ? -static_cast<float>(kBiasValue16) / 134217728.0F
                              : -static_cast<float>(kBiasValue) / 8388608.0F;
  constexpr float kMul = kX16 ? 0x1p122F : 0x1p126F;
  return __ffma2_rn(make_float2(__uint_as_float(x0), __uint_as_float(x1)), make_float2(kMul, kMul),
                    make_float2(kNeg, kNeg));
}
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Byte offset of (row, 16-byte K chunk) in a no-swizzle K-major tile of 128-byte rows.
__device__ __forceinline__ uint32_t tile_off(int row, int kchunk) {
  // 128-byte swizzle: 8-row x 128-byte atoms, 16-byte chunk index XOR (row % 8)
  return static_cast<uint32_t>((row >> 3) * 1024 + (row & 7) * 128 + ((kchunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// 1D bulk copy global -> shared (TMA engine), completing transaction bytes on `bar`.
// Both addresses 16-byte aligned, size a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// Tiled 2D TMA load of box {128 bytes, 128 rows} at (x bytes, y rows), completing tx bytes on `bar`.
// x is 0 (16-byte aligned); no multicast.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 16 TMEM lanes x 64 columns: thread t receives, for j = 0..7, columns 8j + 2(t % 4) + {0, 1} of lane
// (t / 4) in r[4j], r[4j + 1] and of lane (t / 4 + 8) in r[4j + 2], r[4j + 3].
__device__ __forceinline__ void tmem_ld16x256b_x8(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 16 TMEM lanes x 32 columns: as tmem_ld16x256b_x8 for j = 0..3.
__device__ __forceinline__ void tmem_ld16x256b_x4(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Maximum of row s (0 or 1) of a 16x256b chunk half X (its 16 values X[4j + 2s], X[4j + 2s + 1]) folded
// into R: four independent chains of three-input maxima.
// Insertion of x into a descending list of K values, keeping the K largest: v'[0] = max(v[0], x),
// v'[i] = max(v[i], min(v[i-1], x)) (2K - 1 min / max instead of K compare-and-swaps).  The list is the
// same multiset, in the same descending order, as the SIMT reducer's insertion gives, so its sum is too.
template <int K>
__device__ __forceinline__ void topk_insert(float (&v)[K], float x) {
#pragma unroll
  for (int i = K - 1; i > 0; --i) v[i] = fmaxf(v[i], fminf(v[i - 1], x));
  v[0] = fmaxf(v[0], x);
}

template <int NJ>
__device__ __forceinline__ float row_max16(const uint32_t* X, int s, float R) {
  if constexpr (NJ == 4) {  // 8 values: X[4j + 2s], X[4j + 2s + 1], j = 0..3
    const float m0 = fmax3(R, __uint_as_float(X[2 * s]), __uint_as_float(X[2 * s + 1]));
    const float m1 = fmax3(__uint_as_float(X[4 + 2 * s]), __uint_as_float(X[4 + 2 * s + 1]), __uint_as_float(X[8 + 2 * s]));
    const float m2 =
        fmax3(__uint_as_float(X[8 + 2 * s + 1]), __uint_as_float(X[12 + 2 * s]), __uint_as_float(X[12 + 2 * s + 1]));
    return fmax3(m0, m1, m2);
  }
  float m0 = fmax3(__uint_as_float(X[2 * s]), __uint_as_float(X[2 * s + 1]), __uint_as_float(X[16 + 2 * s]));
  float m1 = fmax3(__uint_as_float(X[4 + 2 * s]), __uint_as_float(X[4 + 2 * s + 1]), __uint_as_float(X[20 + 2 * s]));
  const float m2 =
      fmax3(__uint_as_float(X[8 + 2 * s]), __uint_as_float(X[8 + 2 * s + 1]), __uint_as_float(X[16 + 2 * s + 1]));
  const float m3 =
      fmax3(__uint_as_float(X[12 + 2 * s]), __uint_as_float(X[12 + 2 * s + 1]), __uint_as_float(X[20 + 2 * s + 1]));
  m0 = fmax3(m0, __uint_as_float(X[24 + 2 * s]), __uint_as_float(X[24 + 2 * s + 1]));
  m1 = fmax3(m1, __uint_as_float(X[28 + 2 * s]), __uint_as_float(X[28 + 2 * s + 1]));
  return fmax3(R, fmax3(m0, m1, m2), m3);
}
template <int NJ>
__device__ __forceinline__ int32_t row_max16i(const uint32_t* X, int s, int32_t R) {
  int32_t m0 = max(static_cast<int32_t>(X[2 * s]), static_cast<int32_t>(X[2 * s + 1]));
  int32_t m1 = max(static_cast<int32_t>(X[4 + 2 * s]), static_cast<int32_t>(X[4 + 2 * s + 1]));
#pragma unroll
  for (int j = 2; j < NJ; j += 2) {
    m0 = __vimax3_s32(m0, static_cast<int32_t>(X[4 * j + 2 * s]), static_cast<int32_t>(X[4 * j + 2 * s + 1]));
    m1 = __vimax3_s32(m1, static_cast<int32_t>(X[4 * j + 4 + 2 * s]), static_cast<int32_t>(X[4 * j + 4 + 2 * s + 1]));
  }
  return __vimax3_s32(R, m0, m1);
}

// Row value r of a flushed document: with replicated query rows (kRep copies of 128 / kRep rows, each
// the scaled maximum over one column slice) the largest copy.  The query scale is >= 0, so the maximum of
// the scaled slice maxima equals the scaled maximum over all columns.
template <int kRep>
__device__ __forceinline__ float rep_max(const float* rv, int r) {
  float v = rv[r];
#pragma unroll
  for (int c = 1; c < kRep; ++c) v = fmaxf(v, rv[r + c * (128 / kRep)]);
  return v;
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
struct Ring {
  int idx = 0;
  uint32_t phase = 0;
  template <int N>
  __device__ __forceinline__ void next() {
    if (++idx == N) {
      idx = 0;
      phase ^= 1;
    }
  }
};

// kPre: the int4 codes were expanded once into an int8 copy (same K order); each B stage is a tiled TMA
// load of 128 rows from it, landing in the 128-byte-swizzled layout, and the expanders only stage the
// tile metadata.  Otherwise the loader copies raw int4 rows and the expanders build the B stage.
// A work item is one unit, or in twin mode (a single query tile) the two units 2w and 2w + 1 whose token
// tiles alternate, side 0 first: epilogue group g takes side g's tiles, so both groups work although only
// one query tile exists.  A side whose unit has run out of tiles (or an odd unit count's missing unit)
// contributes empty tiles (no columns), so every role enumerates the same steps.
struct Item {
  Unit un[2];
  int64_t nsteps;
};
__device__ __forceinline__ int64_t unit_tiles(const Unit& u) { return (u.tok_hi - u.tok_lo + kTileN - 1) / kTileN; }
template <bool kTwin>
__device__ __forceinline__ Item load_item(const Params& p, int w) {
  Item it;
  if (kTwin) {
    const Unit none{0, 0, 0, 0, 0, 0};
    it.un[0] = p.units[2 * w];
    it.un[1] = 2 * w + 1 < p.num_units ? p.units[2 * w + 1] : none;
    it.nsteps = 2 * max(unit_tiles(it.un[0]), unit_tiles(it.un[1]));
  } else {
    it.un[0] = p.units[w];
    it.un[1] = it.un[0];
    it.nsteps = unit_tiles(it.un[0]);
  }
  return it;
}
struct Step {
  int side;       // unit of the item (0 outside twin mode)
  int valid;      // columns of the tile (0: an empty tile)
  bool last;      // the unit's last tile
  int64_t t0;     // first token
};
template <bool kTwin>
__device__ __forceinline__ Step step_of(const Item& it, int64_t i) {
  Step st;
  st.side = kTwin ? static_cast<int>(i & 1) : 0;
  const Unit& u = (kTwin && st.side) ? it.un[1] : it.un[0];
  st.t0 = u.tok_lo + (kTwin ? (i >> 1) : i) * kTileN;
  const int64_t rem = u.tok_hi - st.t0;
  st.valid = rem <= 0 ? 0 : (rem < kTileN ? static_cast<int>(rem) : kTileN);
  st.last = rem > 0 && rem <= kTileN;
  return st;
}

// kDigits: fp32 queries as three int8 digit planes (split_query_digits_kernel).  Query row rho of a tile
// (32 per tile) has its digit k on TMEM lane 32 (rho / 8) + 8 k + rho % 8 (k = 3: zeros), the four lanes
// one epilogue thread holds, which combines them to d0 + 256 d1 + 65536 d2 before the scale and maximum.
// kTwin: the pass has one query tile and runs in twin mode (see Item); a template parameter, so that the
// passes with several query tiles compile to the plain one-unit loop.
// kRes: the fused two-stream residual (fp32 queries as digit planes, per-token scales on both streams):
// per token tile the prefix tile (tmap) and the residual tile (tmap2) each get an accumulator per query
// tile, so one accumulator buffer fills the 512 TMEM columns; the epilogue forms
// fl(fl(fl(v1 * scale1) * s1) + fl(fl(v2 * scale2) * s2)) before the maximum.
// kTopK (2 or 4): the TopK reducers of digit-plane queries: each thread keeps a descending list of its
// columns' largest values per row and a token count; at a document end the four threads holding the row
// merge lists and counts, and the row value is the mean of the top min(K, tokens) values (summed in
// descending order), as the SIMT reducer forms it.
// kBias: biased accumulators (kBiasValue, int8 queries with per-token scales): the epilogue converts and
// scales two values with two packed FMA-pipe instructions (bias_scale2) instead of an int32 -> fp32
// conversion and a product per value; the token scales are staged as s * 2^23 (the host keeps this
// variant for corpora whose token scales are below 2^104, so that s * 2^23 is exact).
// kRep (2 or 4; twin mode, int8 queries, at most 128 / kRep query rows): the query tile is replicated over
// the four TMEM lane quarters (kRep copies of 128 / kRep rows), so every epilogue warp holds each of its rows
// for only its slice of 128 / kRep columns of a token tile; a document's row maximum is completed across the
// kRep copies when its group is flushed.  One or two live warps per group would otherwise do a whole
// tile's epilogue alone.
// kFuse: the full-scan top-k is selected in the scan (int8 queries, unreplicated rows): each CTA (twin
// mode: each epilogue group) keeps the k best documents of every query in shared memory and writes them as
// one candidate block for a merge kernel.  A template parameter, so that the other scans carry none of it.
template <bool kTokenScale, bool kPre, bool kF16, bool kDigits = false, bool kTwin = false, bool kRes = false,
          int kTopK = 0, bool kBias = false, bool kSmooth = false, int kRep = 1, bool kFuse = false>
__global__ void __launch_bounds__(kThreads, 1) tc_scan_kernel(Params p, const __grid_constant__ CUtensorMap tmap,
                                                              const __grid_constant__ CUtensorMap tmap2) {
  using L = Layout<kPre, kF16, kRes, kBias>;
  static_assert(!kBias || (!kF16 && !kRes && (kDigits || (kTokenScale && kTopK == 0))),
                "biased accumulators: int8 queries with per-token scales, or digit-plane queries");
  static_assert(!kRes || (kPre && kDigits && kTokenScale && !kF16), "the residual stream reads both int8 copies");
  static_assert(kTopK == 0 || (kTopK <= 4 && kPre && kDigits && !kRes), "TopK: digit-plane queries, int8 copies");
  static_assert(!kSmooth || (kTopK == 0 && kPre && kDigits && !kRes), "SmoothSim: digit-plane queries, int8 copies");
  static_assert(kRep == 1 || ((kRep == 2 || kRep == 4) && kTwin && !kDigits && !kF16 && !kRes && !kSmooth),
                "replicated query rows: one tile of int8 query rows");
  static_assert(!kFuse || (kRep == 1 && !kDigits && !kF16 && !kRes && kTopK == 0 && !kSmooth),
                "fused top-k: int8-query MaxSim");
  constexpr int kQuarters = 4 / kRep;               // lane quarters holding distinct query rows
  constexpr int kChunkCols = kRep == 4 ? 32 : 64;   // columns of one pair of TMEM loads
  constexpr int kNJ = kChunkCols / 8;               // 8-column groups per load
  constexpr int kChunks = kRep == 1 ? 2 : 1;        // load pairs per token tile and warp
  // Expanding path (operand tiles built from int4 rows in shared memory): the two expander warps take
  // alternate tiles, each a whole tile, and the tiles hold 16 x the codes (accumulators of 16 x the dot).
  constexpr bool kAlt = !kPre;
  constexpr bool kList = kTopK > 0 || kSmooth;     // reducers that take the per-segment path in every chunk
  constexpr int kTk = kTopK > 0 ? kTopK : 1;
  constexpr int kAcc = kRes ? 1 : kAccBufs;         // accumulator buffers
  constexpr int kStreams = kRes ? 2 : 1;            // accumulators per query tile
  static_assert(!kF16 || (kPre && kTokenScale), "f16 operands come from the resident copy, with token scales");
  static_assert(!(kF16 && kDigits), "digit-plane queries use int8 operands");
  constexpr bool kFloat = kTokenScale || kDigits;  // row maxima in fp32; int32 for the tensor-scale dots
  constexpr int kRows = kDigits ? 1 : 4;            // query rows an epilogue thread holds
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                         ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::off_bar);
  uint64_t* full = bars;                         // [stages]   expanders or TMA -> MMA
  uint64_t* tile_done = full + L::stages;        // [stages]   MMA commit -> loader/expanders (stage free), epilogue
  uint64_t* m_full = tile_done + L::stages;      // [kMeta]    expanders -> epilogue
  uint64_t* m_empty = m_full + kMeta;            // [kMeta]    epilogue -> expanders
  uint64_t* raw_full = m_empty + kMeta;          // [kRaw]     bulk copies -> expanders
  uint64_t* raw_empty = raw_full + kRaw;         // [kRaw]     expanders -> loader
  uint64_t* acc_empty = raw_empty + kRaw;        // [kAccBufs] epilogue -> MMA
  uint64_t* a_full = acc_empty + kAccBufs;       // [2]        expanders -> MMA
  uint64_t* a_empty = a_full + 2;                // [2]        MMA commit -> expanders
  uint64_t* u_full = a_empty + 2;                // [2]        unit offsets bulk copy -> segment warp
  uint64_t* u_empty = u_full + 2;                // [2]        segment warp -> loader
  uint64_t* epi_bar = u_empty + 2;               // [2]        epilogue warps among themselves (document flush;
                                                 //            one per group in twin mode)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::num_bars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* rowval = reinterpret_cast<float*>(smem + L::off_row);                      // [group][kG][128]
  int32_t* group_doc = reinterpret_cast<int32_t*>(smem + L::off_row + kRowBytes);  // [2][kSegGroup]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int Q = p.qtok;
  // fused top-k: per list group (twin mode: one per epilogue group) and query, k entries kept in
  // (score desc, document asc) order; an entry with document -1 is empty
  constexpr int kLists = kTwin ? 2 : 1;
  const int tk_n = kFuse ? kLists * p.batch * p.topk_k : 0;
  float* tks = reinterpret_cast<float*>(smem + L::off_topk);
  int32_t* tki = reinterpret_cast<int32_t*>(tks + tk_n);
  for (int e = threadIdx.x; e < tk_n; e += kThreads) {
    tks[e] = -INFINITY;
    tki[e] = -1;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < L::stages; ++s) {
      mbar_init(&full[s], 1);  // kPre: the loader's expect_tx + the TMA's bytes; else the tile's expander
      mbar_init(&tile_done[s], 1);
    }
    for (int s = 0; s < kMeta; ++s) {
      // kPre: the expanders' metadata and the MMA warp's commit of the tile's products (kXWarps + 1)
      mbar_init(&m_full[s], kPre ? kXWarps + 1 : 1);
      mbar_init(&m_empty[s], kTwin ? kEpiWarps / 2 : kEpiWarps);  // twin: only the owning group reads a tile
    }
    for (int s = 0; s < kRaw; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], kAlt ? 1 : kXWarps);
    }
    for (int a = 0; a < kAccBufs; ++a) mbar_init(&acc_empty[a], kEpiWarps);
    for (int a = 0; a < 2; ++a) {
      mbar_init(&a_full[a], kXWarps);
      mbar_init(&a_empty[a], 1);
      mbar_init(&u_full[a], 1);
      mbar_init(&u_empty[a], kAlt ? kXWarps : 1);  // the warps that walk the unit's offsets
    }
    if (kTwin) {
      mbar_init(&epi_bar[0], kEpiWarps / 2);
      mbar_init(&epi_bar[1], kEpiWarps / 2);
    } else {
      mbar_init(&epi_bar[0], kEpiWarps);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (kBias) {
    // the constant bias operand, made visible to the tensor core (async proxy) before the first MMA
    constexpr uint32_t kc = kPre ? 0x7F7F7F7Fu : 0xFFFFFFFFu;  // s8 127, or u8 255 for 16 x the codes
    for (int i = threadIdx.x; i < kBiasBytes / 16; i += kThreads)
      reinterpret_cast<uint4*>(smem + L::off_bias)[i] = make_uint4(kc, kc, kc, kc);
    fence_proxy_async();
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == kLoadWarp) {
    // =================== loader: bulk copies run ahead of the expanders ===================
    if (lane == 0) {
      Ring raw, stg;
      int iter = 0;
      for (int w = blockIdx.x; w < p.num_items; w += gridDim.x, ++iter) {
        const Item it = load_item<kTwin>(p, w);
        // Each unit's offsets[d_lo .. d_hi] as a 16-byte-aligned superset (the buffer is padded): slots
        // alternate between items, or (twin mode) slot s holds side s.
        for (int side = 0; side < (kTwin ? 2 : 1); ++side) {
          const int ub = kTwin ? side : (iter & 1);
          const int use = kTwin ? iter : (iter >> 1);  // earlier uses of the slot
          if (use >= 1 && !mbar_wait(&u_empty[ub], (use - 1) & 1, abort_flag, p.error, 41)) goto done;
          const Unit& unit = side ? it.un[1] : it.un[0];
          if (unit.d_hi > unit.d_lo) {
            const int64_t first = unit.d_lo & ~1LL;
            const int64_t count = ((unit.d_hi + 1 - first) + 1) & ~1LL;
            const uint32_t bytes = static_cast<uint32_t>(count * 8);
            mbar_expect_tx(&u_full[ub], bytes);
            bulk_g2s(smem + L::off_uoff + ub * kUoffEntries * 8, p.offsets + first, bytes, &u_full[ub]);
          } else {
            mbar_arrive(&u_full[ub]);  // an odd unit count's missing unit: no documents
          }
        }
        for (int64_t i = 0; i < it.nsteps; ++i) {
          const Step st = step_of<kTwin>(it, i);
          const int64_t t0 = st.t0;
          const int valid = st.valid;
          if (kPre) {
            // B stage: wait until the MMAs that read it have completed, then one tiled TMA load
            if (!mbar_wait(&tile_done[stg.idx], stg.phase ^ 1, abort_flag, p.error, 43)) goto done;
            if (valid > 0) {
              mbar_expect_tx(&full[stg.idx], static_cast<uint32_t>(L::b_tile));
              unsigned char* bdst = smem + L::off_b + stg.idx * L::b_tile;
              tma_load_2d(bdst, &tmap, 0, static_cast<int>(t0), &full[stg.idx]);
              // f16: the second K half (values 64..127, byte 128 of each row: x * 2 B is 16-byte aligned)
              if (kF16) tma_load_2d(bdst + kBTileBytes, &tmap, 64, static_cast<int>(t0), &full[stg.idx]);
              // residual stream: the same tokens of the residual int8 copy
              if (kRes) tma_load_2d(bdst + kBTileBytes, &tmap2, 0, static_cast<int>(t0), &full[stg.idx]);
            } else {
              mbar_arrive(&full[stg.idx]);  // an empty tile: nothing to load
            }
            stg.next<L::stages>();
          }
          if (!mbar_wait(&raw_empty[raw.idx], raw.phase ^ 1, abort_flag, p.error, 42)) goto done;
          unsigned char* rb = smem + L::off_raw + raw.idx * L::raw_bytes;
          const uint32_t code_bytes = kPre ? 0u : static_cast<uint32_t>(valid) * 64u;
          uint32_t scale_bytes = 0;
          const int64_t s_first = t0 & ~3LL;
          if (kTokenScale && valid > 0) scale_bytes = static_cast<uint32_t>(((t0 + valid - s_first + 3) & ~3LL) * 4);
          mbar_expect_tx(&raw_full[raw.idx], code_bytes + (kRes ? 2 : 1) * scale_bytes);
          if (code_bytes) bulk_g2s(rb, p.codes + t0 * 64, code_bytes, &raw_full[raw.idx]);
          if (scale_bytes) bulk_g2s(rb + L::raw_code_bytes, p.token_scale + s_first, scale_bytes, &raw_full[raw.idx]);
          if (kRes && scale_bytes)
            bulk_g2s(rb + L::raw_code_bytes + L::raw_scale_bytes, p.token_scale2 + s_first, scale_bytes,
                     &raw_full[raw.idx]);
          raw.next<kRaw>();
        }
      }
    }
  } else if (warp >= kXWarp0) {
    // =================== expanders: int4 -> int8 bytes, UMMA layout ===================
    const int xtid = threadIdx.x - kXWarp0 * 32;  // 0..63
    const int xwarp = warp - kXWarp0;
    Ring raw, stg, mst;
    int iter = 0;
    // the tile pair whose query rows each A buffer holds: within a launch they depend on the pair alone, so
    // a buffer that already holds the item's pair is handed to the MMA again unwritten (runs of units of
    // one pair: small batches, candidate lists)
    int32_t a_held[2] = {-1, -1};
    for (int w = blockIdx.x; w < p.num_items; w += gridDim.x, ++iter) {
      const Item it = load_item<kTwin>(p, w);
      const int32_t qpair = it.un[0].qpair;  // twin mode: both units hold the one query tile
      const int abuf = iter % L::a_bufs;
      const int ause = iter / L::a_bufs;
      if (ause >= 1 && !mbar_wait(&a_empty[abuf], (ause - 1) & 1, abort_flag, p.error, 11)) goto done;
      const bool a_build = a_held[abuf] != qpair;
      a_held[abuf] = qpair;
#pragma unroll 1
      for (int row = xtid; row < (a_build ? 128 : 0); row += kXWarps * 32) {  // query rows of each tile of the pair
#pragma unroll
        for (int g = 0; g < kG; ++g) {
          unsigned char* A = smem + L::off_a + (abuf * kG + g) * L::a_tile;
          int b, qrow;
          bool valid;
          int64_t src_row;
          if (kDigits) {
            const int k = (row >> 3) & 3;                   // digit plane of this lane
            const int rho = ((row >> 5) << 3) | (row & 7);  // query row of the tile
            b = (qpair * kG + g) * p.qpt + rho / Q;
            qrow = rho % Q;
            valid = k < 3 && rho < p.qpt * Q && b < p.batch;
            src_row = valid ? static_cast<int64_t>(k) * p.batch * Q + static_cast<int64_t>(b) * Q + qrow : 0;
          } else {
            const int rr = row & (128 / kRep - 1);  // kRep > 1: the copies of rows 0 .. 128 / kRep - 1
            b = (qpair * kG + g) * p.qpt + rr / Q;
            qrow = rr % Q;
            valid = rr < p.qpt * Q && b < p.batch;
            src_row = valid ? static_cast<int64_t>(b) * Q + qrow : 0;
          }
          const int4* src = reinterpret_cast<const int4*>(p.qwords + src_row * 32);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            int4 v = valid ? __ldg(src + c) : make_int4(0, 0, 0, 0);
            if (kF16) {
              // 16 int8 values -> 16 f16 (exact): 32 bytes at byte 32c of the row, K half c / 4
              const uint32_t w[4] = {static_cast<uint32_t>(v.x), static_cast<uint32_t>(v.y),
                                     static_cast<uint32_t>(v.z), static_cast<uint32_t>(v.w)};
              uint32_t h2[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int8_t lo = static_cast<int8_t>((w[i >> 1] >> (16 * (i & 1))) & 0xFF);
                const int8_t hi = static_cast<int8_t>((w[i >> 1] >> (16 * (i & 1) + 8)) & 0xFF);
                h2[i] = static_cast<uint32_t>(__half_as_ushort(__int2half_rn(lo))) |
                        (static_cast<uint32_t>(__half_as_ushort(__int2half_rn(hi))) << 16);
              }
              unsigned char* Ah = A + (c >> 2) * kATileBytes;
              *reinterpret_cast<uint4*>(Ah + tile_off(row, 2 * (c & 3))) = make_uint4(h2[0], h2[1], h2[2], h2[3]);
              *reinterpret_cast<uint4*>(Ah + tile_off(row, 2 * (c & 3) + 1)) = make_uint4(h2[4], h2[5], h2[6], h2[7]);
            } else {
              *reinterpret_cast<int4*>(A + tile_off(row, c)) = v;
            }
          }
        }
      }
      {
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[abuf]);
      }
      if (kAlt || xwarp == 0) {
        for (int side = 0; side < (kTwin ? 2 : 1); ++side) {
          const int ub = kTwin ? side : (iter & 1);
          const int use = kTwin ? iter : (iter >> 1);
          if (!mbar_wait(&u_full[ub], use & 1, abort_flag, p.error, 13)) goto done;
        }
      }
      int64_t next_doc0 = it.un[0].d_lo, next_doc1 = it.un[1].d_lo;  // first documents whose ends are ahead
      for (int64_t i = 0; i < it.nsteps; ++i) {
        if (kAlt && static_cast<int>(i & 1) != xwarp) {
          // the other expander warp's tile
          raw.next<kRaw>();
          stg.next<L::stages>();
          mst.next<kMeta>();
          continue;
        }
        const Step st = step_of<kTwin>(it, i);
        const Unit& unit = st.side ? it.un[1] : it.un[0];
        const int ub = kTwin ? st.side : (iter & 1);
        const int64_t* uoff = reinterpret_cast<const int64_t*>(smem + L::off_uoff + ub * kUoffEntries * 8);
        const int64_t ufirst = unit.d_lo & ~1LL;
        const int64_t t0 = st.t0;
        if (!mbar_wait(&raw_full[raw.idx], raw.phase, abort_flag, p.error, 14)) goto done;
        if (!kPre && !mbar_wait(&tile_done[stg.idx], stg.phase ^ 1, abort_flag, p.error, 12)) goto done;
        if (!mbar_wait(&m_empty[mst.idx], mst.phase ^ 1, abort_flag, p.error, 15)) goto done;
        const unsigned char* rb = smem + L::off_raw + raw.idx * L::raw_bytes;
        unsigned char* Bt = smem + L::off_b + stg.idx * L::b_tile;
        StageMeta* meta = reinterpret_cast<StageMeta*>(smem + L::off_meta + mst.idx * kMetaBytes);
        const int valid = st.valid;
        if (kPre && kTokenScale) {
          const float* rs = reinterpret_cast<const float*>(rb + L::raw_code_bytes);
          // biased accumulators take s * 2^23 (exact: the host checked s < 2^104)
          for (int r = xtid; r < valid; r += kXWarps * 32)
            meta->scale[scale_slot(r)] = kBias ? __fmul_rn(rs[(t0 & 3) + r], 8388608.0F) : rs[(t0 & 3) + r];
          if (kRes) {
            const float* rs2 = reinterpret_cast<const float*>(rb + L::raw_code_bytes + L::raw_scale_bytes);
            float* sc2 = reinterpret_cast<float*>(smem + L::off_scale2 + mst.idx * 160 * 4);
            for (int r = xtid; r < valid; r += kXWarps * 32) sc2[scale_slot(r)] = rs2[(t0 & 3) + r];
          }
        }
        if (!kPre) {
          // One warp expands the whole tile: lane l takes tokens l + 32u, u = 0..3, each 64 bytes of int4
          // codes -> 128 bytes of 16 * code (an exact int8: the nibble in the high half of its byte, its
          // sign bit the byte's), so the products are 16 x the integer dots.  Per 32-bit word: the high
          // nibbles (odd dims) are w & 0xF0F0F0F0 and the low nibbles (even dims) (w << 4) & 0xF0F0F0F0.
          // Chunk order c = M(a) ^ step with a = (r / 2) % 4 and M multiplication by a generator of GF(4)
          // ({0, 2, 3, 1}): both c and c ^ a run over all four values within each 8-token quarter warp,
          // so the raw loads (bank slot 4(r % 2) + c) and the swizzled stores (slot 2(c ^ a) + r % 2) are
          // conflict-free.  A full tile issues its sixteen loads per lane before the arithmetic.
          const int qa = (lane >> 1) & 3;
          const int qm = ((qa << 1) & 3) ^ ((qa >> 1) * 3);
          auto expand = [&](int r, int c, const uint4 v) {
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
            uint32_t o[8];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              o[2 * k] = (w[k] << 4) & 0xF0F0F0F0u;  // even dims (low nibbles)
              o[2 * k + 1] = w[k] & 0xF0F0F0F0u;     // odd dims (high nibbles)
            }
            *reinterpret_cast<uint4*>(Bt + tile_off(r, 2 * c)) = make_uint4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<uint4*>(Bt + tile_off(r, 2 * c + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
          };
          if (valid == kTileN) {
            uint4 v[4][4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
              for (int step = 0; step < 4; ++step)
                v[u][step] = *reinterpret_cast<const uint4*>(rb + (lane + 32 * u) * 64 + (qm ^ step) * 16);
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
              for (int step = 0; step < 4; ++step) expand(lane + 32 * u, qm ^ step, v[u][step]);
          } else {
#pragma unroll 1
            for (int r = lane; r < valid; r += 32)
#pragma unroll
              for (int step = 0; step < 4; ++step)
                expand(r, qm ^ step, *reinterpret_cast<const uint4*>(rb + r * 64 + (qm ^ step) * 16));
          }
          if (kTokenScale) {
            const float* rs = reinterpret_cast<const float*>(rb + L::raw_code_bytes);
            for (int r = lane; r < valid; r += 32)
              meta->scale[scale_slot(r)] = kBias ? __fmul_rn(rs[(t0 & 3) + r], 8388608.0F) : rs[(t0 & 3) + r];
          }
        }
        // Documents ending inside (t0, t0 + valid]: the tile's warp (expanding path; each warp skips the
        // ends of the other warp's tiles first) or expander warp 0 walks the unit's offsets in smem.
        if (kAlt || xwarp == 0) {
          int nseg = 0;
          const int64_t tile_end = t0 + valid;
          int64_t next_doc = st.side ? next_doc1 : next_doc0;
          while (valid > 0) {
            const int64_t d = next_doc + lane;
            const bool in = d < unit.d_hi;
            const int64_t e = in ? uoff[d + 1 - ufirst] : INT64_MAX;
            const int64_t s = in ? uoff[d - ufirst] : INT64_MAX;
            const bool ends = in && e <= tile_end;
            const bool nonempty = ends && e > t0 && e > s;  // e <= t0: the other warp's tile (kAlt)
            const uint32_t end_mask = __ballot_sync(0xFFFFFFFFu, ends);
            const uint32_t ne_mask = __ballot_sync(0xFFFFFFFFu, nonempty);
            if (nonempty) {
              const int slot = nseg + __popc(ne_mask & ((1u << lane) - 1u));
              meta->seg_end[slot] = static_cast<int16_t>(e - t0);
              meta->seg_doc[slot] = static_cast<int32_t>(d);
            }
            nseg += __popc(ne_mask);
            const int consumed = __popc(end_mask);  // ends are monotone: a prefix of the lanes
            next_doc += consumed;
            if (consumed < 32) break;
          }
          if (st.side) next_doc1 = next_doc;
          else next_doc0 = next_doc;
          if (lane == 0) {
            meta->nseg = nseg;
            meta->valid = valid;
          }
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          if (!kPre) mbar_arrive(&full[stg.idx]);
          mbar_arrive(&raw_empty[raw.idx]);
        }
        // With TMA operand tiles the MMA warp also commits the tile's products to m_full, so that one
        // barrier tells the epilogue both that the metadata is written and that the accumulators are
        // ready: one wait per tile on the epilogue's critical path, and no relay through this warp.
        if (lane == 0) mbar_arrive(&m_full[mst.idx]);
        raw.next<kRaw>();
        stg.next<L::stages>();
        mst.next<kMeta>();
      }
      if ((kAlt || xwarp == 0) && lane == 0) {
        for (int side = 0; side < (kTwin ? 2 : 1); ++side) mbar_arrive(&u_empty[kTwin ? side : (iter & 1)]);
      }
    }
  } else if (warp == kMmaWarp) {
    // =================== MMA issuer ===================
    // instruction descriptors: D s32, A/B s8 (kind::i8) or D f32, A/B f16 (kind::f16); K-major; N, M
    constexpr uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kTileN >> 3) << 17) |
                               (static_cast<uint32_t>(128 >> 4) << 24);
    constexpr uint32_t idesc16 = (1u << 4) | (static_cast<uint32_t>(kTileN >> 3) << 17) |
                                 (static_cast<uint32_t>(128 >> 4) << 24);
    // Descriptors are formed once: their start-address field is the shared-memory address / 16, so an
    // operand offset of 32 bytes along K adds 2 and a stage offset adds stage * b_tile / 16 (addresses stay
    // below 2^18, so the 14-bit field never carries into the next one).
    const uint64_t b_desc0 = umma_desc(smem_u32(smem + L::off_b), 16u, 1024u);
    const uint64_t c_desc = kBias ? umma_desc_plain(smem_u32(smem + L::off_bias)) : 0ull;
    Ring stg, acc, mst;
    int iter = 0;
    for (int w = blockIdx.x; w < p.num_items; w += gridDim.x, ++iter) {
      const Item it = load_item<kTwin>(p, w);
      const int abuf = iter % L::a_bufs;
      // query tiles of the pair that hold at least one query
      const int n_tiles = min(kG, (p.batch - it.un[0].qpair * kG * p.qpt + p.qpt - 1) / p.qpt);
      if (!mbar_wait(&a_full[abuf], (iter / L::a_bufs) & 1, abort_flag, p.error, 21)) goto done;
      const uint32_t a_addr = smem_u32(smem + L::off_a + abuf * kG * L::a_tile);
      for (int64_t i = 0; i < it.nsteps; ++i) {
        const Step st = step_of<kTwin>(it, i);
        if (!mbar_wait(&full[stg.idx], stg.phase, abort_flag, p.error, 22)) goto done;
        // twin mode: the steps of sides 0 and 1 share one accumulator buffer (slots 0 and 1)
        if ((!kTwin || st.side == 0) && !mbar_wait(&acc_empty[acc.idx], acc.phase ^ 1, abort_flag, p.error, 23))
          goto done;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t b_addr = smem_u32(smem + L::off_b + stg.idx * L::b_tile);
          // twin mode: query tile 0 against this side's tile, into slot `side`; an empty tile issues nothing
          const int g_first = kTwin ? st.side : 0;
          const int g_end = kTwin ? (st.valid > 0 ? st.side + 1 : st.side) : n_tiles;
          for (int g = g_first; g < g_end; ++g) {
            // accumulator of (query tile g, stream 0); the residual stream's follows it
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>((acc.idx * kG + g) * kStreams * kTileN);
            const uint32_t ag = a_addr + static_cast<uint32_t>((kTwin ? 0 : g) * L::a_tile);
            if (kF16) {
              // 8 steps of K = 16 f16 (32 bytes): 4 per 128-byte K half, the halves 16 KB apart
#pragma unroll
              for (int k = 0; k < 8; ++k) {
                const uint32_t off = static_cast<uint32_t>((k >> 2) * kBTileBytes + 32 * (k & 3));
                const uint64_t ad = umma_desc(ag + off, 16u, 1024u);
                const uint64_t bd = umma_desc(b_addr + off, 16u, 1024u);
                mma_f16(d_tmem, ad, bd, idesc16, k > 0 ? 1u : 0u);
              }
            } else {
              // every accumulator opens at kBiasValue: constant x constant, K = 32
              // (expanding path: unsigned 0xFF operands, A and B formats 0 = u8)
              if (kBias) mma_i8(d_tmem, c_desc, c_desc, kPre ? idesc : (idesc & ~((7u << 7) | (7u << 10))), 0u);
              const uint64_t ad0 = umma_desc(ag, 16u, 1024u);
              const uint64_t bd0 = b_desc0 + static_cast<uint64_t>((stg.idx * L::b_tile) >> 4);
#pragma unroll
              for (int sm = 0; sm < kStreams; ++sm) {  // prefix tile; residual tile 16 KB after it
#pragma unroll
                for (int k = 0; k < 4; ++k)
                  mma_i8(d_tmem + static_cast<uint32_t>(sm * kTileN), ad0 + 2u * k,
                         bd0 + static_cast<uint64_t>((sm * kBTileBytes) >> 4) + 2u * k, idesc,
                         (kBias || k > 0) ? 1u : 0u);
              }
            }
          }
          mma_commit(&tile_done[stg.idx]);
          if (kPre) mma_commit(&m_full[mst.idx]);  // the accumulators are ready for the epilogue
        }
        __syncwarp();
        stg.next<L::stages>();
        mst.next<kMeta>();
        if (!kTwin || st.side == 1) acc.next<kAcc>();
      }
      if (lane == 0) mma_commit(&a_empty[abuf]);
      __syncwarp();
    }
  } else {
    // =================== epilogue: warps 0-7; query tile g = warp / 4, TMEM lane quarter warp % 4 ===========
    // 16x256b TMEM loads: thread t holds rows R(i) = 32 (warp % 4) + 16 (i / 2) + 8 (i % 2) + t / 4,
    // i = 0..3, and per 64-column chunk the 16 columns 8j + 2(t % 4) + {0, 1}, so it needs 16 token
    // scales per chunk instead of 64.  A row's maximum is completed across the four threads
    // t % 4 = 0..3 with two butterfly shuffles when a document ends.
    const int q4 = warp & 3;
    const int g = warp >> 2;                      // query tile of the pair
    const int rq = q4 % kQuarters;                // kRep > 1: the quarter of distinct rows this warp holds
    const int slice = q4 / kQuarters;             //           and its slice of 128 / kRep columns
    const int etid = threadIdx.x;                 // 0..255
    const int tq = lane >> 2, tc = lane & 3;
    const uint32_t lane_base = static_cast<uint32_t>(q4 * 32) << 16;
    Ring stg, acc, mst;
    // Barrier among the epilogue warps around a document flush: an mbarrier with bounded waits, so a
    // warp that gives up on a timeout never leaves the others waiting for good.  In twin mode each
    // group flushes its own unit's documents, with its own barrier and document-id slots.
    uint64_t* const flush_bar = epi_bar + (kTwin ? g : 0);
    int32_t* const gdoc = group_doc + (kTwin ? g * kSegGroup : 0);
    const int ftid = kTwin ? etid - 128 * g : etid;            // thread index among the flushing threads
    const int fthreads = kTwin ? 128 : kEpiWarps * 32;
    uint32_t epi_phase = 0;
    auto epi_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(flush_bar);
      const bool ok = mbar_wait(flush_bar, epi_phase, abort_flag, p.error, 33);
      epi_phase ^= 1u;
      return ok;
    };
    for (int w = blockIdx.x; w < p.num_items; w += gridDim.x) {
      const Item it = load_item<kTwin>(p, w);
      const Unit& unit = (kTwin && g) ? it.un[1] : it.un[0];
      const int tile = kTwin ? 0 : unit.qpair * kG + g;  // twin mode: both groups score query tile 0
      // Rows of this warp's TMEM lane quarter that hold query tokens; a quarter without any (small
      // batches) skips its loads and arithmetic and only walks the document ends with the others.
      const int tile_rows = max(0, min(p.qpt, p.batch - tile * p.qpt)) * Q;
      const bool tile_live = (kDigits ? 8 * q4 : 32 * rq) < tile_rows;
      // the row this thread stores when a document ends: i = t % 4 (digit planes: the one query row of
      // the four lanes, stored by t % 4 = 0)
      const int wrow = kDigits ? 8 * q4 + tq : rq * 32 + 16 * (tc >> 1) + 8 * (tc & 1) + tq;
      const int wslot = kDigits ? wrow : q4 * 32 + 16 * (tc >> 1) + 8 * (tc & 1) + tq;  // its TMEM lane
      const bool w_store = !kDigits || tc == 0;
      const int wb = tile * p.qpt + wrow / Q;
      const bool w_valid = wrow < p.qpt * Q && wb < p.batch;
      // (biased digit planes without token scales: row values are 2^-23 x, the query scale 2^23 x; exact)
      constexpr float kQsFold = (kDigits && kBias && !kTokenScale) ? 8388608.0F : 1.0F;
      const float qs = w_valid ? __ldg(p.qscale + static_cast<int64_t>(wb) * Q + wrow % Q) * kQsFold : 0.0F;
      const int nq0 = max(0, min(p.qpt, p.batch - (unit.qpair * kG) * p.qpt));
      const int nq1 = kTwin ? 0 : max(0, min(p.qpt, p.batch - (unit.qpair * kG + 1) * p.qpt));
      const int nq = nq0 + nq1;
      float run[4] = {kLowest, kLowest, kLowest, kLowest};                // open document, per row
      float tk[kTk];                                                      // TopK: open document's list
      int tk_cnt = 0;                                                     // TopK: its tokens in my columns
      float sm_m = kLowest, sm_s = 0.0F;                                  // SmoothSim: open document's state
      const float sm_v = qs * p.smooth_scale;                             // SmoothSim: digit units -> values
      // exponent units in base 2: exp((v - m) / t) = exp2((u - m_u) * qscale * scale * log2(e) / t)
      const float sm_c = sm_v * 1.4426950408889634F / p.temperature;
#pragma unroll
      for (int i = 0; i < kTk; ++i) tk[i] = kLowest;
      int32_t run_i[4] = {INT32_MIN, INT32_MIN, INT32_MIN, INT32_MIN};    // tensor-scale variant
      int pending = 0;
      for (int64_t si = 0; si < it.nsteps; ++si) {
        const Step st = step_of<kTwin>(it, si);
        if (kTwin && st.side != g) {
          // the other group's tile: keep the rings in step without touching its barriers
          stg.next<L::stages>();
          if (st.side == 1) acc.next<kAcc>();
          mst.next<kMeta>();
          continue;
        }
        if (!kPre && !mbar_wait(&tile_done[stg.idx], stg.phase, abort_flag, p.error, 31)) goto done;
        // Acquire the expanders' metadata writes for this tile (meta ring slot) and, with TMA operand
        // tiles, the completion of its MMAs (the MMA warp's commit is the slot's last arrival).
        if (!mbar_wait(&m_full[mst.idx], mst.phase, abort_flag, p.error, 32)) goto done;
        tc_fence_after();
        const StageMeta* meta = reinterpret_cast<const StageMeta*>(smem + L::off_meta + mst.idx * kMetaBytes);
        const int valid = meta->valid;
        const int nseg = meta->nseg;
        const bool last_tile = st.last;
        const uint32_t tbase =
            tmem_base + lane_base + static_cast<uint32_t>((acc.idx * kG + g) * kStreams * kTileN);
        int sgi = 0;
        bool released = false;
#pragma unroll
        for (int ci = 0; ci < kChunks; ++ci) {
          // kRep == 1: two 64-column chunks; kRep > 1: this warp's slice of the tile, possibly empty
          const int c0 = kRep == 1 ? 64 * ci : slice * (128 / kRep);
          if (kRep == 1 && c0 >= valid) break;
          const int c1 = max(c0, min(c0 + kChunkCols, valid));  // this chunk's valid columns [c0, c1)
          uint32_t ra[4 * kNJ], rb[4 * kNJ];  // lanes +0..15 (rows i = 0, 1) and +16..31 (rows i = 2, 3)
          if (tile_live && c1 > c0) {
            float2 sc[kNJ], sc2[kNJ];
            if (kTokenScale) {
              const float* s2base = reinterpret_cast<const float*>(smem + L::off_scale2 + mst.idx * 160 * 4);
              // columns c0 + 8j + 2(t % 4) + {0, 1}: slots from (c0 / 64) * 80 + (t % 4) * 20 + ((c0 % 64) / 8) * 2
              const int sb = (c0 >> 6) * 80 + tc * 20 + ((c0 & 63) >> 3) * 2;
#pragma unroll
              for (int k4 = 0; k4 < kNJ / 2; ++k4) {
                const float4 x = *reinterpret_cast<const float4*>(meta->scale + sb + 4 * k4);
                sc[2 * k4] = make_float2(x.x, x.y);
                sc[2 * k4 + 1] = make_float2(x.z, x.w);
                if (kRes) {  // the residual stream's scales, in the same slots
                  const float4 y = *reinterpret_cast<const float4*>(s2base + sb + 4 * k4);
                  sc2[2 * k4] = make_float2(y.x, y.y);
                  sc2[2 * k4 + 1] = make_float2(y.z, y.w);
                }
              }
            }
            if constexpr (kNJ == 8) {
              tmem_ld16x256b_x8(tbase + c0, ra);
              tmem_ld16x256b_x8(tbase + (16u << 16) + c0, rb);
            } else {
              tmem_ld16x256b_x4(tbase + c0, ra);
              tmem_ld16x256b_x4(tbase + (16u << 16) + c0, rb);
            }
            tmem_wait_ld();
            float v1[2 * kNJ];  // residual stream: the prefix's combined digit dots of this thread's row
            if (kRes) {
#pragma unroll
              for (int j = 0; j < kNJ; ++j) {
#pragma unroll
                for (int b2 = 0; b2 < 2; ++b2) {
                  const int32_t d0 = static_cast<int32_t>(ra[4 * j + b2]);
                  const int32_t d1 = static_cast<int32_t>(ra[4 * j + 2 + b2]);
                  const int32_t d2 = static_cast<int32_t>(rb[4 * j + b2]);
                  v1[2 * j + b2] = __fmaf_rn(__int2float_rn(d2), 65536.0F, __int2float_rn(d0 + 256 * d1));
                }
              }
              tmem_ld16x256b_x8(tbase + kTileN + c0, ra);  // the residual stream's accumulator
              tmem_ld16x256b_x8(tbase + kTileN + (16u << 16) + c0, rb);
              tmem_wait_ld();
            }
            if (kRep > 1 || c0 + 64 >= valid) {
              // last chunk of the tile is in registers: hand the accumulators back to the MMA now
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&acc_empty[acc.idx]);
              released = true;
            }
            if (kDigits && kBias) {
              // biased planes: each exactly d * 2^-23 by one packed FMA; then fl(d0 + 256 d1) and
              // fl(that + 65536 d2) by two more, the same roundings as the int32 / fmaf path below, scaled by
              // 2^-23 (token scales are staged as s * 2^23, so fl(v * s) comes out unscaled; without token
              // scales the row values stay 2^-23 x and the query scale takes the 2^23)
#pragma unroll
              for (int j = 0; j < kNJ; ++j) {
                const float2 p0 = bias_unscale2<!kPre>(ra[4 * j], ra[4 * j + 1]);
                const float2 p1 = bias_unscale2<!kPre>(ra[4 * j + 2], ra[4 * j + 3]);
                const float2 p2 = bias_unscale2<!kPre>(rb[4 * j], rb[4 * j + 1]);
                float2 v = __ffma2_rn(p2, make_float2(65536.0F, 65536.0F),
                                      __ffma2_rn(p1, make_float2(256.0F, 256.0F), p0));
                if (kTokenScale) v = __fmul2_rn(v, sc[j]);
                ra[4 * j] = __float_as_uint(v.x);
                ra[4 * j + 1] = __float_as_uint(v.y);
              }
            } else if (kDigits) {
              // rows 0, 1, 2 are the digit planes' exact dots: d0 + 256 d1 is exact in int32 (|d| <= 2^17),
              // one rounding to float and one fused multiply-add, then fl(dot * s_t); the result in row 0
#pragma unroll
              for (int j = 0; j < kNJ; ++j) {
#pragma unroll
                for (int b2 = 0; b2 < 2; ++b2) {
                  const int32_t d0 = static_cast<int32_t>(ra[4 * j + b2]);
                  const int32_t d1 = static_cast<int32_t>(ra[4 * j + 2 + b2]);
                  const int32_t d2 = static_cast<int32_t>(rb[4 * j + b2]);
                  // expanding path: 16 x the dots, so d0 + 256 d1 >> 4 and d2 * 2^12 (both exact)
                  float v = kPre ? __fmaf_rn(__int2float_rn(d2), 65536.0F, __int2float_rn(d0 + 256 * d1))
                                 : __fmaf_rn(__int2float_rn(d2), 4096.0F, __int2float_rn((d0 + 256 * d1) >> 4));
                  if (kRes) {
                    // fl(fl(fl(v1 * scale1) * s1) + fl(fl(v2 * scale2) * s2)), as the SIMT kernel orders it
                    const float a = __fmul_rn(__fmul_rn(v1[2 * j + b2], p.res_scale1), b2 ? sc[j].y : sc[j].x);
                    const float b = __fmul_rn(__fmul_rn(v, p.res_scale2), b2 ? sc2[j].y : sc2[j].x);
                    v = __fadd_rn(a, b);
                  } else if (kTokenScale) {
                    v = __fmul_rn(v, b2 ? sc[j].y : sc[j].x);
                  }
                  ra[4 * j + b2] = __float_as_uint(v);
                }
              }
            } else if (kBias) {
              // (dot + kBiasValue) bits -> fl(dot * s_t): two packed instructions per two columns
#pragma unroll
              for (int j = 0; j < kNJ; ++j) {
                bias_scale2<!kPre>(ra[4 * j], ra[4 * j + 1], sc[j]);
                bias_scale2<!kPre>(ra[4 * j + 2], ra[4 * j + 3], sc[j]);
                bias_scale2<!kPre>(rb[4 * j], rb[4 * j + 1], sc[j]);
                bias_scale2<!kPre>(rb[4 * j + 2], rb[4 * j + 3], sc[j]);
              }
            } else if (kTokenScale) {
              // exact int32 dot -> float (all 64 first; expanding path: 16 x dot, shifted back first), then
              // fl(dot * s_t); f16 operands accumulate the
              // same integer exactly in fp32 (|products| <= 1016, |sums| < 2^17), so nothing to convert
              if (!kF16) {
#pragma unroll
                for (int k = 0; k < 4 * kNJ; ++k) {
                  ra[k] = __float_as_uint(__int2float_rn(static_cast<int32_t>(ra[k]) >> (kPre ? 0 : 4)));
                  rb[k] = __float_as_uint(__int2float_rn(static_cast<int32_t>(rb[k]) >> (kPre ? 0 : 4)));
                }
              }
              // fl(dot * s_t) two columns at a time (packed products round each element as a scalar one)
#pragma unroll
              for (int j = 0; j < kNJ; ++j) {
#pragma unroll
                for (int e = 0; e < 4; e += 2) {
                  const float2 x = __fmul2_rn(make_float2(__uint_as_float(ra[4 * j + e]), __uint_as_float(ra[4 * j + e + 1])), sc[j]);
                  const float2 y = __fmul2_rn(make_float2(__uint_as_float(rb[4 * j + e]), __uint_as_float(rb[4 * j + e + 1])), sc[j]);
                  ra[4 * j + e] = __float_as_uint(x.x);
                  ra[4 * j + e + 1] = __float_as_uint(x.y);
                  rb[4 * j + e] = __float_as_uint(y.x);
                  rb[4 * j + e + 1] = __float_as_uint(y.y);
                }
              }
            }
          }
          if (!kList && nseg == 0 && tile_live && c1 == c0 + kChunkCols) {
            // no document ends in this tile and the open document covers the whole chunk: no walk
            if (kFloat) {
              run[0] = row_max16<kNJ>(ra, 0, run[0]);
              if (!kDigits) {
                run[1] = row_max16<kNJ>(ra, 1, run[1]);
                run[2] = row_max16<kNJ>(rb, 0, run[2]);
                run[3] = row_max16<kNJ>(rb, 1, run[3]);
              }
            } else {
              run_i[0] = row_max16i<kNJ>(ra, 0, run_i[0]);
              run_i[1] = row_max16i<kNJ>(ra, 1, run_i[1]);
              run_i[2] = row_max16i<kNJ>(rb, 0, run_i[2]);
              run_i[3] = row_max16i<kNJ>(rb, 1, run_i[3]);
            }
            continue;
          }
          int a = c0;
          bool carry = false;        // the document opened inside this chunk already holds [e, c1)
          float carry_max[4];
          while (true) {
            const int e = nseg == 0 ? 0x7FFF : (sgi < nseg ? meta->seg_end[sgi] : 0x7FFF);
            const int bnd = min(e, c1);
            const bool split = !kList && kFloat && tile_live && a == c0 && c1 == c0 + kChunkCols && e > c0 && e < c1 &&
                               (sgi + 1 < nseg ? meta->seg_end[sgi + 1] : 0x7FFF) > c1;
            if (split) {
              // Exactly one document ends strictly inside the chunk: one pass sends each value to the
              // closing document (columns < e) or to the one that opens (columns >= e), each side
              // reduced by three-input maxima.
              const int le = e - c0 - 2 * tc;  // element (j, b) is column c0 + 8j + 2(t % 4) + b
              float lo[4][2], hi[4][2];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                lo[i][0] = lo[i][1] = hi[i][0] = hi[i][1] = kLowest;
              }
#pragma unroll
              for (int j = 0; j < kNJ; ++j) {
                const bool in0 = 8 * j < le, in1 = 8 * j + 1 < le;
#pragma unroll
                for (int i = 0; i < kRows; ++i) {
                  const uint32_t* X = i < 2 ? ra : rb;
                  const float v0 = __uint_as_float(X[4 * j + 2 * (i & 1)]);
                  const float v1 = __uint_as_float(X[4 * j + 2 * (i & 1) + 1]);
                  lo[i][j & 1] = fmax3(lo[i][j & 1], in0 ? v0 : kLowest, in1 ? v1 : kLowest);
                  hi[i][j & 1] = fmax3(hi[i][j & 1], in0 ? kLowest : v0, in1 ? kLowest : v1);
                }
              }
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                run[i] = fmax3(run[i], lo[i][0], lo[i][1]);
                carry_max[i] = fmaxf(hi[i][0], hi[i][1]);
              }
              carry = true;
              a = e;
            } else if (bnd > a && tile_live) {
              if (kSmooth && a == c0 && bnd == c0 + kChunkCols) {
                // the whole chunk inside the open document: no column tests, two partial sums
                const float mn = fmaxf(sm_m, row_max16<kNJ>(ra, 0, kLowest));
                float acc0 = sm_s > 0.0F ? sm_s * exp2f((sm_m - mn) * sm_c) : 0.0F, acc1 = 0.0F;
#pragma unroll
                for (int j = 0; j < kNJ; ++j) {
                  acc0 += exp2f((__uint_as_float(ra[4 * j]) - mn) * sm_c);
                  acc1 += exp2f((__uint_as_float(ra[4 * j + 1]) - mn) * sm_c);
                }
                sm_m = mn;
                sm_s = acc0 + acc1;
              } else if (kSmooth) {
                // columns [a, bnd) of the open document into this thread's running log-sum-exp, in the
                // row's digit-plane units u (v = u * qscale * scale): the segment's maximum first, then
                // s = s * 2^((m - m') c) + sum 2^((u - m') c), c = qscale * scale * log2(e) / temperature
                const int la = a - c0 - 2 * tc, lb = bnd - c0 - 2 * tc;
                float mx = kLowest;
                bool any = false;
#pragma unroll
                for (int j = 0; j < kNJ; ++j) {
#pragma unroll
                  for (int b2 = 0; b2 < 2; ++b2) {
                    const int cc = 8 * j + b2;
                    const bool in = cc >= la && cc < lb;
                    mx = in ? fmaxf(mx, __uint_as_float(ra[4 * j + b2])) : mx;
                    any = any || in;
                  }
                }
                if (any) {
                  const float mn = fmaxf(sm_m, mx);
                  float acc_s = sm_s > 0.0F ? sm_s * exp2f((sm_m - mn) * sm_c) : 0.0F;
#pragma unroll
                  for (int j = 0; j < kNJ; ++j) {
#pragma unroll
                    for (int b2 = 0; b2 < 2; ++b2) {
                      const int cc = 8 * j + b2;
                      if (cc >= la && cc < lb) acc_s += exp2f((__uint_as_float(ra[4 * j + b2]) - mn) * sm_c);
                    }
                  }
                  sm_m = mn;
                  sm_s = acc_s;
                }
              } else if (kTopK && a == c0 && bnd == c0 + kChunkCols) {
                // the whole chunk inside the open document: every column, no tests
#pragma unroll
                for (int j = 0; j < kNJ; ++j) {
                  topk_insert<kTk>(tk, __uint_as_float(ra[4 * j]));
                  topk_insert<kTk>(tk, __uint_as_float(ra[4 * j + 1]));
                }
                tk_cnt += 2 * kNJ;
              } else if (kTopK) {
                // columns [a, bnd) of the open document into this thread's list
                const int la = a - c0 - 2 * tc, lb = bnd - c0 - 2 * tc;
#pragma unroll
                for (int j = 0; j < kNJ; ++j) {
#pragma unroll
                  for (int b2 = 0; b2 < 2; ++b2) {
                    const int cc = 8 * j + b2;
                    if (cc >= la && cc < lb) {
                      topk_insert<kTk>(tk, __uint_as_float(ra[4 * j + b2]));
                      ++tk_cnt;
                    }
                  }
                }
              } else if (a == c0 && bnd == c0 + kChunkCols) {
                // whole chunk inside one document: two independent chains per row
                if (kFloat) {
                  run[0] = row_max16<kNJ>(ra, 0, run[0]);
                  if (!kDigits) {
                    run[1] = row_max16<kNJ>(ra, 1, run[1]);
                    run[2] = row_max16<kNJ>(rb, 0, run[2]);
                    run[3] = row_max16<kNJ>(rb, 1, run[3]);
                  }
                } else {
                  run_i[0] = row_max16i<kNJ>(ra, 0, run_i[0]);
                  run_i[1] = row_max16i<kNJ>(ra, 1, run_i[1]);
                  run_i[2] = row_max16i<kNJ>(rb, 0, run_i[2]);
                  run_i[3] = row_max16i<kNJ>(rb, 1, run_i[3]);
                }
              } else {
                const int la = a - c0 - 2 * tc, lb = bnd - c0 - 2 * tc;  // element (j, b) is column 8j + b here
#pragma unroll
                for (int j = 0; j < kNJ; ++j) {
#pragma unroll
                  for (int b2 = 0; b2 < 2; ++b2) {
                    const int cc = 8 * j + b2;
                    const bool in = cc >= la && cc < lb;
                    if (kFloat) {
                      run[0] = in ? fmaxf(run[0], __uint_as_float(ra[4 * j + b2])) : run[0];
                      if (!kDigits) {
                        run[1] = in ? fmaxf(run[1], __uint_as_float(ra[4 * j + 2 + b2])) : run[1];
                        run[2] = in ? fmaxf(run[2], __uint_as_float(rb[4 * j + b2])) : run[2];
                        run[3] = in ? fmaxf(run[3], __uint_as_float(rb[4 * j + 2 + b2])) : run[3];
                      }
                    } else {
                      run_i[0] = in ? max(run_i[0], static_cast<int32_t>(ra[4 * j + b2])) : run_i[0];
                      run_i[1] = in ? max(run_i[1], static_cast<int32_t>(ra[4 * j + 2 + b2])) : run_i[1];
                      run_i[2] = in ? max(run_i[2], static_cast<int32_t>(rb[4 * j + b2])) : run_i[2];
                      run_i[3] = in ? max(run_i[3], static_cast<int32_t>(rb[4 * j + 2 + b2])) : run_i[3];
                    }
                  }
                }
              }
            }
            if (!split && bnd > a) a = bnd;
            // the open document continues past this chunk (or no ends are left); with replicated rows a
            // warp's one slice is its only chunk, so it also takes the ends after its slice (documents
            // that hold no further columns of it), keeping every warp's flushes in step
            if (e > (kRep > 1 ? valid : c1)) break;
            // document meta->seg_doc[sgi] ends: complete each row's maximum across the four threads
            // holding it, stage the row value scaled by the query scale, flush finished documents.
            float best;
            if (kSmooth) {
              // merge the four threads' (maximum, sum) pairs, then max + temperature * log(sum) in the
              // document's units
#pragma unroll
              for (int delta = 1; delta <= 2; delta <<= 1) {
                const float om = __shfl_xor_sync(0xFFFFFFFFu, sm_m, delta);
                const float os = __shfl_xor_sync(0xFFFFFFFFu, sm_s, delta);
                const float mn = fmaxf(sm_m, om);
                sm_s = (sm_s > 0.0F ? sm_s * exp2f((sm_m - mn) * sm_c) : 0.0F) +
                       (os > 0.0F ? os * exp2f((om - mn) * sm_c) : 0.0F);
                sm_m = mn;
              }
              best = sm_s > 0.0F ? sm_m * sm_v + p.temperature * logf(sm_s) : 0.0F;
            } else if (kTopK) {
              // merge the four threads' lists and counts, then the mean of the top min(K, tokens)
#pragma unroll
              for (int delta = 1; delta <= 2; delta <<= 1) {
                float other[kTk];
#pragma unroll
                for (int i = 0; i < kTk; ++i) other[i] = __shfl_xor_sync(0xFFFFFFFFu, tk[i], delta);
                tk_cnt += __shfl_xor_sync(0xFFFFFFFFu, tk_cnt, delta);
#pragma unroll
                for (int i = 0; i < kTk; ++i) topk_insert<kTk>(tk, other[i]);
              }
              const int c = min(kTk, tk_cnt);
              float total = 0.0F;
#pragma unroll
              for (int i = 0; i < kTk; ++i)
                if (i < c) total = __fadd_rn(total, tk[i]);
              best = c > 0 ? __fdiv_rn(total, static_cast<float>(c)) : 0.0F;
            } else if (kFloat) {
#pragma unroll
              for (int i = 0; i < kRows; ++i) {
                run[i] = fmaxf(run[i], __shfl_xor_sync(0xFFFFFFFFu, run[i], 1));
                run[i] = fmaxf(run[i], __shfl_xor_sync(0xFFFFFFFFu, run[i], 2));
              }
              best = kDigits ? run[0] : tc == 0 ? run[0] : tc == 1 ? run[1] : tc == 2 ? run[2] : run[3];
            } else {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                run_i[i] = max(run_i[i], __shfl_xor_sync(0xFFFFFFFFu, run_i[i], 1));
                run_i[i] = max(run_i[i], __shfl_xor_sync(0xFFFFFFFFu, run_i[i], 2));
              }
              const int32_t bi = tc == 0 ? run_i[0] : tc == 1 ? run_i[1] : tc == 2 ? run_i[2] : run_i[3];
              best = bi == INT32_MIN ? kLowest : __int2float_rn(bi >> (kPre ? 0 : 4));  // expanding: 16 x dot
            }
            if (w_store) rowval[(pending * kG + g) * 128 + wslot] = w_valid ? (kSmooth ? best : __fmul_rn(best, qs)) : 0.0F;
            if (ftid == 0) gdoc[pending] = meta->seg_doc[sgi];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              run[i] = carry ? carry_max[i] : kLowest;
              run_i[i] = INT32_MIN;
            }
#pragma unroll
            for (int i = 0; i < kTk; ++i) tk[i] = kLowest;
            tk_cnt = 0;
            sm_m = kLowest;
            sm_s = 0.0F;
            if (carry) {
              carry = false;
              a = c1;
            }
            ++sgi;
            if (++pending == kSegGroup || (sgi == nseg && last_tile)) {
              if (!epi_sync()) goto done;
              if (kFuse) {
                // fused top-k: one thread per query takes the group's documents in turn into its list
                const int K = p.topk_k;
                for (int qx = ftid; qx < nq; qx += fthreads) {
                  const int gq = qx < nq0 ? 0 : 1;
                  const int qq = qx < nq0 ? qx : qx - nq0;
                  const float* rvq = rowval + (kTwin ? g : gq) * 128 + qq * Q;
                  const int b = (unit.qpair * kG + gq) * p.qpt + qq;
                  float* ls = tks + ((kTwin ? g : 0) * p.batch + b) * K;
                  int32_t* li = tki + ((kTwin ? g : 0) * p.batch + b) * K;
                  for (int gd = 0; gd < pending; ++gd) {
                    const float* rv = rvq + gd * kG * 128;
                    float sacc = 0.0F;
                    for (int r = 0; r < Q; ++r) sacc = __fadd_rn(sacc, rep_max<kRep>(rv, r));
                    const float sc = __fmul_rn(sacc, p.scale);
                    const uint32_t key = float_to_ordered(sc);
                    const int32_t dd = gdoc[gd];
                    auto worse = [&](int i) {  // entry i loses to the candidate
                      const int32_t di = li[i];
                      if (di < 0) return true;
                      const uint32_t ki = float_to_ordered(ls[i]);
                      return key > ki || (key == ki && dd < di);
                    };
                    if (!worse(K - 1)) continue;
                    int pos = K - 1;
                    while (pos > 0 && worse(pos - 1)) {
                      ls[pos] = ls[pos - 1];
                      li[pos] = li[pos - 1];
                      --pos;
                    }
                    ls[pos] = sc;
                    li[pos] = dd;
                  }
                }
              } else
              for (int x = ftid; x < pending * nq; x += fthreads) {
                const int gd = x / nq, qx = x % nq;
                const int gq = qx < nq0 ? 0 : 1;
                const int qq = qx < nq0 ? qx : qx - nq0;
                // twin mode: the group's own row values (slot g) of query tile 0
                const float* rv = rowval + (gd * kG + (kTwin ? g : gq)) * 128 + qq * Q;
                // row order as the reference sums; the loads are issued ahead of the dependent additions
                float sacc = 0.0F;
                int k = 0;
                for (; k + 8 <= Q; k += 8) {
                  float v[8];
#pragma unroll
                  for (int i = 0; i < 8; ++i) v[i] = rep_max<kRep>(rv, k + i);
#pragma unroll
                  for (int i = 0; i < 8; ++i) sacc = __fadd_rn(sacc, v[i]);
                }
                for (; k < Q; ++k) sacc = __fadd_rn(sacc, rep_max<kRep>(rv, k));
                p.out[static_cast<int64_t>((unit.qpair * kG + gq) * p.qpt + qq) * p.num_docs + gdoc[gd]] =
                    __fmul_rn(sacc, p.scale);
              }
              if (!epi_sync()) goto done;
              pending = 0;
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (!released) mbar_arrive(&acc_empty[acc.idx]);
          mbar_arrive(&m_empty[mst.idx]);
        }
        stg.next<L::stages>();
        if (!kTwin || st.side == 1) acc.next<kAcc>();
        mst.next<kMeta>();
      }
    }
    if (kFuse) {
      // this CTA's (group's) lists as one candidate block: [B, k] fp32 scores, then [B, k] int64 documents
      // (an empty entry: -inf, INT64_MAX)
      if (!epi_sync()) goto done;
      const int K = p.topk_k, lg = kTwin ? g : 0;
      unsigned char* blk = p.cand + static_cast<size_t>(blockIdx.x * kLists + lg) * 16ull * p.batch * K;
      const float* ls = tks + lg * p.batch * K;
      const int32_t* li = tki + lg * p.batch * K;
      for (int e = ftid; e < p.batch * K; e += fthreads) {
        const bool full = li[e] >= 0;
        reinterpret_cast<float*>(blk)[e] = full ? ls[e] : -INFINITY;
        reinterpret_cast<int64_t*>(blk + 8ull * p.batch * K)[e] = full ? static_cast<int64_t>(li[e]) : INT64_MAX;
      }
    }
  }
done:
  // On abort, outstanding MMAs and bulk copies finish on their own; give them
  // time to land before TMEM is released and the CTA exits.
  if ((warp == kMmaWarp || warp == kLoadWarp) && *abort_flag) {
    const uint64_t t0 = global_ns();
    while (global_ns() - t0 < 2000000ull) {
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                 : "memory");
  }
}

}  // namespace tc

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {

struct TcPlan {
  int qpt;
  int n_qtiles;
  int n_pairs;
  int64_t n_ranges;  // token-quantile document ranges before the per-range document cap
};

constexpr int kMaxDevices = 64;

int sm_count() {
  static std::atomic<int> cached[kMaxDevices] = {};  // per device, queried once
  int dev = 0, sms = 0;
  check(cudaGetDevice(&dev), "get device");
  if (dev >= 0 && dev < kMaxDevices && (sms = cached[dev].load(std::memory_order_relaxed)) > 0) return sms;
  check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "query SM count");
  if (dev >= 0 && dev < kMaxDevices) cached[dev].store(sms, std::memory_order_relaxed);
  return sms;
}

// The dynamic shared-memory limit of a kernel, raised once per (device, kernel) to the most it was asked for.
void raise_smem_limit(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::vector<std::pair<std::pair<int, const void*>, int>> raised;
  int dev = 0;
  check(cudaGetDevice(&dev), "get device");
  std::lock_guard<std::mutex> lock(mu);
  for (auto& e : raised)
    if (e.first.first == dev && e.first.second == kernel) {
      if (e.second >= bytes) return;
      check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), "set tc smem");
      e.second = bytes;
      return;
    }
  check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), "set tc smem");
  raised.push_back({{dev, kernel}, bytes});
}

TcPlan plan_for(const DocsView& d, const QueryView& q, int sms) {
  TcPlan pl{};
  // int8 queries: 128 query rows per tile; fp32 queries as digit planes: 32 (four TMEM lanes a row)
  pl.qpt = (q.mode == kQueryF32 ? 32 : 128) / q.qtok;
  pl.n_qtiles = (q.batch + pl.qpt - 1) / pl.qpt;
  pl.n_pairs = (pl.n_qtiles + tc::kG - 1) / tc::kG;
  // 2 x SM-count ranges: every CTA gets 2 * n_pairs equal units; ranges of
  // fewer than 8 tiles only for small corpora.
  pl.n_ranges = std::max<int64_t>(1, std::min<int64_t>(2LL * sms, d.num_tokens / (8 * tc::kTileN)));
  return pl;
}

}  // namespace

// Replicated query rows for one small tile of int8 query rows (option tc_row_replicas, on by default).
static std::atomic<int> g_tc_row_replicas{1};
void set_tc_row_replicas(int on) { g_tc_row_replicas.store(on); }
int get_tc_row_replicas() { return g_tc_row_replicas.load(); }

bool tc_int8_cache_supported(const DocsView& d) {
  // TMA row coordinates are 32-bit
  return (d.format == kFormatInt4 || d.format == kFormatBinary) && d.dim == 128 && d.num_tokens > 0 &&
         d.num_tokens < 0x7FFFFF00LL;
}

namespace tc {
// int4 rows [N, 64] -> int8 rows [N, 128] in the scan's K order (per 16-byte input chunk: low
// nibbles of word 0, high nibbles of word 0, ..., of word 3), identical to the expander warps.
__global__ void expand_codes8_kernel(const uint4* __restrict__ in, int64_t n_chunks, uint4* __restrict__ out) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_chunks;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint4 v = __ldg(in + i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t lo = w[j] & 0x0F0F0F0Fu, hi = (w[j] >> 4) & 0x0F0F0F0Fu;
      o[2 * j] = lo + (lo & 0x08080808u) * 30u;
      o[2 * j + 1] = hi + (hi & 0x08080808u) * 30u;
    }
    out[2 * i] = make_uint4(o[0], o[1], o[2], o[3]);
    out[2 * i + 1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}
// int4 codes -> f16 values in the same K order as the int8 copy (16 input bytes -> 32 values, 64 bytes).
__global__ void expand_codes16_kernel(const uint4* __restrict__ in, int64_t n_chunks, uint4* __restrict__ out) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_chunks;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint4 v = __ldg(in + i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t o[4];
#pragma unroll
      for (int half = 0; half < 2; ++half) {  // low nibbles of bytes 4j..4j+3, then their high nibbles
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          int n0 = static_cast<int>((w[j] >> (16 * q + 4 * half)) & 0xF);
          int n1 = static_cast<int>((w[j] >> (16 * q + 8 + 4 * half)) & 0xF);
          n0 -= (n0 & 8) << 1;  // two's complement nibble
          n1 -= (n1 & 8) << 1;
          o[2 * half + q] = static_cast<uint32_t>(__half_as_ushort(__int2half_rn(n0))) |
                            (static_cast<uint32_t>(__half_as_ushort(__int2half_rn(n1))) << 16);
        }
      }
      out[4 * i + j] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}
}  // namespace tc

void launch_expand_codes16(const uint8_t* codes, int64_t num_tokens, uint16_t* out, cudaStream_t stream) {
  const int64_t chunks = num_tokens * 4;
  if (chunks == 0) return;
  const int blocks = static_cast<int>(std::min<int64_t>((chunks + 255) / 256, 148LL * 16));
  tc::expand_codes16_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<const uint4*>(codes), chunks,
                                                        reinterpret_cast<uint4*>(out));
  count_launch();
  check(cudaGetLastError(), "launch f16 expansion kernel");
}

namespace tc {
// Sign codes [N, 16] (dim 8g + j is bit j of byte g; set = +1) -> int8 rows [N, 128] of +-1 in the scan's
// K order: per 8 dims, the even dims' bytes then the odd dims' (the order of the int4 copy and of the
// query words), so the tensor-core scan reads binary and int4 corpora alike.
__global__ void expand_binary8_kernel(const uint8_t* __restrict__ in, int64_t n_groups, uint2* __restrict__ out) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_groups;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t b = __ldg(in + i);
    uint32_t even = 0, odd = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      even |= (((b >> (2 * k)) & 1u) ? 0x01u : 0xFFu) << (8 * k);
      odd |= (((b >> (2 * k + 1)) & 1u) ? 0x01u : 0xFFu) << (8 * k);
    }
    out[i] = make_uint2(even, odd);
  }
}

// fp32 query rows -> three int8 digit planes for the tensor-core scan (dim 128).  Row r is scaled by
// 2^S, S = 22 - E where max|x| = f * 2^E, f in [0.5, 1), so its largest element lies in [2^21, 2^22],
// and rounded to integers q (|q| <= 2^22).  The signed base-256 digits q = d0 + 256 d1 + 65536 d2
// (d0, d1 in [-128, 127], |d2| <= 65) are packed like the int8 query words (nibble order: per 8 dims
// the even dims' bytes, then the odd dims'), plane k at words + k * rows * 32.  The scan's dot of plane
// k with a token is an exact int32; the three combine to the exact dot of q, and qscale = 2^-S (a power
// of two, exact) brings it back to the query's scale.  A row of zeros has S = 0; a row holding a
// non-finite value gets qscale NaN, so its scores are NaN.  Weighted MaxSim folds the row's weight in:
// qscale = w * 2^-S is exact (a power-of-two scaling of w, unless it leaves the normal range), so the
// epilogue's fl(best' * qscale), best' = best * 2^S, is fl(best * w).  weights: [qtok], or [rows] when
// weights_batched, or nullptr.
__global__ void split_query_digits_kernel(const float* __restrict__ q, int64_t rows, int32_t* __restrict__ words,
                                          float* __restrict__ qscale, const float* __restrict__ weights, int qtok,
                                          int weights_batched) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float4 v = __ldg(reinterpret_cast<const float4*>(q + row * 128) + lane);  // dims 4 lane .. 4 lane + 3
  float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
  const bool finite = __all_sync(0xFFFFFFFFu, isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w));
#pragma unroll
  for (int delta = 16; delta > 0; delta >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, delta));
  int S = 0;
  if (m > 0.0F && finite) {
    int E = 0;
    (void)frexpf(m, &E);
    S = min(22 - E, 149);  // rows below 2^-127 keep fewer bits rather than a zero qscale
  }
  const float x[4] = {v.x, v.y, v.z, v.w};
  uint32_t dig[3] = {0, 0, 0};  // 4 bytes of each plane, dims 4 lane + i
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qi = finite ? __float2int_rn(ldexpf(x[i], S)) : 0;
    const int d0 = static_cast<int8_t>(qi & 0xFF);
    const int r1 = (qi - d0) >> 8;
    const int d1 = static_cast<int8_t>(r1 & 0xFF);
    const int d2 = (r1 - d1) >> 8;
    dig[0] |= static_cast<uint32_t>(d0 & 0xFF) << (8 * i);
    dig[1] |= static_cast<uint32_t>(d1 & 0xFF) << (8 * i);
    dig[2] |= static_cast<uint32_t>(d2 & 0xFF) << (8 * i);
  }
  // nibble order: group g = lane / 2 (dims 8g .. 8g + 7); word 2g holds the even dims, 2g + 1 the odd.
  // Lane 2g holds dims 8g..8g+3 and lane 2g + 1 dims 8g+4..8g+7: exchange and interleave.
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const uint32_t mine = dig[k];
    const uint32_t other = __shfl_xor_sync(0xFFFFFFFFu, mine, 1);
    const uint32_t first = (lane & 1) ? other : mine;   // dims 8g + 0..3
    const uint32_t second = (lane & 1) ? mine : other;  // dims 8g + 4..7
    // even dims: bytes 0, 2 of first, then 0, 2 of second; odd dims: bytes 1, 3 of each
    const uint32_t even = __byte_perm(first, second, 0x6420);
    const uint32_t odd = __byte_perm(first, second, 0x7531);
    words[(static_cast<int64_t>(k) * rows + row) * 32 + lane] = static_cast<int32_t>((lane & 1) ? odd : even);
  }
  if (lane == 0) {
    const float w = weights ? weights[weights_batched ? row : row % qtok] : 1.0F;
    qscale[row] = finite ? ldexpf(w, -S) : __int_as_float(0x7FC00000);
  }
}
}  // namespace tc

void launch_split_query_digits(const float* q, int64_t rows, int32_t* words, float* qscale, const float* weights,
                               int qtok, int weights_batched, cudaStream_t stream) {
  if (rows <= 0) return;
  const int64_t threads = rows * 32;
  tc::split_query_digits_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(
      q, rows, words, qscale, weights, qtok, weights_batched);
  count_launch();
  check(cudaGetLastError(), "launch query digit-split kernel");
}

void launch_expand_binary8(const uint8_t* codes, int64_t num_tokens, uint8_t* out, cudaStream_t stream) {
  const int64_t groups = num_tokens * 16;
  if (groups == 0) return;
  const int blocks = static_cast<int>(std::min<int64_t>((groups + 255) / 256, 148LL * 16));
  tc::expand_binary8_kernel<<<blocks, 256, 0, stream>>>(codes, groups, reinterpret_cast<uint2*>(out));
  count_launch();
  check(cudaGetLastError(), "launch sign-code expansion kernel");
}

void launch_expand_codes8(const uint8_t* codes, int64_t num_tokens, uint8_t* out, cudaStream_t stream) {
  const int64_t chunks = num_tokens * 4;
  if (chunks == 0) return;
  const int blocks = static_cast<int>(std::min<int64_t>((chunks + 255) / 256, 148LL * 16));
  tc::expand_codes8_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<const uint4*>(codes), chunks,
                                                       reinterpret_cast<uint4*>(out));
  count_launch();
  check(cudaGetLastError(), "launch int8 expansion kernel");
}

namespace {
// 2D tensor map over the int8 copy: {128 bytes, N rows}, box {128, 128}, 128-byte swizzle, zero fill.
CUtensorMap encode_operand_map(const void* base, int64_t num_tokens, bool f16) {
  using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static EncodeFn encode = nullptr;
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q{};
      check(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q),
            "look up cuTensorMapEncodeTiled");
      if (!fn || q != cudaDriverEntryPointSuccess) throw CudaFailure("cuTensorMapEncodeTiled is not available");
      encode = reinterpret_cast<EncodeFn>(fn);
    }
  }
  // int8 copy: {128 bytes, N rows}, box {128, 128}; f16 copy: {128 values, N rows} (256-byte rows), box
  // {64, 128} = one 128-byte K half.  128-byte swizzle (the UMMA layout), zero fill.
  CUtensorMap m{};
  const cuuint64_t dims[2] = {128, static_cast<cuuint64_t>(num_tokens)};
  const cuuint64_t strides[1] = {f16 ? 256u : 128u};
  const cuuint32_t box[2] = {f16 ? 64u : 128u, static_cast<cuuint32_t>(tc::kTileN)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(&m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                            const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw CudaFailure("cuTensorMapEncodeTiled failed (" + std::to_string(static_cast<int>(r)) + ")");
  return m;
}

// The map depends only on (base, rows, f16): the last few are kept, so a search encodes none.
CUtensorMap make_operand_map(const void* base, int64_t num_tokens, bool f16) {
  struct Entry {
    const void* base;
    int64_t rows;
    bool f16;
    CUtensorMap map;
  };
  static std::mutex mu;
  static std::vector<Entry> maps;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (const Entry& e : maps)
      if (e.base == base && e.rows == num_tokens && e.f16 == f16) return e.map;
  }
  const CUtensorMap m = encode_operand_map(base, num_tokens, f16);
  std::lock_guard<std::mutex> lock(mu);
  if (maps.size() >= 16) maps.erase(maps.begin());
  maps.push_back(Entry{base, num_tokens, f16, m});
  return m;
}
}  // namespace

bool tc_scan_supported(const DocsView& d, const QueryView& q, const ReduceView& r, const TargetsView& tg,
                       bool residual) {
  // fp32 queries run as digit planes: at most 32 query tokens (one tile), and the digit split reads the
  // query as float4, so a caller's device pointer must be 16-byte aligned
  const bool mode_ok = q.mode == kQueryI8
                           ? q.qtok <= 128
                           : (q.mode == kQueryF32 && q.qtok <= 32 && (reinterpret_cast<uintptr_t>(q.f32) & 15) == 0);
  // binary corpora: a scalar document scale (the epilogue's one factor), read from the resident +-1 copy
  const bool format_ok = d.format == kFormatInt4 || (d.format == kFormatBinary && d.doc_scale == nullptr);
  // weighted MaxSim of fp32 queries: the weights fold into the digit planes' row scales
  // TopK2 / TopK4 of fp32 queries: per-row lists in the epilogue (not with the residual stream)
  const bool reducer_ok = r.reducer == kMaxSim || (r.reducer == kWeighted && q.mode == kQueryF32) ||
                          ((r.reducer == kTopK2 || r.reducer == kTopK4 || r.reducer == kSmooth) &&
                           q.mode == kQueryF32 && !residual);
  // the fused residual stream: an int4 or sign-code prefix and an int4 residual, per-token scales on both,
  // fp32 queries (a sign-code prefix has scale 1, so its term is fl(v1 * s1) as in the SIMT kernel)
  const bool residual_ok = !residual || ((d.format == kFormatInt4 || d.format == kFormatBinary) &&
                                         q.mode == kQueryF32 && d.token_scale != nullptr && d.codes2 != nullptr &&
                                         d.token_scale2 != nullptr);
  // candidate lists run over units built from the lists (launch_tc_scan_candidates)
  (void)tg;
  return residual_ok && format_ok && d.dim == 128 && mode_ok && reducer_ok && q.qtok >= 1 && q.batch >= 1 &&
         d.num_docs <= 0x7FFFFFFF && d.host_offsets != nullptr;
}

size_t tc_scan_workspace_bytes(const DocsView& d, const QueryView& q, const TargetsView&) {
  const TcPlan pl = plan_for(d, q, sm_count());
  const int64_t max_ranges = pl.n_ranges + d.num_docs / tc::kMaxRangeDocs + 2;
  return 256 + sizeof(tc::Unit) * static_cast<size_t>(max_ranges) * pl.n_pairs;
}

struct UnitCacheKey {
  const void* ws;
  uint64_t corpus_id;
  int64_t n_ranges;
  int n_pairs;
  bool split;  // the last pair's units at the end of the table (see launch_tc_scan)
  bool operator==(const UnitCacheKey& o) const {
    return ws == o.ws && corpus_id == o.corpus_id && n_ranges == o.n_ranges && n_pairs == o.n_pairs &&
           split == o.split;
  }
};

void launch_merge_shard_topk(const void*, int, int, int, const int64_t*, float*, int64_t*, cudaStream_t);
void launch_empty_block(void*, int, int, const int64_t*, int, cudaStream_t);

// Room for the fused top-k lists in the shared-memory layout the launch below picks for this scan.
int tc_topk_room(const DocsView& d, const QueryView& q, const ReduceView& red) {
  const bool digits = q.mode == kQueryF32;
  const bool f16 = !digits && d.format == kFormatInt4 && d.codes16 != nullptr && d.token_scale != nullptr;
  const bool pre = f16 || d.codes8 != nullptr;
  const bool res = d.codes2 != nullptr;
  // the fused variants: int8-query MaxSim on int8 operands
  if (res || digits || f16 || red.reducer != kMaxSim) return 0;
  if (d.token_scale && d.token_scale_small)
    return pre ? tc::Layout<true, false, false, true>::topk_bytes : tc::Layout<false, false, false, true>::topk_bytes;
  return pre ? tc::Layout<true>::topk_bytes : tc::Layout<false>::topk_bytes;
}

// Candidate workspace of a fused top-k: a block per CTA and list group (at most two) and the empty
// documents' block.
size_t tc_topk_cand_bytes(const QueryView& q, int k) {
  return static_cast<size_t>(2 * sm_count() + 1) * 16ull * q.batch * k;
}

namespace {
// Query rows copied over the TMEM lane quarters for a pass of one tile of int8 query rows: four copies of
// at most 32 rows, two of at most 64 (option tc_row_replicas), else 1.
int row_copies(const TcPlan& pl, const QueryView& q) {
  const int q_rows = q.batch * q.qtok;
  if (pl.n_qtiles != 1 || q.mode == kQueryF32 || !g_tc_row_replicas.load()) return 1;
  return q_rows <= 32 ? 4 : (q_rows <= 64 ? 2 : 1);
}

// Fused top-k when the pass has no row copies, the lists fit the chosen layout (twin mode keeps one set per
// epilogue group) and the caller's candidate workspace holds a block per CTA and group plus one for the
// empty documents.
bool fuse_fits(const DocsView& d, const QueryView& q, const ReduceView& red, const TcPlan& pl, int sms,
               const TopkFuse* fuse) {
  const int lists = pl.n_qtiles == 1 ? 2 : 1;
  return fuse != nullptr && fuse->k >= 1 && row_copies(pl, q) == 1 &&
         static_cast<int64_t>(lists) * q.batch * fuse->k * 8 <= tc_topk_room(d, q, red) &&
         static_cast<size_t>(lists * sms + 1) * 16ull * q.batch * fuse->k <= fuse->cand_bytes;
}

// The scan over a unit table on the device: the kernel variant for the corpus, queries and reducer, then
// (fused top-k) the merge of the CTAs' candidate blocks.
void dispatch_tc(const DocsView& d, const QueryView& q, const ReduceView& red, const TcPlan& pl, int sms,
                 const tc::Unit* d_units, int num_units, float* out, int* err, bool fused, TopkFuse* fuse,
                 cudaStream_t stream, bool clear_err = true) {
  const int reps = row_copies(pl, q);
  const int lists = pl.n_qtiles == 1 ? 2 : 1;
  if (clear_err) check(cudaMemsetAsync(err, 0, sizeof(int), stream), "clear tc error flag");
  tc::Params prm{};
  prm.codes = d.codes;
  prm.token_scale = d.token_scale;
  prm.offsets = d.offsets;
  prm.qwords = q.i8_words;
  prm.qscale = q.row_scale;
  prm.units = d_units;
  prm.num_units = num_units;
  // One query tile: twin mode lets the two epilogue groups take two units' tiles in turn
  const bool twin = pl.n_qtiles == 1;
  prm.num_items = twin ? (num_units + 1) / 2 : num_units;
  prm.batch = q.batch;
  prm.qtok = q.qtok;
  prm.qpt = pl.qpt;
  // the fused residual stream applies its scalar scales per token, not to the document score
  const bool res = d.codes2 != nullptr;
  prm.scale = res ? 1.0F : d.scale;
  prm.token_scale2 = d.token_scale2;
  prm.res_scale1 = d.scale;
  prm.res_scale2 = d.scale2;
  prm.num_docs = d.num_docs;
  prm.out = fused ? nullptr : out;
  prm.error = err;
  prm.topk_k = fused ? fuse->k : 0;
  prm.cand = fused ? static_cast<unsigned char*>(fuse->cand) : nullptr;
  const int grid = std::min<int>(sms, prm.num_items);
  const bool digits = q.mode == kQueryF32;
  const bool f16 = !digits && d.format == kFormatInt4 && d.codes16 != nullptr && d.token_scale != nullptr;
  const bool pre = f16 || d.codes8 != nullptr;
  // the expanding path decodes int4 rows: binary corpora need their +-1 copy, the residual stream both
  // int8 copies
  if (d.format == kFormatBinary && !d.codes8) throw CudaFailure("binary tensor-core scan without the int8 copy");
  if (res && !(digits && d.token_scale && d.token_scale2 && d.codes8 && d.codes2_8))
    throw CudaFailure("residual tensor-core scan without its int8 copies");
  const int topk = red.reducer == kTopK2 ? 2 : (red.reducer == kTopK4 ? 4 : 0);
  if (topk && !(digits && d.codes8 && !res)) throw CudaFailure("TopK tensor-core scan without the int8 copy");
  const bool smooth = red.reducer == kSmooth;
  if (smooth && !(digits && d.codes8 && !res)) throw CudaFailure("SmoothSim tensor-core scan without the int8 copy");
  if (smooth) {
    // SmoothSim scales every value before the reduction (the reference's kScaleFirst): the document
    // scale goes into the epilogue's exponent, not onto the document score
    prm.smooth_scale = prm.scale;
    prm.scale = 1.0F;
    prm.temperature = red.temperature;
  }
  const CUtensorMap tmap = f16   ? make_operand_map(d.codes16, d.num_tokens, true)
                           : pre ? make_operand_map(d.codes8, d.num_tokens, false)
                                 : CUtensorMap{};
  const CUtensorMap tmap2 = res ? make_operand_map(d.codes2_8, d.num_tokens, false) : CUtensorMap{};
  auto go = [&](auto plain, auto twin_kernel, int smem_bytes) {
    auto kernel = twin ? twin_kernel : plain;
    raise_smem_limit(reinterpret_cast<const void*>(kernel), smem_bytes);
    kernel<<<grid, tc::kThreads, smem_bytes, stream>>>(prm, tmap, tmap2);
  };
  // int8 queries: replicated rows (reps), or the fused top-k, or the plain scan
  auto go8 = [&](auto plain, auto twin_kernel, auto twin2, auto twin4, auto fplain, auto ftwin, int smem_plain,
                 int smem_fused) {
    if (fused) go(fplain, ftwin, smem_fused);
    else if (reps == 4) go(twin4, twin4, smem_plain);
    else if (reps == 2) go(twin2, twin2, smem_plain);
    else go(plain, twin_kernel, smem_plain);
  };
  using LayoutF16 = tc::Layout<true, true>;
#define MSB_TC_GO(TS, PRE, F16, DIG, LAYOUT) \
  go(tc::tc_scan_kernel<TS, PRE, F16, DIG, false>, tc::tc_scan_kernel<TS, PRE, F16, DIG, true>, LAYOUT::bytes_plain)
  // int8 queries (one tile: optionally replicated rows); BIAS: biased accumulators
#define MSB_TC_GO8(TS, PRE, BIAS)                                                                        \
  go8(tc::tc_scan_kernel<TS, PRE, false, false, false, false, 0, BIAS>,                                 \
      tc::tc_scan_kernel<TS, PRE, false, false, true, false, 0, BIAS>,                                  \
      tc::tc_scan_kernel<TS, PRE, false, false, true, false, 0, BIAS, false, 2>,                        \
      tc::tc_scan_kernel<TS, PRE, false, false, true, false, 0, BIAS, false, 4>,                        \
      tc::tc_scan_kernel<TS, PRE, false, false, false, false, 0, BIAS, false, 1, true>,                 \
      tc::tc_scan_kernel<TS, PRE, false, false, true, false, 0, BIAS, false, 1, true>,                  \
      tc::Layout<PRE, false, false, BIAS>::bytes_plain, tc::Layout<PRE, false, false, BIAS>::bytes)
  using LayoutRes = tc::Layout<true, false, true>;
  if (res) {
    go(tc::tc_scan_kernel<true, true, false, true, false, true>, tc::tc_scan_kernel<true, true, false, true, true, true>,
       LayoutRes::bytes_plain);
  } else if (digits) {
    // digit planes: biased accumulators unless a token scale is too large for the exact s * 2^23
    const bool bias = d.token_scale == nullptr || d.token_scale_small;
#define MSB_TC_DIG(TS, PRE, K, SM, B)                                                     \
  go(tc::tc_scan_kernel<TS, PRE, false, true, false, false, K, B, SM>,                   \
     tc::tc_scan_kernel<TS, PRE, false, true, true, false, K, B, SM>, tc::Layout<PRE, false, false, B>::bytes_plain)
#define MSB_TC_DIG2(TS, PRE, K, SM) \
  if (bias) MSB_TC_DIG(TS, PRE, K, SM, true); else MSB_TC_DIG(TS, PRE, K, SM, false)
    if (smooth) {
      if (d.token_scale) MSB_TC_DIG2(true, true, 0, true);
      else MSB_TC_DIG2(false, true, 0, true);
    } else if (topk == 2) {
      if (d.token_scale) MSB_TC_DIG2(true, true, 2, false);
      else MSB_TC_DIG2(false, true, 2, false);
    } else if (topk == 4) {
      if (d.token_scale) MSB_TC_DIG2(true, true, 4, false);
      else MSB_TC_DIG2(false, true, 4, false);
    } else if (d.token_scale) {
      if (pre) MSB_TC_DIG2(true, true, 0, false);
      else MSB_TC_DIG2(true, false, 0, false);
    } else {
      if (pre) MSB_TC_DIG2(false, true, 0, false);
      else MSB_TC_DIG2(false, false, 0, false);
    }
#undef MSB_TC_DIG2
#undef MSB_TC_DIG
  } else if (d.token_scale) {
    // biased accumulators unless a token scale is too large for the exact s * 2^23
    if (f16) MSB_TC_GO(true, true, true, false, LayoutF16);
    else if (pre && d.token_scale_small) MSB_TC_GO8(true, true, true);
    else if (pre) MSB_TC_GO8(true, true, false);
    else if (d.token_scale_small) MSB_TC_GO8(true, false, true);
    else MSB_TC_GO8(true, false, false);
  } else {
    if (pre) MSB_TC_GO8(false, true, false);
    else MSB_TC_GO8(false, false, false);
  }
#undef MSB_TC_GO8
#undef MSB_TC_GO
  count_launch();
  check(cudaGetLastError(), "launch tensor-core scan kernel");
  if (fused) {
    // the CTAs' candidate blocks, then the empty documents' block, merged in the single-pass order
    int blocks = lists * grid;
    const int n_empty = std::min(fuse->n_empty, fuse->k);
    if (n_empty > 0) {
      launch_empty_block(static_cast<unsigned char*>(fuse->cand) + static_cast<size_t>(blocks) * 16ull * q.batch * fuse->k,
                         q.batch, fuse->k, fuse->empty_ids, n_empty, stream);
      ++blocks;
    }
    launch_merge_shard_topk(fuse->cand, blocks, q.batch, fuse->k, nullptr, fuse->out_s, fuse->out_i, stream);
    fuse->done = true;
  }
}
}  // namespace

void launch_tc_scan(const DocsView& d, const QueryView& q, const ReduceView& red, const TargetsView&, float* out, void* ws,
                    size_t ws_bytes, cudaStream_t stream, TopkFuse* fuse) {
  // The unit table depends only on the corpus and the query tiling; it is
  // built once per (workspace, corpus, tiling) and kept in the workspace.
  static std::mutex cache_mu;
  static std::vector<std::pair<UnitCacheKey, int>> cache;  // key -> number of units
  const int sms = sm_count();
  const TcPlan pl = plan_for(d, q, sms);
  UnitCacheKey key{ws, d.corpus_id, pl.n_ranges, pl.n_pairs, false};
  int* err = static_cast<int*>(ws);
  tc::Unit* d_units = reinterpret_cast<tc::Unit*>(static_cast<unsigned char*>(ws) + 256);
  const bool fused = fuse_fits(d, q, red, pl, sms, fuse);
  if (fuse) fuse->done = false;
  // An odd number (> 1) of int8 query tiles: the last tile would fill only half of its pair's units (four
  // of the eight epilogue warps working), so it runs as a launch of its own in twin mode, its two epilogue
  // groups taking two document ranges in turn, after the full pairs' launch.  The table then lists the
  // full pairs' units (range-major) and after them the last tile's, one per range.
  const bool split = !fused && q.mode == kQueryI8 && pl.n_qtiles > 1 && (pl.n_qtiles & 1) != 0;
  key.split = split;
  int num_units = -1;
  {
    std::lock_guard<std::mutex> lock(cache_mu);
    for (auto& e : cache)
      if (e.first == key) num_units = e.second;
  }
  // Empty documents never appear in a tile; their score is 0.
  if (!fused)
    check(cudaMemsetAsync(out, 0, sizeof(float) * static_cast<size_t>(q.batch) * d.num_docs, stream), "zero scores");
  if (num_units < 0) {
    // Document ranges cut at the token quantiles r * N / n_ranges, each split
    // further to at most kMaxRangeDocs documents; range-major units.
    std::vector<tc::Unit> units, tail;
    const int64_t* off = d.host_offsets;
    const int64_t D = d.num_docs, N = d.num_tokens;
    int64_t lo = 0;
    for (int64_t r = 1; r <= pl.n_ranges && lo < D; ++r) {
      int64_t hi = D;
      if (r < pl.n_ranges) {
        const int64_t target = static_cast<int64_t>((static_cast<__int128>(N) * r) / pl.n_ranges);
        hi = static_cast<int64_t>(std::lower_bound(off + lo, off + D + 1, target) - off);
        if (hi > D) hi = D;
      }
      while (lo < hi) {
        const int64_t h2 = std::min<int64_t>(hi, lo + tc::kMaxRangeDocs);  // unit offsets live in shared memory
        if (off[h2] > off[lo]) {
          for (int t = 0; t < pl.n_pairs - (split ? 1 : 0); ++t) units.push_back(tc::Unit{lo, h2, off[lo], off[h2], t, 0});
          // split: the last tile's unit, as query tile 0 of its own launch
          if (split) tail.push_back(tc::Unit{lo, h2, off[lo], off[h2], 0, 0});
        }
        lo = h2;
      }
    }
    units.insert(units.end(), tail.begin(), tail.end());
    const size_t need = 256 + sizeof(tc::Unit) * units.size();
    if (need > ws_bytes) throw CudaFailure("tensor-core scan workspace too small");
    if (!units.empty()) {
      check(cudaMemcpyAsync(d_units, units.data(), sizeof(tc::Unit) * units.size(), cudaMemcpyHostToDevice, stream),
            "upload tc work units");
      check(cudaStreamSynchronize(stream), "synchronize tc unit upload");
    }
    num_units = static_cast<int>(units.size());
    std::lock_guard<std::mutex> lock(cache_mu);
    for (auto it = cache.begin(); it != cache.end();)
      it = it->first.ws == ws ? cache.erase(it) : it + 1;
    cache.emplace_back(key, num_units);
  }
  if (num_units == 0) {
    if (!fused) return;
    // every document is empty: the empty documents' block alone
    launch_empty_block(fuse->cand, q.batch, fuse->k, fuse->empty_ids, std::min(fuse->n_empty, fuse->k), stream);
    launch_merge_shard_topk(fuse->cand, 1, q.batch, fuse->k, nullptr, fuse->out_s, fuse->out_i, stream);
    fuse->done = true;
    return;
  }
  if (split) {
    const int n_tail = num_units / pl.n_pairs;  // every range lists n_pairs units
    dispatch_tc(d, q, red, pl, sms, d_units, num_units - n_tail, out, err, false, nullptr, stream);
    // the last tile's queries as a one-tile batch of their own: query rows, scales and score rows offset
    const int b0 = (pl.n_qtiles - 1) * pl.qpt;
    const int64_t r0 = static_cast<int64_t>(b0) * q.qtok;
    QueryView q1 = q;
    q1.batch = q.batch - b0;
    if (q.f32) q1.f32 = q.f32 + r0 * d.dim;
    if (q.i8) q1.i8 = q.i8 + r0 * d.dim;
    q1.i8_words = q.i8_words + r0 * (d.dim / 4);
    q1.row_scale = q.row_scale + r0;
    if (q.row_sum) q1.row_sum = q.row_sum + r0;
    TcPlan pl1 = pl;
    pl1.n_qtiles = 1;
    pl1.n_pairs = 1;
    dispatch_tc(d, q1, red, pl1, sms, d_units + (num_units - n_tail), n_tail, out + static_cast<int64_t>(b0) * d.num_docs,
                err, false, nullptr, stream, false);
    return;
  }
  dispatch_tc(d, q, red, pl, sms, d_units, num_units, out, err, fused, fuse, stream);
}

namespace tc {
// Work units of a candidate-list scan, one per (candidate document, query-tile pair): a shared list gives
// every pair every candidate, per-row lists give each candidate to the pair holding its row.  An empty
// candidate document gets an empty unit and its score 0 in the rows concerned (an empty document never
// appears in a tile); an id outside [0, D) gets an empty unit.  A document listed twice is scanned twice
// and writes the same values twice.
__global__ void candidate_units_kernel(const int64_t* __restrict__ ids, int64_t count, int per_row, int batch,
                                       int qpt, int n_pairs, const int64_t* __restrict__ offsets, int64_t num_docs,
                                       Unit* __restrict__ units, float* __restrict__ scores) {
  const int64_t n = per_row ? static_cast<int64_t>(batch) * count : count * n_pairs;
  for (int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < n;
       u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t d;
    int pair, row = 0;
    if (per_row) {
      row = static_cast<int>(u / count);
      d = ids[u];
      pair = (row / qpt) / kG;
    } else {
      d = ids[u / n_pairs];
      pair = static_cast<int>(u % n_pairs);
    }
    Unit un{0, 0, 0, 0, pair, 0};
    if (d >= 0 && d < num_docs) {
      const int64_t lo = offsets[d], hi = offsets[d + 1];
      un.d_lo = d;
      un.d_hi = hi > lo ? d + 1 : d;
      un.tok_lo = lo;
      un.tok_hi = hi > lo ? hi : lo;
      if (hi <= lo) {
        if (per_row) {
          scores[static_cast<int64_t>(row) * num_docs + d] = 0.0F;
        } else {
          const int r0 = pair * kG * qpt, r1 = min(batch, r0 + kG * qpt);
          for (int r = r0; r < r1; ++r) scores[static_cast<int64_t>(r) * num_docs + d] = 0.0F;
        }
      }
    }
    units[u] = un;
  }
}
}  // namespace tc

// Units a candidate-list scan needs (tc::Unit each).
size_t tc_candidate_units_bytes(const DocsView& d, const QueryView& q, const TargetsView& tg) {
  const TcPlan pl = plan_for(d, q, sm_count());
  const int64_t n = tg.per_row ? static_cast<int64_t>(q.batch) * tg.count : tg.count * pl.n_pairs;
  return sizeof(tc::Unit) * static_cast<size_t>(n > 0 ? n : 1);
}

// A candidate-list scan on the tensor cores: the documents the lists name, each its own work unit, scored
// into `scores` [B, D] at their document positions (only those positions are written; the caller gathers
// them).  `ws` holds the kernel's error word, `units` the unit table.
void launch_tc_scan_candidates(const DocsView& d, const QueryView& q, const ReduceView& red, const TargetsView& tg,
                               float* scores, void* ws, void* units, size_t units_bytes, cudaStream_t stream) {
  const int sms = sm_count();
  const TcPlan pl = plan_for(d, q, sms);
  const int64_t n = tg.per_row ? static_cast<int64_t>(q.batch) * tg.count : tg.count * pl.n_pairs;
  if (n <= 0) return;
  if (n > 0x3FFFFFFF || sizeof(tc::Unit) * static_cast<size_t>(n) > units_bytes)
    throw CudaFailure("candidate unit workspace too small");
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148LL * 8));
  tc::candidate_units_kernel<<<blocks, 256, 0, stream>>>(tg.ids, tg.count, tg.per_row ? 1 : 0, q.batch, pl.qpt,
                                                         pl.n_pairs, d.offsets, d.num_docs,
                                                         static_cast<tc::Unit*>(units), scores);
  count_launch();
  check(cudaGetLastError(), "launch candidate unit kernel");
  dispatch_tc(d, q, red, pl, sms, static_cast<const tc::Unit*>(units), static_cast<int>(n), scores,
              static_cast<int*>(ws), false, nullptr, stream);
}

}  // namespace msb
