// Sign-code (binary) MaxSim by AND + population count, dim 128.
//
// The reference scores sign codes either by a per-bit select-and-add over fp32 query values
// (cpp/maxsim/cuda_extension.cu:297-352) or, for int8 queries, by the integer identity
// dot = 2 * (sum of q over set bits) - sum(q) (maxsim_binary_int8q_dim128_kernel, :1368-1449).  Here a
// query row of integers q_i is held as bit-planes P_b (bit b of every q_i, two's complement, b < NB), so
// that for a token's 128 sign bits D
//     sum_{i : D_i = 1} q_i = sum_b w_b popc(P_b & D),   w_b = 2^b for b < NB - 1, w_{NB-1} = -2^(NB-1),
// and the signed dot is 2 * that - sum(q): exact integer arithmetic, 4 * NB AND + popcount pairs per
// (token, query row) and no per-dimension work.
//   * int8 queries (NB = 8): the quantiser's codes; the dot is the reference's integer dot, bit for bit.
//   * fp32 queries (NB = 24): each row as the 23-bit fixed-point integers of the tensor-core digit planes
//     (rint(x * 2^S), S = 22 - E for max|x| = f * 2^E), qscale = 2^-S (times the row's weight for weighted
//     MaxSim); the dot is that integer dot, so the scores equal the tensor-core engine's bit for bit and
//     stay within 1e-4 of the reference's fp32 sums.
// Epilogue as the reference's: fl(float(dot) * s_t) with per-token scales, the maximum per row,
// doc += fl(best * qscale) in row order, then the document scale (scalar or per-document vector).
//
// Layout: one warp per (document, group of whole queries): lane r holds query row r of the group (its NB
// x 4 plane words in registers), lanes take 32 tokens at a time with one 16-byte load each, and each
// token's words reach every lane by shuffles.  The code stream is 16 bytes per token, read once per
// query group.
#include <algorithm>

#include "common.cuh"

namespace msb {

namespace {
constexpr int kPopcWarps = 4;

// Query rows -> bit-planes [rows][NB][4] (word w holds dims 32w .. 32w + 31, bit j = dim 32w + j), the
// row sums and (fp32 rows) the power-of-two row scales.  One 128-thread block per row.
__global__ void __launch_bounds__(128) popc_planes_kernel(const float* __restrict__ qf, const int8_t* __restrict__ qi,
                                                          int64_t rows, int nb, const float* __restrict__ weights,
                                                          int qtok, int weights_batched, uint32_t* __restrict__ planes,
                                                          int32_t* __restrict__ qsum, float* __restrict__ qscale) {
  __shared__ int32_t qv[128];
  __shared__ float red_max[4];
  __shared__ int red_fin[4];
  __shared__ int32_t red_sum[4];
  const int64_t row = blockIdx.x;
  const int i = threadIdx.x, lane = i & 31, warp = i >> 5;
  int32_t q;
  if (qi) {
    q = qi[row * 128 + i];
  } else {
    const float x = qf[row * 128 + i];
    float m = fabsf(x);
    int fin = isfinite(x) ? 1 : 0;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
      m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, d));
      fin &= __shfl_xor_sync(0xFFFFFFFFu, fin, d);
    }
    if (lane == 0) {
      red_max[warp] = m;
      red_fin[warp] = fin;
    }
    __syncthreads();
    m = fmaxf(fmaxf(red_max[0], red_max[1]), fmaxf(red_max[2], red_max[3]));
    const bool finite = red_fin[0] && red_fin[1] && red_fin[2] && red_fin[3];
    int S = 0;
    if (m > 0.0F && finite) {
      int E = 0;
      (void)frexpf(m, &E);
      S = min(22 - E, 149);
    }
    q = finite ? __float2int_rn(ldexpf(x, S)) : 0;
    if (i == 0) {
      const float w = weights ? weights[weights_batched ? row : row % qtok] : 1.0F;
      qscale[row] = finite ? ldexpf(w, -S) : __int_as_float(0x7FC00000);
    }
  }
  qv[i] = q;
  int32_t s = q;
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, d);
  if (lane == 0) red_sum[warp] = s;
  __syncthreads();
  if (i == 0) qsum[row] = red_sum[0] + red_sum[1] + red_sum[2] + red_sum[3];
  if (i < nb * 4) {
    const int b = i >> 2, w = i & 3;
    uint32_t mask = 0;
    for (int j = 0; j < 32; ++j) mask |= ((static_cast<uint32_t>(qv[32 * w + j]) >> b) & 1u) << j;
    planes[(row * nb + b) * 4 + w] = mask;
  }
}

template <int NB>
__device__ __forceinline__ int32_t plane_dot(const uint32_t (&P)[NB][4], uint4 D) {
  // Horner over the planes, sign plane first: sum over set bits of q
  int32_t acc = -(__popc(P[NB - 1][0] & D.x) + __popc(P[NB - 1][1] & D.y) + __popc(P[NB - 1][2] & D.z) +
                  __popc(P[NB - 1][3] & D.w));
#pragma unroll
  for (int b = NB - 2; b >= 0; --b)
    acc = 2 * acc + (__popc(P[b][0] & D.x) + __popc(P[b][1] & D.y) + __popc(P[b][2] & D.z) + __popc(P[b][3] & D.w));
  return acc;
}

template <int NB>
__global__ void __launch_bounds__(kPopcWarps * 32) popc_scan_kernel(DocsView docs, const uint32_t* __restrict__ planes,
                                                                    const int32_t* __restrict__ qsum,
                                                                    const float* __restrict__ qscale, int batch,
                                                                    int qtok, const int64_t* __restrict__ targets,
                                                                    int64_t num_targets, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int qpw = 32 / qtok;                                   // whole queries per warp
  const int groups = (batch + qpw - 1) / qpw;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * kPopcWarps + (threadIdx.x >> 5);
  const int64_t T = targets ? num_targets : docs.num_docs;
  if (item >= T * groups) return;
  const int64_t j = item / groups;
  const int grp = static_cast<int>(item % groups);
  const int64_t d = targets ? targets[j] : j;
  const int qloc = lane / qtok;                                // query of the group this lane's row belongs to
  const int b = grp * qpw + qloc;
  const bool live = qloc < qpw && b < batch;
  const int64_t row = live ? static_cast<int64_t>(b) * qtok + lane % qtok : 0;
  uint32_t P[NB][4];
#pragma unroll
  for (int p = 0; p < NB; ++p) {
    const uint4 v = live ? __ldg(reinterpret_cast<const uint4*>(planes) + row * NB + p) : make_uint4(0, 0, 0, 0);
    P[p][0] = v.x;
    P[p][1] = v.y;
    P[p][2] = v.z;
    P[p][3] = v.w;
  }
  const int32_t qs_int = live ? qsum[row] : 0;
  const int64_t start = docs.offsets[d], end = docs.offsets[d + 1];
  const uint4* codes = reinterpret_cast<const uint4*>(docs.codes);
  float best = kLowest;
  for (int64_t t0 = start; t0 < end; t0 += 32) {
    const int n = end - t0 < 32 ? static_cast<int>(end - t0) : 32;
    const uint4 mine = lane < n ? __ldg(codes + t0 + lane) : make_uint4(0, 0, 0, 0);
    const float my_s = (docs.token_scale && lane < n) ? __ldg(docs.token_scale + t0 + lane) : 1.0F;
    for (int k = 0; k < n; ++k) {
      uint4 D;
      D.x = __shfl_sync(0xFFFFFFFFu, mine.x, k);
      D.y = __shfl_sync(0xFFFFFFFFu, mine.y, k);
      D.z = __shfl_sync(0xFFFFFFFFu, mine.z, k);
      D.w = __shfl_sync(0xFFFFFFFFu, mine.w, k);
      const float s = __shfl_sync(0xFFFFFFFFu, my_s, k);
      float v = __int2float_rn(2 * plane_dot<NB>(P, D) - qs_int);
      if (docs.token_scale) v = __fmul_rn(v, s);
      best = fmaxf(best, v);
    }
  }
  // row value, then each query's rows summed in order by the query's first lane
  const float rv = (live && end > start) ? __fmul_rn(best, qscale[row]) : 0.0F;
  float acc = 0.0F;
  const int base = qloc * qtok;
  for (int r = 0; r < qtok; ++r) {
    const float x = __shfl_sync(0xFFFFFFFFu, rv, min(base + r, 31));
    acc = __fadd_rn(acc, x);
  }
  if (live && lane % qtok == 0) {
    const float ds = docs.doc_scale ? docs.doc_scale[d] : docs.scale;
    out[static_cast<int64_t>(b) * T + j] = __fmul_rn(acc, ds);
  }
}
}  // namespace

bool popc_scan_supported(const DocsView& d, const QueryView& q, const ReduceView& r, const TargetsView& tg,
                         bool residual) {
  const bool mode_ok = q.mode == kQueryI8 || (q.mode == kQueryF32 && q.f32 != nullptr);
  const bool red_ok = r.reducer == kMaxSim || (r.reducer == kWeighted && q.mode == kQueryF32);
  return d.format == kFormatBinary && d.dim == 128 && !residual && mode_ok && red_ok && q.qtok >= 1 && q.qtok <= 32 &&
         q.batch >= 1 && (tg.ids == nullptr || !tg.per_row);
}

size_t popc_scan_workspace_bytes(const QueryView& q) {
  const size_t rows = static_cast<size_t>(q.batch) * q.qtok;
  return rows * (24 * 16 + 4 + 4) + 256;
}

// q.i8 (int8 mode: natural-order codes and q.row_scale) or q.f32 (fp32 mode); ws holds the planes.
void launch_popc_scan(const DocsView& d, const QueryView& q, const ReduceView& r, const TargetsView& tg, float* out,
                      void* ws, size_t ws_bytes, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(q.batch) * q.qtok;
  const int nb = q.mode == kQueryI8 ? 8 : 24;
  if (ws_bytes < popc_scan_workspace_bytes(q)) throw CudaFailure("popcount scan workspace too small");
  uint32_t* planes = static_cast<uint32_t*>(ws);
  int32_t* qsum = reinterpret_cast<int32_t*>(planes + rows * 24 * 4);
  float* qscale = reinterpret_cast<float*>(qsum + rows);
  const bool weighted = r.reducer == kWeighted;
  popc_planes_kernel<<<static_cast<unsigned>(rows), 128, 0, stream>>>(
      q.mode == kQueryI8 ? nullptr : q.f32, q.mode == kQueryI8 ? q.i8 : nullptr, rows, nb,
      weighted ? r.weights : nullptr, q.qtok, weighted ? r.weights_batched : 0, planes, qsum, qscale);
  count_launch();
  check(cudaGetLastError(), "launch popcount query-plane kernel");
  const float* qs = q.mode == kQueryI8 ? q.row_scale : qscale;
  const int qpw = 32 / q.qtok;
  const int64_t groups = (q.batch + qpw - 1) / qpw;
  const int64_t T = tg.ids ? tg.count : d.num_docs;
  const int64_t items = T * groups;
  if (items == 0) return;
  const unsigned blocks = static_cast<unsigned>((items + kPopcWarps - 1) / kPopcWarps);
  if (nb == 8)
    popc_scan_kernel<8><<<blocks, kPopcWarps * 32, 0, stream>>>(d, planes, qsum, qs, q.batch, q.qtok, tg.ids, tg.count,
                                                               out);
  else
    popc_scan_kernel<24><<<blocks, kPopcWarps * 32, 0, stream>>>(d, planes, qsum, qs, q.batch, q.qtok, tg.ids,
                                                                tg.count, out);
  count_launch();
  check(cudaGetLastError(), "launch popcount scan kernel");
}

}  // namespace msb
