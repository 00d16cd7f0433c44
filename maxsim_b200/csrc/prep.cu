// Device-side corpus encoders (large corpora are packed where they are made).
//
// Bit-exact with the reference NumPy encoders:
//   per-token int4  src/maxsim/experimental.py:240-246   s_t = max|x_t| / 7 (fp32, 0 -> 1),
//                                                         code = clip(rint(x / s_t), -7, 7)
//   tensor int4     src/maxsim/experimental.py:247-255   s = float64(max|X|) / 7, codes
//                                                         use x / float32(s)
//   nibble layout   src/maxsim/experimental.py:604-609   even dim in the low nibble
//   sign bits       src/maxsim/_api.py:49-54             bit i of byte i/8, x >= 0 -> 1
// fp32 division is IEEE (__fdiv_rn) and rintf rounds half to even, as NumPy.
#include <algorithm>

#include "common.cuh"

namespace msb {

// One warp per token; dim % 8 == 0 and dim <= 1024.
__global__ void pack_int4_token_kernel(const float* __restrict__ x, int64_t n, int dim, uint8_t* __restrict__ codes,
                                       float* __restrict__ token_scale) {
  const int64_t t = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= n) return;
  const float* row = x + t * dim;
  float m = 0.0F;
  for (int i = lane; i < dim; i += 32) m = fmaxf(m, fabsf(row[i]));
#pragma unroll
  for (int delta = 16; delta > 0; delta >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, delta));
  float s = __fdiv_rn(m, 7.0F);
  if (s == 0.0F) s = 1.0F;
  if (lane == 0) token_scale[t] = s;
  uint8_t* out = codes + t * (dim / 2);
  for (int p = lane; p < dim / 2; p += 32) {
    float a = rintf(__fdiv_rn(row[2 * p], s));
    float b = rintf(__fdiv_rn(row[2 * p + 1], s));
    int ia = static_cast<int>(fminf(fmaxf(a, -7.0F), 7.0F));
    int ib = static_cast<int>(fminf(fmaxf(b, -7.0F), 7.0F));
    out[p] = static_cast<uint8_t>((ia & 0xF) | ((ib & 0xF) << 4));
  }
}

__global__ void absmax_kernel(const float* __restrict__ x, int64_t count, unsigned int* __restrict__ out_bits) {
  float m = 0.0F;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    m = fmaxf(m, fabsf(x[i]));
#pragma unroll
  for (int delta = 16; delta > 0; delta >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, delta));
  if ((threadIdx.x & 31) == 0) atomicMax(out_bits, __float_as_uint(m));  // non-negative floats order as uints
}

__global__ void pack_int4_scaled_kernel(const float* __restrict__ x, int64_t pairs, float s,
                                        uint8_t* __restrict__ codes) {
  for (int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; p < pairs;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float a = rintf(__fdiv_rn(x[2 * p], s));
    float b = rintf(__fdiv_rn(x[2 * p + 1], s));
    int ia = static_cast<int>(fminf(fmaxf(a, -7.0F), 7.0F));
    int ib = static_cast<int>(fminf(fmaxf(b, -7.0F), 7.0F));
    codes[p] = static_cast<uint8_t>((ia & 0xF) | ((ib & 0xF) << 4));
  }
}

// One warp per token: sign bits and the float64 mean |x| (token scale source).
__global__ void pack_signs_kernel(const float* __restrict__ x, int64_t n, int dim, uint8_t* __restrict__ bits,
                                  float* __restrict__ mean_abs) {
  const int64_t t = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= n) return;
  const float* row = x + t * dim;
  double acc = 0.0;
  for (int i = lane; i < dim; i += 32) acc += fabs(static_cast<double>(row[i]));
#pragma unroll
  for (int delta = 16; delta > 0; delta >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, delta);
  if (lane == 0 && mean_abs) mean_abs[t] = static_cast<float>(acc / dim);
  for (int byte = lane; byte < dim / 8; byte += 32) {
    uint32_t v = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) v |= (row[8 * byte + j] >= 0.0F ? 1u : 0u) << j;
    bits[t * (dim / 8) + byte] = static_cast<uint8_t>(v);
  }
}

void launch_pack_int4(const float* x, int64_t n, int dim, bool per_token, uint8_t* codes, float* token_scale,
                      float* tensor_scale_out, void* scratch_u32, cudaStream_t stream) {
  if (n <= 0) return;
  if (per_token) {
    const int64_t threads = n * 32;
    pack_int4_token_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(x, n, dim, codes,
                                                                                          token_scale);
    count_launch();
    check(cudaGetLastError(), "launch per-token int4 pack kernel");
    return;
  }
  unsigned int* bits = static_cast<unsigned int*>(scratch_u32);
  check(cudaMemsetAsync(bits, 0, sizeof(unsigned int), stream), "clear absmax");
  absmax_kernel<<<1184, 256, 0, stream>>>(x, n * dim, bits);
  count_launch();
  unsigned int host_bits = 0;
  check(cudaMemcpyAsync(&host_bits, bits, sizeof(host_bits), cudaMemcpyDeviceToHost, stream), "read absmax");
  check(cudaStreamSynchronize(stream), "synchronize absmax");
  float max_abs;
  memcpy(&max_abs, &host_bits, sizeof(max_abs));
  const double scale = max_abs == 0.0F ? 1.0 : static_cast<double>(max_abs) / 7.0;
  const float s32 = static_cast<float>(scale);
  pack_int4_scaled_kernel<<<1184, 256, 0, stream>>>(x, n * dim / 2, s32, codes);
  count_launch();
  check(cudaGetLastError(), "launch tensor int4 pack kernel");
  if (tensor_scale_out) *tensor_scale_out = s32;
}

void launch_pack_signs(const float* x, int64_t n, int dim, uint8_t* bits, float* mean_abs, cudaStream_t stream) {
  if (n <= 0) return;
  const int64_t threads = n * 32;
  pack_signs_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(x, n, dim, bits, mean_abs);
  count_launch();
  check(cudaGetLastError(), "launch sign pack kernel");
}

// Sets *bad to 1 when any value is not finite or not > 0 (the reference's token-scale rule,
// cuda_extension.cu:2753-2758 / experimental.py:699-700, checked on the device after an upload).
__global__ void check_positive_finite_kernel(const float* __restrict__ x, int64_t n, unsigned int* __restrict__ bad) {
  bool ok = true;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float v = x[i];
    ok = ok && v > 0.0F && isfinite(v);
  }
  if (__any_sync(0xFFFFFFFFu, !ok) && (threadIdx.x & 31) == 0) atomicOr(bad, 1u);
}

// Sets *bad to 1 when any nibble of the int4 codes is 8 (the value -8): symmetric int4 codes lie in
// [-7, 7] (reference experimental.py _validate_int4_packed, checked on the unpacked values).
// A byte holds a nibble n == 8 iff (n ^ 8) == 0; zero bytes are found four at a time.
__global__ void check_int4_codes_kernel(const uint32_t* __restrict__ words, int64_t nwords,
                                        unsigned int* __restrict__ bad) {
  bool ok = true;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nwords;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t w = words[i];
    const uint32_t lo = (w & 0x0F0F0F0Fu) ^ 0x08080808u, hi = ((w >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
    const uint32_t zl = (lo - 0x01010101u) & ~lo & 0x80808080u, zh = (hi - 0x01010101u) & ~hi & 0x80808080u;
    ok = ok && (zl | zh) == 0u;
  }
  if (__any_sync(0xFFFFFFFFu, !ok) && (threadIdx.x & 31) == 0) atomicOr(bad, 1u);
}

void launch_check_int4_codes(const uint8_t* codes, int64_t bytes, unsigned int* bad, cudaStream_t stream) {
  if (bytes <= 0) return;
  const int64_t nwords = bytes / 4;  // int4 rows are dim / 2 bytes, dim % 8 == 0
  const int64_t blocks = std::min<int64_t>((nwords + 255) / 256, 148 * 16);
  check_int4_codes_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
      reinterpret_cast<const uint32_t*>(codes), nwords, bad);
  count_launch();
  check(cudaGetLastError(), "launch int4 code check kernel");
}

// Sets *big to 1 when any finite value has magnitude >= 2^104 (too large for the tensor-core scan's
// exact s * 2^23 staging of token scales).
__global__ void check_scale_range_kernel(const float* __restrict__ x, int64_t n, unsigned int* __restrict__ big) {
  bool small = true;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float a = fabsf(x[i]);
    small = small && !(isfinite(a) && a >= 0x1p104F);
  }
  if (__any_sync(0xFFFFFFFFu, !small) && (threadIdx.x & 31) == 0) atomicOr(big, 1u);
}

void launch_check_scale_range(const float* x, int64_t n, unsigned int* big, cudaStream_t stream) {
  if (n <= 0) return;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 16);
  check_scale_range_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(x, n, big);
  count_launch();
  check(cudaGetLastError(), "launch scale range check kernel");
}

void launch_check_positive_finite(const float* x, int64_t n, unsigned int* bad, cudaStream_t stream) {
  if (n <= 0) return;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 16);
  check_positive_finite_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(x, n, bad);
  count_launch();
  check(cudaGetLastError(), "launch token scale check kernel");
}

}  // namespace msb
