/*
 * Plain-C restatement of the reference's int8-query scans (CPU oracle).
 *
 * TEST INFRASTRUCTURE ONLY: called by tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py.  The product library
 * (maxsim_b200/csrc) does not link or call this file.
 *
 * Restated reference code (paths relative to the reference project root):
 *   quantiser      cpp/maxsim/cuda_extension.cu:1455-1492
 *   int4 x int8    cpp/maxsim/cuda_extension.cu:1494-1627 (exact int dot,
 *                  scale-before-max for per-token scales, fp32 epilogue)
 *   binary x int8  cpp/maxsim/cuda_extension.cu:1328-1449 (sum of +-q)
 * The epilogue reproduces the CUDA kernel's fp32 rounding sequence exactly:
 *   best_r = max_t fl(float(dot) * s_t); acc = fl(acc + fl(best_r * qs_r))
 *   in query-row order; score = fl(acc * scale).
 * Build flags must not enable fast-math or FP contraction (see Makefile).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* Per-row int8 quantisation with the kernel's formula.  dim-major rows. */
void oracle_quantize_int8(const float* query, int64_t rows, int dim, int8_t* codes, float* scales) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* x = query + r * dim;
    float max_abs = 0.0f;
    for (int i = 0; i < dim; ++i) {
      float a = fabsf(x[i]);
      max_abs = a > max_abs ? a : max_abs;
    }
    volatile float s = max_abs == 0.0f ? 1.0f : max_abs / 127.0f;
    volatile float inv = 1.0f / s;
    scales[r] = s;
    for (int i = 0; i < dim; ++i) {
      volatile float p = x[i] * inv;
      float q = rintf(p);
      if (q > 127.0f) q = 127.0f;
      if (q < -127.0f) q = -127.0f;
      codes[r * dim + i] = (int8_t)q;
    }
  }
}

static inline int nibble(uint8_t byte, int hi) {
  int v = hi ? (byte >> 4) : (byte & 0x0F);
  return v >= 8 ? v - 16 : v;
}

/* Exact int4 x int8 scores for a list of target documents.
 * qcodes [B*Q, dim] int8, qscales [B*Q], packed [N, dim/2], token_scale [N] or NULL,
 * offsets [D+1], targets [T] (NULL = all docs), out [B, T]. */
int oracle_int4_int8q_scores(const int8_t* qcodes, const float* qscales, int batch, int qtok, int dim,
                             const uint8_t* packed, const float* token_scale, float scale,
                             const int64_t* offsets, int64_t num_docs, const int64_t* targets,
                             int64_t num_targets, float* out, int threads) {
  const int64_t T = targets ? num_targets : num_docs;
  const int half = dim / 2;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(dynamic, 4) collapse(2)
#endif
  for (int b = 0; b < batch; ++b) {
    for (int64_t j = 0; j < T; ++j) {
      int64_t d = targets ? targets[j] : j;
      int64_t s = offsets[d], e = offsets[d + 1];
      float acc = 0.0f;
      if (s < e && qtok > 0) {
        int8_t unpacked[512];
        for (int r = 0; r < qtok; ++r) {
          const int8_t* qc = qcodes + ((int64_t)b * qtok + r) * dim;
          float best = -3.402823466e+38f;
          for (int64_t t = s; t < e; ++t) {
            const uint8_t* row = packed + t * half;
            for (int i = 0; i < half; ++i) {
              unpacked[2 * i] = (int8_t)nibble(row[i], 0);
              unpacked[2 * i + 1] = (int8_t)nibble(row[i], 1);
            }
            int32_t dot = 0;
            for (int i = 0; i < dim; ++i) dot += (int32_t)qc[i] * (int32_t)unpacked[i];
            volatile float v = (float)dot;
            if (token_scale) v = v * token_scale[t];
            best = v > best ? v : best;
          }
          volatile float c = best * qscales[(int64_t)b * qtok + r];
          acc = acc + c;
        }
      }
      volatile float res = acc * scale;
      out[(int64_t)b * T + j] = res;
    }
  }
  return 0;
}

/* The same scores as oracle_int4_int8q_scores (exact integer dots, then the identical fp32 epilogue
 * sequence per (query, document)), organised for large corpora: threads take documents, each
 * document's tokens are unpacked to int8 once and shared by every query row, and the integer dot is
 * a plain loop the compiler vectorises (integer sums do not depend on their order). */
int oracle_int4_int8q_scores_docs(const int8_t* qcodes, const float* qscales, int batch, int qtok, int dim,
                                  const uint8_t* packed, const float* token_scale, float scale,
                                  const int64_t* offsets, int64_t num_docs, const int64_t* targets,
                                  int64_t num_targets, float* out, int threads) {
  const int64_t T = targets ? num_targets : num_docs;
  const int half = dim / 2;
  int failed = 0;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel
#endif
  {
    int8_t* buf = NULL;
    int64_t cap = 0;
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
    for (int64_t j = 0; j < T; ++j) {
      int64_t d = targets ? targets[j] : j;
      int64_t s = offsets[d], e = offsets[d + 1], n = e - s;
      if (n > cap) {
        free(buf);
        buf = (int8_t*)malloc((size_t)n * (size_t)dim);
        cap = buf ? n : 0;
        if (!buf) {
          failed = 1;
          continue;
        }
      }
      for (int64_t t = 0; t < n; ++t) {
        const uint8_t* row = packed + (s + t) * half;
        for (int i = 0; i < half; ++i) {
          buf[t * dim + 2 * i] = (int8_t)nibble(row[i], 0);
          buf[t * dim + 2 * i + 1] = (int8_t)nibble(row[i], 1);
        }
      }
      for (int b = 0; b < batch; ++b) {
        float acc = 0.0f;
        if (n > 0 && qtok > 0) {
          for (int r = 0; r < qtok; ++r) {
            const int8_t* qc = qcodes + ((int64_t)b * qtok + r) * dim;
            float best = -3.402823466e+38f;
            for (int64_t t = 0; t < n; ++t) {
              const int8_t* tok = buf + t * dim;
              int32_t dot = 0;
              for (int i = 0; i < dim; ++i) dot += (int32_t)qc[i] * (int32_t)tok[i];
              volatile float v = (float)dot;
              if (token_scale) v = v * token_scale[s + t];
              best = v > best ? v : best;
            }
            volatile float c = best * qscales[(int64_t)b * qtok + r];
            acc = acc + c;
          }
        }
        volatile float res = acc * scale;
        out[(int64_t)b * T + j] = res;
      }
    }
    free(buf);
  }
  return failed ? -1 : 0;
}

/* Exact binary x int8 scores: dot = sum_i (bit_i ? q_i : -q_i). */
int oracle_binary_int8q_scores(const int8_t* qcodes, const float* qscales, int batch, int qtok, int dim,
                               const uint8_t* packed, const float* token_scale, const float* doc_scale,
                               float scale, const int64_t* offsets, int64_t num_docs,
                               const int64_t* targets, int64_t num_targets, float* out, int threads) {
  const int64_t T = targets ? num_targets : num_docs;
  const int bytes = dim / 8;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(dynamic, 4) collapse(2)
#endif
  for (int b = 0; b < batch; ++b) {
    for (int64_t j = 0; j < T; ++j) {
      int64_t d = targets ? targets[j] : j;
      int64_t s = offsets[d], e = offsets[d + 1];
      float acc = 0.0f;
      if (s < e && qtok > 0) {
        for (int r = 0; r < qtok; ++r) {
          const int8_t* qc = qcodes + ((int64_t)b * qtok + r) * dim;
          float best = -3.402823466e+38f;
          for (int64_t t = s; t < e; ++t) {
            const uint8_t* row = packed + t * bytes;
            int32_t dot = 0;
            for (int i = 0; i < dim; ++i) {
              int bit = (row[i >> 3] >> (i & 7)) & 1;
              dot += bit ? (int32_t)qc[i] : -(int32_t)qc[i];
            }
            volatile float v = (float)dot;
            if (token_scale) v = v * token_scale[t];
            best = v > best ? v : best;
          }
          volatile float c = best * qscales[(int64_t)b * qtok + r];
          acc = acc + c;
        }
      }
      float ds = doc_scale ? doc_scale[d] : scale;
      volatile float res = acc * ds;
      out[(int64_t)b * T + j] = res;
    }
  }
  return 0;
}
