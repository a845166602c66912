/*
 * oracle.c -- TEST INFRASTRUCTURE ONLY.  Plain-C restatement of the exact
 * integer / index reductions of the b200 op path, used to check the GPU
 * kernels bit for bit at sizes where numpy would be slow or memory-hungry.
 *
 *  oracle_sum_i32_i64_rows   int64 sum of each int32 row (torch.sum of an
 *                            int32 tensor promotes to int64: csrc/aten/
 *                            backends/cuda/sum.cu:32-66 through
 *                            make_reduction's int64 promotion).
 *  oracle_argmax_rows_bf16   index of the first maximum of each row of bf16
 *                            bit patterns, NaN counting as the maximum and the
 *                            first NaN winning (torch.argmax; unregistered in
 *                            the reference, so it runs in the CPU fallback of
 *                            csrc/aten/register.cc:439-442).
 *  oracle_amax_rows_f32      max of each float row, NaN propagating.
 *
 * Built by oracle/Makefile into oracle/_build/liboracle.so.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float bf16_to_float(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

void oracle_sum_i32_i64_rows(const int32_t* x, int64_t rows, int64_t cols, int64_t ld,
                             int64_t* out) {
  for (int64_t r = 0; r < rows; ++r) {
    const int32_t* p = x + r * ld;
    int64_t s = 0;
    for (int64_t c = 0; c < cols; ++c) s += (int64_t)p[c];
    out[r] = s;
  }
}

void oracle_argmax_rows_bf16(const uint16_t* x, int64_t rows, int64_t cols, int64_t ld,
                             int64_t* out) {
  for (int64_t r = 0; r < rows; ++r) {
    const uint16_t* p = x + r * ld;
    int64_t best = 0;
    float bv = bf16_to_float(p[0]);
    int bnan = isnan(bv);
    for (int64_t c = 1; c < cols && !bnan; ++c) {
      const float v = bf16_to_float(p[c]);
      if (isnan(v)) {
        best = c;
        bnan = 1;
      } else if (v > bv) {
        best = c;
        bv = v;
      }
    }
    out[r] = best;
  }
}

void oracle_amax_rows_f32(const float* x, int64_t rows, int64_t cols, int64_t ld,
                          float* out) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* p = x + r * ld;
    float m = -INFINITY;
    for (int64_t c = 0; c < cols; ++c) {
      if (isnan(p[c])) {
        m = p[c];
        break;
      }
      if (p[c] > m) m = p[c];
    }
    out[r] = m;
  }
}
