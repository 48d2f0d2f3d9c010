/*
 * C restatement of the reference's emitted host golden (test infrastructure,
 * never part of the product path).
 *
 * Follows the CPU golden that tensixflow prints into every generated host
 * program: goldenRmsnorm / goldenMatmul (lib/tensixflow/Codegen/EmitHost.cpp:
 * 727-762) and goldenMlp (:1176-1227). Unlike the numpy golden
 * (python/tensixflow/golden.py), that golden rounds the normalised row and the
 * GELU output to bf16 and accumulates each dot product sequentially in fp32.
 * bf16 rounding is round-to-nearest-even with NaN made quiet, as in
 * python/tensixflow/rounding.py:54-67. The reference's bfloat16 type comes from
 * tt-metalium (not in the reference tree), so this file carries its own.
 *
 * All matrices are row-major float arrays holding bf16-representable values.
 * Rows are independent; OpenMP splits them across host threads.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static float bf16_round(float v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) {
    u = (u & 0x80000000u) | 0x7FC00000u;
  } else {
    const uint32_t dropped = u & 0xFFFFu;
    const uint32_t odd = (u >> 16) & 1u;
    u &= 0xFFFF0000u;
    if (dropped > 0x8000u || (dropped == 0x8000u && odd)) u += 0x10000u;
  }
  float r;
  memcpy(&r, &u, 4);
  return r;
}

void tfo_bf16_round(const float* in, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = bf16_round(in[i]);
}

/* goldenRmsnorm: normalized[r,c] = bf16(x[r,c] * inv_rms(r) * gamma[c]). */
void tfo_rmsnorm_bf16(const float* x, const float* gamma, int64_t m, int64_t k, float eps, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < m; ++r) {
    float ss = 0.0f;
    for (int64_t c = 0; c < k; ++c) ss += x[r * k + c] * x[r * k + c];
    const float inv = 1.0f / sqrtf(ss / (float)k + eps);
    for (int64_t c = 0; c < k; ++c) out[r * k + c] = bf16_round(x[r * k + c] * inv * gamma[c]);
  }
}

/* goldenMatmul: out[i,j] = bf16(sum_k a[i,k] * b[k,j]) (sequential fp32 sum). */
void tfo_matmul_bf16(const float* a, const float* b, int64_t m, int64_t k, int64_t n, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < m; ++i) {
    for (int64_t j = 0; j < n; ++j) {
      float s = 0.0f;
      for (int64_t kk = 0; kk < k; ++kk) s += a[i * k + kk] * b[kk * n + j];
      out[i * n + j] = bf16_round(s);
    }
  }
}

/* goldenMlp with a selectable GELU (0 = exact erf as in the reference, 1 = tanh
 * form, which the reference does not have):
 *   h = bf16(gelu(normalized @ w1 + bias)); y = bf16(h @ w2 + residual). */
void tfo_mlp_bf16(const float* x, const float* gamma, const float* w1, const float* bias, const float* w2,
                  const float* residual, int64_t m, int64_t k, int64_t h, int64_t n, float eps, int gelu_mode,
                  float* out) {
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t r = 0; r < m; ++r) {
    float ss = 0.0f;
    for (int64_t c = 0; c < k; ++c) ss += x[r * k + c] * x[r * k + c];
    const float inv = 1.0f / sqrtf(ss / (float)k + eps);
    float* nrm = (float*)malloc(sizeof(float) * (size_t)(k > 0 ? k : 1));
    float* hid = (float*)malloc(sizeof(float) * (size_t)(h > 0 ? h : 1));
    for (int64_t c = 0; c < k; ++c) nrm[c] = bf16_round(x[r * k + c] * inv * gamma[c]);
    for (int64_t j = 0; j < h; ++j) hid[j] = 0.0f;
    for (int64_t kk = 0; kk < k; ++kk) {
      const float a = nrm[kk];
      const float* wr = w1 + kk * h;
      for (int64_t j = 0; j < h; ++j) hid[j] += a * wr[j];
    }
    for (int64_t j = 0; j < h; ++j) {
      const float s = hid[j] + (bias ? bias[j] : 0.0f);
      float g;
      if (gelu_mode == 0) {
        g = 0.5f * s * (1.0f + erff(s * 0.70710678f));
      } else {
        const float u = 0.7978845608028654f * (s + 0.044715f * s * s * s);
        g = 0.5f * s * (1.0f + tanhf(u));
      }
      hid[j] = bf16_round(g);
    }
    for (int64_t j = 0; j < n; ++j) out[r * n + j] = 0.0f;
    for (int64_t hh = 0; hh < h; ++hh) {
      const float a = hid[hh];
      const float* wr = w2 + hh * n;
      for (int64_t j = 0; j < n; ++j) out[r * n + j] += a * wr[j];
    }
    for (int64_t j = 0; j < n; ++j) out[r * n + j] = bf16_round(out[r * n + j] + residual[r * n + j]);
    free(nrm);
    free(hid);
  }
}
