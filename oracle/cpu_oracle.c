/*
 * cpu_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference engine's scalar CPU oracle for the
 * matrix-multiply hot path (Parag63/bare-metal-llm-engine, src/cpu_ref/).  It is
 * the CHECKER for the CUDA library in bare-metal-llm-engine_b200/: only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it.  Nothing in
 * the product path calls it, and the product path has no CPU fallback.
 *
 * Arithmetic contract (identical to the reference):
 *   - dot products accumulate in double, in increasing-k order, one product
 *     (double)a * (double)b per step, and are rounded to float once at the end;
 *   - RMSNorm sums squares in double, forms scale = (float)(1/sqrt(mean + eps))
 *     with eps INSIDE the square root, then temp = (src * scale) * w in float;
 *   - FP16 values widen exactly to float; results narrow with IEEE
 *     round-to-nearest-even (the reference's CUDA build uses __float2half, which
 *     rounds to nearest even).
 *
 * The [N,K] ("W") variants index W[n*K + k] directly.  They are the same
 * arithmetic as feeding the reference function the exact transpose W^T, which is
 * how the reference would be used for the B200 configurations.
 *
 * The *_mt variants split the output rows into contiguous blocks over POSIX
 * threads and run the same per-element arithmetic, so their output is
 * bit-identical to the single-thread call (the all-cores CPU baseline).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- FP16 / BF16 */

/* IEEE 754 binary32 -> binary16, round to nearest, ties to even. */
uint16_t orc_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) { /* inf / nan */
    return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x0200u : 0u));
  }
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 -> inf */
  const int32_t e = (int32_t)(ax >> 23);
  if (e >= 113) { /* normal half: biased float exponent 113..142 */
    const uint32_t mant = ax & 0x7fffffu;
    uint32_t h = ((uint32_t)(e - 112) << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
  }
  /* subnormal half: value = m * 2^(E-150), unit 2^-24 -> q = m * 2^(E-126) */
  const uint32_t m = (e == 0) ? (ax & 0x7fffffu) : ((ax & 0x7fffffu) | 0x800000u);
  const int32_t shift = 126 - (e == 0 ? 1 : e);
  if (shift >= 25) return (uint16_t)sign; /* below half the smallest subnormal */
  uint32_t q = m >> shift;
  const uint32_t rem = m & ((1u << shift) - 1u);
  const uint32_t halfway = 1u << (shift - 1);
  if (rem > halfway || (rem == halfway && (q & 1u))) q++;
  return (uint16_t)(sign | q);
}

float orc_f16_to_f32(uint16_t h) {
  const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1fu;
  uint32_t mant = h & 0x3ffu;
  uint32_t out;
  if (e == 0) {
    if (mant == 0) {
      out = sign;
    } else { /* subnormal: normalise */
      int32_t ee = 113;
      while ((mant & 0x400u) == 0) {
        mant <<= 1;
        ee--;
      }
      out = sign | ((uint32_t)ee << 23) | ((mant & 0x3ffu) << 13);
    }
  } else if (e == 31) {
    out = sign | 0x7f800000u | (mant << 13);
  } else {
    out = sign | ((e + 112u) << 23) | (mant << 13);
  }
  float f;
  memcpy(&f, &out, 4);
  return f;
}

/* IEEE binary32 -> bfloat16, round to nearest even (NaN stays quiet NaN). */
uint16_t orc_f32_to_bf16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
  const uint32_t lsb = (x >> 16) & 1u;
  return (uint16_t)((x + 0x7fffu + lsb) >> 16);
}

float orc_bf16_to_f32(uint16_t h) {
  const uint32_t x = (uint32_t)h << 16;
  float f;
  memcpy(&f, &x, 4);
  return f;
}

void orc_f32_to_f16_array(const float* in, uint16_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = orc_f32_to_f16(in[i]);
}
void orc_f16_to_f32_array(const uint16_t* in, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = orc_f16_to_f32(in[i]);
}

/* ------------------------------------------------------------------ FP32 path */

/* C[M,N] = A[M,K] * B[K,N], row-major.  Follows src/cpu_ref/matmul_cpu.cpp:16-29. */
static void matmul_rows(const float* A, const float* B, float* C, int64_t r0, int64_t r1,
                        int64_t N, int64_t K) {
  for (int64_t i = r0; i < r1; ++i) {
    for (int64_t j = 0; j < N; ++j) {
      double acc = 0.0;
      for (int64_t k = 0; k < K; ++k) acc += (double)A[i * K + k] * (double)B[k * N + j];
      C[i * N + j] = (float)acc;
    }
  }
}

void orc_matmul(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K) {
  matmul_rows(A, B, C, 0, M, N, K);
}

/* out[N] = x[K] * A[K,N].  Follows src/cpu_ref/gemv_cpu.cpp:15-23. */
void orc_gemv(const float* A, const float* x, float* out, int64_t N, int64_t K) {
  for (int64_t j = 0; j < N; ++j) {
    double acc = 0.0;
    for (int64_t k = 0; k < K; ++k) acc += (double)x[k] * (double)A[k * N + j];
    out[j] = (float)acc;
  }
}

/* Follows src/cpu_ref/rmsnorm_cpu.cpp:19-43 (eps inside the sqrt). */
static float row_scale(const float* src, int64_t K, float eps) {
  double sumsq = 0.0;
  for (int64_t k = 0; k < K; ++k) sumsq += (double)src[k] * (double)src[k];
  const double mean_sq = sumsq / (double)K;
  return (float)(1.0 / sqrt(mean_sq + (double)eps));
}

void orc_rmsnorm(const float* in, const float* weight, float* out, int64_t rows, int64_t cols,
                 float eps) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* src = in + r * cols;
    float* dst = out + r * cols;
    const float scale = row_scale(src, cols, eps);
    for (int64_t c = 0; c < cols; ++c) {
      const float w = weight ? weight[c] : 1.0f;
      dst[c] = src[c] * scale * w;
    }
  }
}

/* sum_out = x + residual; norm_out = rmsnorm(sum_out) * weight.  Follows
 * src/cpu_ref/residual_rmsnorm_cpu.cpp:19-51: the float sum, squares of it
 * accumulated in double in increasing-c order, scale = float(1 / sqrt(mean +
 * eps)) in double, norm = (s * scale) * w in float.  residual, weight and
 * sum_out may be NULL, as in the reference. */
void orc_residual_rmsnorm(const float* x, const float* residual, const float* weight,
                          float* norm_out, float* sum_out, int64_t rows, int64_t cols,
                          float eps) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* sx = x + r * cols;
    const float* sr = residual ? residual + r * cols : NULL;
    float* dn = norm_out + r * cols;
    float* ds = sum_out ? sum_out + r * cols : NULL;
    double sumsq = 0.0;
    for (int64_t c = 0; c < cols; ++c) {
      const float v = sx[c] + (sr ? sr[c] : 0.0f);
      if (ds) ds[c] = v;
      sumsq += (double)v * (double)v;
    }
    const float scale = (float)(1.0 / sqrt(sumsq / (double)cols + (double)eps));
    for (int64_t c = 0; c < cols; ++c) {
      const float v = ds ? ds[c] : sx[c] + (sr ? sr[c] : 0.0f);
      const float w = weight ? weight[c] : 1.0f;
      dn[c] = v * scale * w;
    }
  }
}

/* out[M,N] = rmsnorm(in)[M,K] * W[K,N].  Follows src/cpu_ref/rmsnorm_linear_cpu.cpp:18-51. */
static void rmsnorm_linear_rows(const float* in, const float* rms_weight, const float* W,
                                float* out, int64_t r0, int64_t r1, int64_t N, int64_t K,
                                float eps) {
  float* temp = (float*)malloc((size_t)(K > 0 ? K : 1) * sizeof(float));
  for (int64_t r = r0; r < r1; ++r) {
    const float* src = in + r * K;
    float* dst = out + r * N;
    const float scale = row_scale(src, K, eps);
    for (int64_t k = 0; k < K; ++k) {
      const float w = rms_weight ? rms_weight[k] : 1.0f;
      temp[k] = src[k] * scale * w;
    }
    for (int64_t n = 0; n < N; ++n) {
      double acc = 0.0;
      for (int64_t k = 0; k < K; ++k) acc += (double)temp[k] * (double)W[k * N + n];
      dst[n] = (float)acc;
    }
  }
  free(temp);
}

void orc_rmsnorm_linear(const float* in, const float* rms_weight, const float* W, float* out,
                        int64_t M, int64_t N, int64_t K, float eps) {
  rmsnorm_linear_rows(in, rms_weight, W, out, 0, M, N, K, eps);
}

/* out[i] = a[i] + b[i].  Follows src/cpu_ref/vector_add_cpu.cpp:8-12. */
void orc_vector_add(const float* a, const float* b, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
}

/* ------------------------------------------------------------------ FP16 path */

/* out[N] = x[K] * A[K,N], FP16 in/out, double accumulate.
 * Follows src/cpu_ref/gemv_cpu.cpp:25-35. */
void orc_gemv_fp16(const uint16_t* A, const uint16_t* x, uint16_t* out, int64_t N, int64_t K) {
  for (int64_t j = 0; j < N; ++j) {
    double acc = 0.0;
    for (int64_t k = 0; k < K; ++k)
      acc += (double)orc_f16_to_f32(x[k]) * (double)orc_f16_to_f32(A[k * N + j]);
    out[j] = orc_f32_to_f16((float)acc);
  }
}

/* Shared inner kernel of the [N,K] forms: y[r, n] for rows r0..r1 of X[M,K] and
 * W[N,K] (element type selected by `bf16`), double accumulate over increasing k.
 * If `residual` is non-null the double sum is rounded to float, the (widened)
 * residual is added in float, and the result is rounded to the output type --
 * the order in which the reference composes matmul then vector_add
 * (tests/test_kernels.cu:2805-2810), with the fp16 rounding of the projection
 * removed because the B200 kernels fold the add into the epilogue. */
static inline float widen(uint16_t v, int bf16) {
  return bf16 ? orc_bf16_to_f32(v) : orc_f16_to_f32(v);
}
static inline uint16_t narrow(float v, int bf16) {
  return bf16 ? orc_f32_to_bf16(v) : orc_f32_to_f16(v);
}

static void linear_rows(const uint16_t* X, const uint16_t* W, const uint16_t* residual,
                        uint16_t* Y, int64_t r0, int64_t r1, int64_t N, int64_t K, int bf16,
                        float* Y32) {
  for (int64_t r = r0; r < r1; ++r) {
    for (int64_t n = 0; n < N; ++n) {
      double acc = 0.0;
      for (int64_t k = 0; k < K; ++k)
        acc += (double)widen(X[r * K + k], bf16) * (double)widen(W[n * K + k], bf16);
      float v = (float)acc;
      if (residual) v = v + widen(residual[r * N + n], bf16);
      if (Y32) Y32[r * N + n] = v;
      if (Y) Y[r * N + n] = narrow(v, bf16);
    }
  }
}

/* Y[M,N] = X[M,K] * W[N,K]^T (+ residual).  The reference's cpu::matmul
 * (matmul_cpu.cpp:16-29) fed W^T, with FP16/BF16 inputs widened exactly. */
void orc_linear_f16(const uint16_t* X, const uint16_t* W, const uint16_t* residual, uint16_t* Y,
                    int64_t M, int64_t N, int64_t K, int bf16, float* Y32) {
  linear_rows(X, W, residual, Y, 0, M, N, K, bf16, Y32);
}

/* C[M,N] = A[M,K] * B[K,N] with FP16/BF16 inputs; also returns the float
 * (pre-narrowing) value in C32 when non-null.  cpu::matmul on widened inputs. */
static void matmul16_rows(const uint16_t* A, const uint16_t* B, uint16_t* C, float* C32,
                          int64_t r0, int64_t r1, int64_t N, int64_t K, int bf16) {
  for (int64_t i = r0; i < r1; ++i) {
    for (int64_t j = 0; j < N; ++j) {
      double acc = 0.0;
      for (int64_t k = 0; k < K; ++k)
        acc += (double)widen(A[i * K + k], bf16) * (double)widen(B[k * N + j], bf16);
      const float v = (float)acc;
      if (C32) C32[i * N + j] = v;
      if (C) C[i * N + j] = narrow(v, bf16);
    }
  }
}

void orc_matmul_f16(const uint16_t* A, const uint16_t* B, uint16_t* C, float* C32, int64_t M,
                    int64_t N, int64_t K, int bf16) {
  matmul16_rows(A, B, C, C32, 0, M, N, K, bf16);
}

/* Y[M,N] = rmsnorm(x)[M,K] * W[N,K]^T (+ residual), FP16 in/out.
 * cpu::rmsnorm_linear (rmsnorm_linear_cpu.cpp:18-51) on widened FP16 inputs,
 * fed W^T; gamma may be null (unit gain). */
static void rmsnorm_linear_f16_rows(const uint16_t* x, const uint16_t* gamma, const uint16_t* W,
                                    const uint16_t* residual, uint16_t* Y, float* Y32,
                                    int64_t r0, int64_t r1, int64_t N, int64_t K, float eps) {
  float* src = (float*)malloc((size_t)(K > 0 ? K : 1) * sizeof(float));
  float* temp = (float*)malloc((size_t)(K > 0 ? K : 1) * sizeof(float));
  for (int64_t r = r0; r < r1; ++r) {
    for (int64_t k = 0; k < K; ++k) src[k] = orc_f16_to_f32(x[r * K + k]);
    const float scale = row_scale(src, K, eps);
    for (int64_t k = 0; k < K; ++k) {
      const float w = gamma ? orc_f16_to_f32(gamma[k]) : 1.0f;
      temp[k] = src[k] * scale * w;
    }
    for (int64_t n = 0; n < N; ++n) {
      double acc = 0.0;
      for (int64_t k = 0; k < K; ++k) acc += (double)temp[k] * (double)orc_f16_to_f32(W[n * K + k]);
      float v = (float)acc;
      if (residual) v = v + orc_f16_to_f32(residual[r * N + n]);
      if (Y32) Y32[r * N + n] = v;
      if (Y) Y[r * N + n] = orc_f32_to_f16(v);
    }
  }
  free(src);
  free(temp);
}

void orc_rmsnorm_linear_f16(const uint16_t* x, const uint16_t* gamma, const uint16_t* W,
                            const uint16_t* residual, uint16_t* Y, float* Y32, int64_t M,
                            int64_t N, int64_t K, float eps) {
  rmsnorm_linear_f16_rows(x, gamma, W, residual, Y, Y32, 0, M, N, K, eps);
}

/* SwiGLU glue: out = silu(gate) * up in double, rounded once.
 * Follows src/cpu_ref/swiglu_cpu.cpp:28-40. */
void orc_swiglu_f16(const uint16_t* gate, const uint16_t* up, uint16_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    const double g = (double)orc_f16_to_f32(gate[i]);
    const double u = (double)orc_f16_to_f32(up[i]);
    const double silu = g / (1.0 + exp(-g));
    out[i] = orc_f32_to_f16((float)(silu * u));
  }
}

/* Causal / non-causal MHA / GQA attention, the two-pass FP64 oracle of
 * src/cpu_ref/attention_cpu.cpp:87-155 (contract checks :27-66).
 * Layouts: q / out [s_q][n_heads][head_dim]; k / v [n_kv_heads][s_kv][head_dim]
 * with kv_head_stride elements between consecutive KV heads.  Query row i sees
 * keys j <= q_pos_offset + i when causal (all keys otherwise); its scores are
 * FP64 dot products of the widened halves times scale, the softmax is shifted
 * by the row max, exponentials and the P.V accumulation are FP64, and the
 * output is (acc / sum) rounded to float, then to half; lse = float(m +
 * log(sum)).  A row with no visible key is zero with lse = -inf; s_kv == 0
 * zeroes every row.  Returns 0, or 1 when an argument breaks the contract (the
 * reference throws there). */
int orc_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out,
                  int64_t s_q, int64_t s_kv, int64_t n_heads, int64_t n_kv_heads,
                  int64_t head_dim, int64_t kv_head_stride, float scale, int64_t q_pos_offset,
                  int is_causal, float* out_lse) {
  if (!q || !k || !v || !out) return 1;
  if (s_q < 0 || s_kv < 0 || q_pos_offset < 0 || n_heads <= 0 || n_kv_heads <= 0) return 1;
  if (n_heads % n_kv_heads != 0 || (head_dim != 64 && head_dim != 128) || !isfinite(scale))
    return 1;
  if (kv_head_stride < (s_kv > 0 ? s_kv * head_dim : 0)) return 1;
  if (s_q == 0) return 0;
  const uint16_t zero = orc_f32_to_f16(0.0f);
  if (s_kv == 0) {
    for (int64_t i = 0; i < s_q * n_heads * head_dim; ++i) out[i] = zero;
    if (out_lse)
      for (int64_t i = 0; i < s_q * n_heads; ++i) out_lse[i] = -INFINITY;
    return 0;
  }
  const int64_t group = n_heads / n_kv_heads;
  const double scale_d = (double)scale;
  double* scores = (double*)malloc((size_t)s_kv * sizeof(double));
  double* acc = (double*)malloc((size_t)head_dim * sizeof(double));
  if (!scores || !acc) {
    free(scores);
    free(acc);
    return 1;
  }
  for (int64_t i = 0; i < s_q; ++i) {
    int64_t max_j = s_kv - 1;
    if (is_causal && q_pos_offset + i < max_j) max_j = q_pos_offset + i;
    for (int64_t h = 0; h < n_heads; ++h) {
      const int64_t row = i * n_heads + h;
      const uint16_t* qr = q + row * head_dim;
      uint16_t* orow = out + row * head_dim;
      const uint16_t* kh = k + (h / group) * kv_head_stride;
      const uint16_t* vh = v + (h / group) * kv_head_stride;
      double m = -INFINITY;
      for (int64_t j = 0; j <= max_j; ++j) {
        double dot = 0.0;
        for (int64_t d = 0; d < head_dim; ++d)
          dot += (double)orc_f16_to_f32(qr[d]) * (double)orc_f16_to_f32(kh[j * head_dim + d]);
        const double sc = dot * scale_d;
        scores[j] = sc;
        if (sc > m) m = sc;
      }
      double sum = 0.0;
      if (max_j >= 0 && !(isinf(m) && m < 0.0)) {
        for (int64_t d = 0; d < head_dim; ++d) acc[d] = 0.0;
        for (int64_t j = 0; j <= max_j; ++j) {
          const double w = exp(scores[j] - m);
          sum += w;
          for (int64_t d = 0; d < head_dim; ++d)
            acc[d] += w * (double)orc_f16_to_f32(vh[j * head_dim + d]);
        }
      }
      if (sum == 0.0) {  /* no visible key, or all scores -inf */
        for (int64_t d = 0; d < head_dim; ++d) orow[d] = zero;
        if (out_lse) out_lse[row] = -INFINITY;
        continue;
      }
      const double inv = 1.0 / sum;
      for (int64_t d = 0; d < head_dim; ++d) orow[d] = orc_f32_to_f16((float)(acc[d] * inv));
      if (out_lse) out_lse[row] = (float)(m + log(sum));
    }
  }
  free(scores);
  free(acc);
  return 0;
}

/* The online-softmax form of the same attention, src/cpu_ref/attention_cpu.cpp:
 * 159-244: keys in tiles of 16; per tile the FP64 scores and their max m_b,
 * m' = max(m, m_b), alpha = exp(m - m') (0 while m = -inf), l and acc scaled by
 * alpha, then p = exp(s - m') added to l and p * v to acc.  The recurrence a
 * FlashAttention-2 kernel follows, in FP64.  Contract and empty handling as
 * orc_attention. */
int orc_attention_online(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out,
                         int64_t s_q, int64_t s_kv, int64_t n_heads, int64_t n_kv_heads,
                         int64_t head_dim, int64_t kv_head_stride, float scale,
                         int64_t q_pos_offset, int is_causal, float* out_lse) {
  enum { kTile = 16 };
  if (!q || !k || !v || !out) return 1;
  if (s_q < 0 || s_kv < 0 || q_pos_offset < 0 || n_heads <= 0 || n_kv_heads <= 0) return 1;
  if (n_heads % n_kv_heads != 0 || (head_dim != 64 && head_dim != 128) || !isfinite(scale))
    return 1;
  if (kv_head_stride < (s_kv > 0 ? s_kv * head_dim : 0)) return 1;
  if (s_q == 0) return 0;
  const uint16_t zero = orc_f32_to_f16(0.0f);
  if (s_kv == 0) {
    for (int64_t i = 0; i < s_q * n_heads * head_dim; ++i) out[i] = zero;
    if (out_lse)
      for (int64_t i = 0; i < s_q * n_heads; ++i) out_lse[i] = -INFINITY;
    return 0;
  }
  const int64_t group = n_heads / n_kv_heads;
  const double scale_d = (double)scale;
  double tile[kTile];
  double* acc = (double*)malloc((size_t)head_dim * sizeof(double));
  if (!acc) return 1;
  for (int64_t i = 0; i < s_q; ++i) {
    int64_t max_j = s_kv - 1;
    if (is_causal && q_pos_offset + i < max_j) max_j = q_pos_offset + i;
    for (int64_t h = 0; h < n_heads; ++h) {
      const int64_t row = i * n_heads + h;
      const uint16_t* qr = q + row * head_dim;
      uint16_t* orow = out + row * head_dim;
      const uint16_t* kh = k + (h / group) * kv_head_stride;
      const uint16_t* vh = v + (h / group) * kv_head_stride;
      double m = -INFINITY, l = 0.0;
      for (int64_t d = 0; d < head_dim; ++d) acc[d] = 0.0;
      for (int64_t j0 = 0; j0 <= max_j; j0 += kTile) {
        const int64_t j_end = (max_j + 1 < j0 + kTile) ? max_j + 1 : j0 + kTile;
        double mb = -INFINITY;
        for (int64_t j = j0; j < j_end; ++j) {
          double dot = 0.0;
          for (int64_t d = 0; d < head_dim; ++d)
            dot += (double)orc_f16_to_f32(qr[d]) * (double)orc_f16_to_f32(kh[j * head_dim + d]);
          tile[j - j0] = dot * scale_d;
          if (tile[j - j0] > mb) mb = tile[j - j0];
        }
        if (isinf(mb) && mb < 0.0) continue;
        const double mn = m > mb ? m : mb;
        const double alpha = (isinf(m) && m < 0.0) ? 0.0 : exp(m - mn);
        l *= alpha;
        for (int64_t d = 0; d < head_dim; ++d) acc[d] *= alpha;
        for (int64_t j = j0; j < j_end; ++j) {
          const double p = exp(tile[j - j0] - mn);
          l += p;
          for (int64_t d = 0; d < head_dim; ++d)
            acc[d] += p * (double)orc_f16_to_f32(vh[j * head_dim + d]);
        }
        m = mn;
      }
      if (l == 0.0) {
        for (int64_t d = 0; d < head_dim; ++d) orow[d] = zero;
        if (out_lse) out_lse[row] = -INFINITY;
        continue;
      }
      const double inv = 1.0 / l;
      for (int64_t d = 0; d < head_dim; ++d) orow[d] = orc_f32_to_f16((float)(acc[d] * inv));
      if (out_lse) out_lse[row] = (float)(m + log(l));
    }
  }
  free(acc);
  return 0;
}

/* ------------------------------------------------- all-cores (row-split) forms */

typedef struct {
  int kind;
  const void* a;
  const void* b;
  const void* c;
  const void* d;
  void* out;
  float* out32;
  int64_t r0, r1, N, K;
  float eps;
  int bf16;
} orc_job;

static void* orc_worker(void* p) {
  orc_job* j = (orc_job*)p;
  switch (j->kind) {
    case 0:
      matmul_rows((const float*)j->a, (const float*)j->b, (float*)j->out, j->r0, j->r1, j->N,
                  j->K);
      break;
    case 1:
      linear_rows((const uint16_t*)j->a, (const uint16_t*)j->b, (const uint16_t*)j->c,
                  (uint16_t*)j->out, j->r0, j->r1, j->N, j->K, j->bf16, j->out32);
      break;
    case 2:
      matmul16_rows((const uint16_t*)j->a, (const uint16_t*)j->b, (uint16_t*)j->out, j->out32,
                    j->r0, j->r1, j->N, j->K, j->bf16);
      break;
    case 3:
      rmsnorm_linear_f16_rows((const uint16_t*)j->a, (const uint16_t*)j->b,
                              (const uint16_t*)j->c, (const uint16_t*)j->d, (uint16_t*)j->out,
                              j->out32, j->r0, j->r1, j->N, j->K, j->eps);
      break;
    case 4:
      rmsnorm_linear_rows((const float*)j->a, (const float*)j->b, (const float*)j->c,
                          (float*)j->out, j->r0, j->r1, j->N, j->K, j->eps);
      break;
  }
  return NULL;
}

static void run_rows(orc_job proto, int64_t M, int nthreads) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  if ((int64_t)nthreads > M) nthreads = (int)(M > 0 ? M : 1);
  pthread_t tid[256];
  orc_job jobs[256];
  const int64_t per = (M + nthreads - 1) / nthreads;
  int launched = 0;
  for (int t = 0; t < nthreads; ++t) {
    jobs[t] = proto;
    jobs[t].r0 = t * per;
    jobs[t].r1 = (t + 1) * per < M ? (t + 1) * per : M;
    if (jobs[t].r0 >= jobs[t].r1) break;
    if (nthreads == 1) {
      orc_worker(&jobs[t]);
    } else {
      pthread_create(&tid[t], NULL, orc_worker, &jobs[t]);
      launched++;
    }
  }
  for (int t = 0; t < launched; ++t) pthread_join(tid[t], NULL);
}

void orc_matmul_mt(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                   int nthreads) {
  orc_job j = {0, A, B, NULL, NULL, C, NULL, 0, 0, N, K, 0.f, 0};
  run_rows(j, M, nthreads);
}

void orc_linear_f16_mt(const uint16_t* X, const uint16_t* W, const uint16_t* residual,
                       uint16_t* Y, int64_t M, int64_t N, int64_t K, int bf16, float* Y32,
                       int nthreads) {
  orc_job j = {1, X, W, residual, NULL, Y, Y32, 0, 0, N, K, 0.f, bf16};
  run_rows(j, M, nthreads);
}

void orc_matmul_f16_mt(const uint16_t* A, const uint16_t* B, uint16_t* C, float* C32, int64_t M,
                       int64_t N, int64_t K, int bf16, int nthreads) {
  orc_job j = {2, A, B, NULL, NULL, C, C32, 0, 0, N, K, 0.f, bf16};
  run_rows(j, M, nthreads);
}

void orc_rmsnorm_linear_f16_mt(const uint16_t* x, const uint16_t* gamma, const uint16_t* W,
                               const uint16_t* residual, uint16_t* Y, float* Y32, int64_t M,
                               int64_t N, int64_t K, float eps, int nthreads) {
  orc_job j = {3, x, gamma, W, residual, Y, Y32, 0, 0, N, K, eps, 0};
  run_rows(j, M, nthreads);
}

void orc_rmsnorm_linear_mt(const float* in, const float* rms_weight, const float* W, float* out,
                           int64_t M, int64_t N, int64_t K, float eps, int nthreads) {
  orc_job j = {4, in, rms_weight, W, NULL, out, NULL, 0, 0, N, K, eps, 0};
  run_rows(j, M, nthreads);
}

/* ---------------------------------------------------------------- block-quantised
 * The engine declares GGUF's block formats but implements neither a kernel nor
 * a CPU path for them (include/engine/dtype.hpp:95-125, kQuantBlockSize = 32, one
 * FP16 scale per block).  This is a restatement of the published format:
 *   qtype 8 (Q8_0): block = { uint16 d; int8 q[32] }      34 bytes, w = d * q
 *   qtype 4 (Q4_0): block = { uint16 d; uint8 nib[16] }   18 bytes,
 *                   w[j] = d * ((nib[j] & 15) - 8), w[j+16] = d * ((nib[j] >> 4) - 8)
 * Blocks are packed back to back, row-major (K/32 blocks per row); d is stored
 * little-endian.  A dequantised weight d * q is exact in float (an 11-bit
 * significand times an integer of at most 8 bits).  It is then accumulated
 * against x in double, like the other oracle dot products. */

static int orc_q_payload(int qtype) { return qtype == 8 ? 32 : 16; }

/* w[N*K] (float) from the packed blocks. */
void orc_dequant_q(int qtype, const uint8_t* blocks, float* w, int64_t N, int64_t K) {
  const int pay = orc_q_payload(qtype);
  const int64_t nblk = K / 32;
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t b = 0; b < nblk; ++b) {
      const uint8_t* blk = blocks + (n * nblk + b) * (2 + pay);
      const float d = orc_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
      float* out = w + n * K + b * 32;
      if (qtype == 8) {
        for (int i = 0; i < 32; ++i) out[i] = d * (float)(int8_t)blk[2 + i];
      } else {
        for (int j = 0; j < 16; ++j) {
          out[j] = d * (float)((int)(blk[2 + j] & 15) - 8);
          out[j + 16] = d * (float)((int)(blk[2 + j] >> 4) - 8);
        }
      }
    }
  }
}

/* y[n] = fp16( sum_k w[n,k] * x[k] (+ residual[n]) ), FP64 accumulation in
 * increasing k; y32 (optional) receives the unrounded value as float. */
void orc_gemv_q(int qtype, const uint8_t* blocks, const uint16_t* x, const uint16_t* residual,
                uint16_t* y, float* y32, int64_t N, int64_t K) {
  const int pay = orc_q_payload(qtype);
  const int64_t nblk = K / 32;
  float w[32];
  for (int64_t n = 0; n < N; ++n) {
    double acc = 0.0;
    for (int64_t b = 0; b < nblk; ++b) {
      orc_dequant_q(qtype, blocks + (n * nblk + b) * (2 + pay), w, 1, 32);
      for (int i = 0; i < 32; ++i) acc += (double)w[i] * (double)orc_f16_to_f32(x[b * 32 + i]);
    }
    if (residual) acc += (double)orc_f16_to_f32(residual[n]);
    if (y32) y32[n] = (float)acc;
    y[n] = orc_f32_to_f16((float)acc);
  }
}
