/*
 * vk_cpu_ref.c -- AVX-512 + OpenMP restatement of the reference's timed CPU
 * path (BENCHMARK BASELINE / TEST INFRASTRUCTURE ONLY).
 */
#include "vk_cpu_ref.h"

#include <immintrin.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ GEMM tiles
 * 6 rows x 64 columns of accumulators, ascending-K FMA (src/specialized.rs:1133-1148). */
static inline void tile_6x64(size_t rows, size_t k, size_t n, const float* a, size_t lda, const float* b,
                             size_t col0, __m512 acc[6][4]) {
  for (size_t r = 0; r < 6; ++r)
    for (int j = 0; j < 4; ++j) acc[r][j] = _mm512_setzero_ps();
  for (size_t kk = 0; kk < k; ++kk) {
    const float* bp = b + kk * n + col0;
    const __m512 b0 = _mm512_loadu_ps(bp), b1 = _mm512_loadu_ps(bp + 16), b2 = _mm512_loadu_ps(bp + 32),
                 b3 = _mm512_loadu_ps(bp + 48);
    for (size_t r = 0; r < rows; ++r) {
      const __m512 av = _mm512_set1_ps(a[r * lda + kk]);
      acc[r][0] = _mm512_fmadd_ps(av, b0, acc[r][0]);
      acc[r][1] = _mm512_fmadd_ps(av, b1, acc[r][1]);
      acc[r][2] = _mm512_fmadd_ps(av, b2, acc[r][2]);
      acc[r][3] = _mm512_fmadd_ps(av, b3, acc[r][3]);
    }
  }
}

void vkr_qkv(size_t tokens, const float* x, const float* w, const float* bias, float* q, float* k, float* v) {
  const size_t N = 2304, K = 768;
#pragma omp parallel for schedule(dynamic, 1)
  for (size_t col0 = 0; col0 < N; col0 += 64) {
    const size_t group = col0 / 768, head = (col0 % 768) / 64;
    float* dst = group == 0 ? q : (group == 1 ? k : v);
    __m512 acc[6][4];
    for (size_t row0 = 0; row0 < tokens; row0 += 6) {
      const size_t rows = tokens - row0 < 6 ? tokens - row0 : 6;
      tile_6x64(rows, K, N, x + row0 * K, K, w, col0, acc);
      for (size_t r = 0; r < rows; ++r) {
        float* p = dst + (head * tokens + row0 + r) * 64;
        for (int j = 0; j < 4; ++j)
          _mm512_storeu_ps(p + 16 * j, _mm512_add_ps(acc[r][j], _mm512_loadu_ps(bias + col0 + 16 * j)));
      }
    }
  }
}

void vkr_linear(size_t m, size_t n, size_t k, const float* a, const float* b, float* c) {
#pragma omp parallel for schedule(dynamic, 1)
  for (size_t col0 = 0; col0 < n; col0 += 64) {
    __m512 acc[6][4];
    for (size_t row0 = 0; row0 < m; row0 += 6) {
      const size_t rows = m - row0 < 6 ? m - row0 : 6;
      tile_6x64(rows, k, n, a + row0 * k, k, b, col0, acc);
      for (size_t r = 0; r < rows; ++r)
        for (int j = 0; j < 4; ++j) _mm512_storeu_ps(c + (row0 + r) * n + col0 + 16 * j, acc[r][j]);
    }
  }
}

void vkr_linear_bias_scale(size_t m, size_t n, size_t k, const float* a, const float* b, const float* bias,
                           const float* scale, float* c) {
  const size_t tiles = (m + 5) / 6;
#pragma omp parallel for schedule(dynamic, 1)
  for (size_t t = 0; t < tiles; ++t) {
    const size_t row0 = t * 6, rows = m - row0 < 6 ? m - row0 : 6;
    __m512 acc[6][4];
    for (size_t col0 = 0; col0 < n; col0 += 64) {
      tile_6x64(rows, k, n, a + row0 * k, k, b, col0, acc);
      for (size_t r = 0; r < rows; ++r)
        for (int j = 0; j < 4; ++j) {
          const size_t off = col0 + 16 * j;
          const __m512 o = _mm512_mul_ps(_mm512_add_ps(acc[r][j], _mm512_loadu_ps(bias + off)), _mm512_loadu_ps(scale + off));
          _mm512_storeu_ps(c + (row0 + r) * n + off, o);
        }
    }
  }
}

/* ------------------------------------------------------------------ exp / erf
 * Cephes-style vector exp (src/simd_avx512.rs:22-69, src/specialized.rs:2700-2744). */
static inline __m512 exp_avx512(__m512 x) {
  const __m512 one = _mm512_set1_ps(1.0f);
  x = _mm512_min_ps(x, _mm512_set1_ps(88.37626f));
  x = _mm512_max_ps(x, _mm512_set1_ps(-88.37626f));
  const __m512 fx0 = _mm512_fmadd_ps(x, _mm512_set1_ps(1.44269504f), _mm512_set1_ps(0.5f));
  const __m512 tr = _mm512_cvtepi32_ps(_mm512_cvttps_epi32(fx0));
  const __mmask16 gt = _mm512_cmp_ps_mask(tr, fx0, _CMP_GT_OQ);
  const __m512 fx = _mm512_mask_sub_ps(tr, gt, tr, one);
  x = _mm512_fnmadd_ps(fx, _mm512_set1_ps(0.693359375f), x);
  x = _mm512_fnmadd_ps(fx, _mm512_set1_ps(-2.12194440e-4f), x);
  const __m512 z = _mm512_mul_ps(x, x);
  __m512 y = _mm512_set1_ps(1.9875691500e-4f);
  y = _mm512_fmadd_ps(y, x, _mm512_set1_ps(1.3981999507e-3f));
  y = _mm512_fmadd_ps(y, x, _mm512_set1_ps(8.3334519073e-3f));
  y = _mm512_fmadd_ps(y, x, _mm512_set1_ps(4.1665795894e-2f));
  y = _mm512_fmadd_ps(y, x, _mm512_set1_ps(1.6666665459e-1f));
  y = _mm512_fmadd_ps(y, x, _mm512_set1_ps(5.0000001201e-1f));
  y = _mm512_fmadd_ps(y, z, x);
  y = _mm512_add_ps(y, one);
  const __m512i e = _mm512_slli_epi32(_mm512_add_epi32(_mm512_cvttps_epi32(fx), _mm512_set1_epi32(0x7f)), 23);
  return _mm512_mul_ps(y, _mm512_castsi512_ps(e));
}

/* src/simd_avx512.rs:141-177 */
static inline __m512 erf_avx512(__m512 x) {
  const __m512 one = _mm512_set1_ps(1.0f);
  const __m512 xa = _mm512_castsi512_ps(_mm512_and_epi32(_mm512_castps_si512(x), _mm512_set1_epi32(0x7fffffff)));
  const __mmask16 neg = _mm512_cmp_ps_mask(x, _mm512_setzero_ps(), _CMP_LT_OQ);
  const __m512 sign = _mm512_mask_blend_ps(neg, one, _mm512_set1_ps(-1.0f));
  const __m512 t = _mm512_div_ps(one, _mm512_fmadd_ps(_mm512_set1_ps(0.3275911f), xa, one));
  __m512 p = _mm512_set1_ps(1.0614054f);
  p = _mm512_fmadd_ps(p, t, _mm512_set1_ps(-1.4531520f));
  p = _mm512_fmadd_ps(p, t, _mm512_set1_ps(1.4214137f));
  p = _mm512_fmadd_ps(p, t, _mm512_set1_ps(-0.28449674f));
  p = _mm512_fmadd_ps(p, t, _mm512_set1_ps(0.25482959f));
  p = _mm512_mul_ps(p, t);
  const __m512 e = exp_avx512(_mm512_sub_ps(_mm512_setzero_ps(), _mm512_mul_ps(xa, xa)));
  return _mm512_mul_ps(sign, _mm512_fnmadd_ps(p, e, one));
}

void vkr_gelu(float* x, size_t n) {
  const size_t chunks = (n + 4095) / 4096;
#pragma omp parallel for schedule(static)
  for (size_t c = 0; c < chunks; ++c) {
    const size_t i0 = c * 4096, i1 = i0 + 4096 < n ? i0 + 4096 : n;
    size_t i = i0;
    for (; i + 16 <= i1; i += 16) {
      const __m512 v = _mm512_loadu_ps(x + i);
      const __m512 e = erf_avx512(_mm512_mul_ps(v, _mm512_set1_ps(0.70710678f)));
      _mm512_storeu_ps(x + i, _mm512_mul_ps(_mm512_mul_ps(_mm512_set1_ps(0.5f), v), _mm512_add_ps(_mm512_set1_ps(1.0f), e)));
    }
    if (i < i1) vko_gelu(x + i, i1 - i);
  }
}

void vkr_add(float* dst, const float* src, size_t n) {
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < n; i += 16) {
    if (i + 16 <= n)
      _mm512_storeu_ps(dst + i, _mm512_add_ps(_mm512_loadu_ps(dst + i), _mm512_loadu_ps(src + i)));
    else
      for (size_t j = i; j < n; ++j) dst[j] += src[j];
  }
}

/* ------------------------------------------------------------------ flash attention */
#define QT 8
#define KVT 64

static void flash_tile(const float* qh, const float* vh, const float* kp, size_t stride, size_t tokens, size_t q0,
                       size_t rows, float* out) {
  __m512 accum[QT][4];
  float sums[QT], maxima[QT];
  for (size_t r = 0; r < QT; ++r) {
    for (int j = 0; j < 4; ++j) accum[r][j] = _mm512_setzero_ps();
    sums[r] = 0.0f;
    maxima[r] = -INFINITY;
  }
  float scores[QT][KVT] __attribute__((aligned(64)));
  for (size_t k0 = 0; k0 < tokens; k0 += KVT) {
    const size_t cols = tokens - k0 < KVT ? tokens - k0 : KVT;
    /* QK^T: 8 x 32 micro-kernels (src/specialized.rs:2331), dimension-major K */
    for (int half = 0; half < 2; ++half) {
      __m512 acc[QT][2];
      for (size_t r = 0; r < QT; ++r) acc[r][0] = acc[r][1] = _mm512_setzero_ps();
      for (size_t d = 0; d < 64; ++d) {
        const float* kr = kp + d * stride + k0 + half * 32;
        const __m512 b0 = _mm512_loadu_ps(kr), b1 = _mm512_loadu_ps(kr + 16);
        for (size_t r = 0; r < rows; ++r) {
          const __m512 av = _mm512_set1_ps(qh[(q0 + r) * 64 + d]);
          acc[r][0] = _mm512_fmadd_ps(av, b0, acc[r][0]);
          acc[r][1] = _mm512_fmadd_ps(av, b1, acc[r][1]);
        }
      }
      for (size_t r = 0; r < rows; ++r) {
        _mm512_store_ps(&scores[r][half * 32], acc[r][0]);
        _mm512_store_ps(&scores[r][half * 32 + 16], acc[r][1]);
      }
    }
    /* online softmax (src/specialized.rs:1489-1515) */
    for (size_t r = 0; r < rows; ++r) {
      float tile_max = -INFINITY;
      for (size_t c = 0; c < cols; ++c) {
        scores[r][c] *= 0.125f;
        tile_max = fmaxf(tile_max, scores[r][c]);
      }
      const float new_max = fmaxf(maxima[r], tile_max);
      const float corr = isfinite(maxima[r]) ? expf(maxima[r] - new_max) : 0.0f;
      sums[r] *= corr;
      const __m512 cv = _mm512_set1_ps(corr);
      for (int j = 0; j < 4; ++j) accum[r][j] = _mm512_mul_ps(accum[r][j], cv);
      for (size_t c = 0; c < KVT; ++c) scores[r][c] -= new_max;
      for (int j = 0; j < 4; ++j) _mm512_store_ps(&scores[r][16 * j], exp_avx512(_mm512_load_ps(&scores[r][16 * j])));
      for (size_t c = 0; c < cols; ++c) sums[r] += scores[r][c];
      maxima[r] = new_max;
    }
    /* P.V (src/specialized.rs:1523-1550) */
    for (size_t c = 0; c < cols; ++c) {
      const float* vr = vh + (k0 + c) * 64;
      const __m512 v0 = _mm512_loadu_ps(vr), v1 = _mm512_loadu_ps(vr + 16), v2 = _mm512_loadu_ps(vr + 32),
                   v3 = _mm512_loadu_ps(vr + 48);
      for (size_t r = 0; r < rows; ++r) {
        const __m512 p = _mm512_set1_ps(scores[r][c]);
        accum[r][0] = _mm512_fmadd_ps(p, v0, accum[r][0]);
        accum[r][1] = _mm512_fmadd_ps(p, v1, accum[r][1]);
        accum[r][2] = _mm512_fmadd_ps(p, v2, accum[r][2]);
        accum[r][3] = _mm512_fmadd_ps(p, v3, accum[r][3]);
      }
    }
  }
  for (size_t r = 0; r < rows; ++r) {
    const __m512 inv = _mm512_set1_ps(1.0f / sums[r]);
    for (int j = 0; j < 4; ++j) _mm512_storeu_ps(out + (q0 + r) * 64 + 16 * j, _mm512_mul_ps(accum[r][j], inv));
  }
}

void vkr_flash_attention(const float* q, const float* k, const float* v, size_t heads, size_t tokens, float* out) {
  const size_t stride = (tokens + KVT - 1) / KVT * KVT;
  float* packed = (float*)aligned_alloc(64, sizeof(float) * heads * 64 * stride);
  memset(packed, 0, sizeof(float) * heads * 64 * stride);
#pragma omp parallel for schedule(static)
  for (size_t h = 0; h < heads; ++h)  /* src/specialized.rs:1307-1318 */
    for (size_t t = 0; t < tokens; ++t)
      for (size_t d = 0; d < 64; ++d) packed[(h * 64 + d) * stride + t] = k[(h * tokens + t) * 64 + d];
  const size_t tiles = (tokens + QT - 1) / QT;
#pragma omp parallel for schedule(dynamic, 4)
  for (size_t i = 0; i < heads * tiles; ++i) {
    const size_t h = i / tiles, t = i % tiles;
    const size_t q0 = t * QT, rows = tokens - q0 < QT ? tokens - q0 : QT;
    flash_tile(q + h * tokens * 64, v + h * tokens * 64, packed + h * 64 * stride, stride, tokens, q0, rows,
               out + h * tokens * 64);
  }
  free(packed);
}

/* ------------------------------------------------------------------ block */
void vkr_encoder_layer(float* x, size_t tokens, size_t grid_h, size_t grid_w, const vko_layer* w, float eps,
                       float rope_freq) {
  const size_t T = tokens, E = 768, F = 3072, H = 12;
  float* h = (float*)malloc(sizeof(float) * T * E);
  float* q = (float*)malloc(sizeof(float) * T * E);
  float* k = (float*)malloc(sizeof(float) * T * E);
  float* v = (float*)malloc(sizeof(float) * T * E);
  float* att = (float*)malloc(sizeof(float) * T * E);
  float* tok = (float*)malloc(sizeof(float) * T * E);
  float* o = (float*)malloc(sizeof(float) * T * E);
  float* f = (float*)malloc(sizeof(float) * T * F);
  int64_t* pos = (int64_t*)malloc(sizeof(int64_t) * 2 * T);
  vko_da3_positions(grid_h, grid_w, pos);

  memcpy(h, x, sizeof(float) * T * E);
  vko_layernorm(h, T, E, w->ln1_g, w->ln1_b, eps);
  vkr_qkv(T, h, w->qkv_w, w->qkv_b, q, k, v);
  vko_rope2d(q, H, T, 64, pos, rope_freq);
  vko_rope2d(k, H, T, 64, pos, rope_freq);
  vkr_flash_attention(q, k, v, H, T, att);
#pragma omp parallel for schedule(static)
  for (size_t t = 0; t < T; ++t)
    for (size_t hh = 0; hh < H; ++hh) memcpy(tok + t * E + hh * 64, att + (hh * T + t) * 64, 64 * sizeof(float));
  vkr_linear_bias_scale(T, E, E, tok, w->proj_w, w->proj_b, w->ls1, o);
  vkr_add(x, o, T * E);

  memcpy(h, x, sizeof(float) * T * E);
  vko_layernorm(h, T, E, w->ln2_g, w->ln2_b, eps);
  vkr_linear(T, F, E, h, w->fc1_w, f);
  vko_add_bias_rows(f, T, F, w->fc1_b);
  vkr_gelu(f, T * F);
  vkr_linear_bias_scale(T, E, F, f, w->fc2_w, w->fc2_b, w->ls2, o);
  vkr_add(x, o, T * E);

  free(h); free(q); free(k); free(v); free(att); free(tok); free(o); free(f); free(pos);
}
