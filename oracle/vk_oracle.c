/*
 * vk_oracle.c -- CPU restatement of the vestra-kernels reference arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker; never on the product path).
 *
 * Compile with -ffp-contract=off: Rust never contracts a*b+c into an FMA, so
 * every multiply-add below is two rounded operations unless the reference
 * itself uses an FMA intrinsic, in which case fmaf() is called explicitly.
 * Rust's `iter().sum::<f32>()` is a left fold that starts from -0.0; the
 * folds below start from -0.0f for the same reason.
 */
#include "vk_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* src/cuda.rs:295-316 (kernel) and 1073-1093 (shape checks) */
int vko_patchify_nchw(const float* image, size_t height, size_t width, size_t patch, size_t channels,
                      float* patches) {
  if (height == 0 || width == 0 || patch == 0 || channels == 0 || height % patch != 0 || width % patch != 0)
    return -1;
  const size_t area = patch * patch, row_width = channels * area, grid_w = width / patch;
  const size_t count = (height / patch) * grid_w * row_width;
  for (size_t index = 0; index < count; ++index) {
    const size_t p = index / row_width, within = index % row_width;
    const size_t c = within / area, spatial = within % area;
    const size_t y = (p / grid_w) * patch + spatial / patch;
    const size_t x = (p % grid_w) * patch + spatial % patch;
    patches[index] = image[(c * height + y) * width + x];
  }
  return 0;
}

/* src/cuda.rs:321-334: value + position, cls for token 0 */
void vko_prepend_cls_add_pos(const float* patches, const float* cls, const float* position, size_t patch_count,
                             size_t embed, float* tokens) {
  const size_t len = (patch_count + 1) * embed;
  for (size_t index = 0; index < len; ++index) {
    const size_t token = index / embed, channel = index % embed;
    const float value = token == 0 ? cls[channel] : patches[(token - 1) * embed + channel];
    tokens[index] = value + position[index];
  }
}

void vko_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* ------------------------------------------------------------------ */
/* half / bfloat16 conversions                                         */
/* ------------------------------------------------------------------ */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* IEEE-754 binary32 -> binary16, round to nearest, ties to even (the rule
 * half::f16::from_f32 implements, in hardware through F16C or in software). */
uint16_t vko_f16_from_f32(float x) {
  uint32_t u = f2u(x);
  uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
  uint32_t exp = (u >> 23) & 0xffu;
  uint32_t man = u & 0x7fffffu;
  if (exp == 0xffu) { /* inf / nan */
    if (man == 0) return sign | 0x7c00u;
    return sign | 0x7e00u | (uint16_t)(man >> 13);
  }
  int e = (int)exp - 127 + 15;
  if (e >= 0x1f) return sign | 0x7c00u; /* overflow -> inf */
  if (e <= 0) {
    /* subnormal half (or zero) */
    if (e < -10) return sign; /* rounds to zero */
    uint32_t m = man | 0x800000u;     /* implicit bit */
    int shift = 14 - e;               /* 24-bit mantissa -> 10-bit field */
    uint32_t half_m = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (half_m & 1u))) half_m++;
    return sign | (uint16_t)half_m;
  }
  uint32_t half_m = man >> 13;
  uint32_t rem = man & 0x1fffu;
  uint16_t h = sign | (uint16_t)((uint32_t)e << 10) | (uint16_t)half_m;
  if (rem > 0x1000u || (rem == 0x1000u && (half_m & 1u))) h++; /* carries into exp ok */
  return h;
}

float vko_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  if (exp == 0) {
    if (man == 0) return u2f(sign);
    /* subnormal: value = man * 2^-24, exact in f32 */
    float v = (float)man * 5.9604644775390625e-8f;
    return sign ? -v : v;
  }
  if (exp == 0x1f) return u2f(sign | 0x7f800000u | (man << 13));
  return u2f(sign | ((exp - 15 + 127) << 23) | (man << 13));
}

float vko_round_bf16(float x) {
  uint32_t u = f2u(x);
  if ((u & 0x7f800000u) == 0x7f800000u) { /* inf / nan */
    if (u & 0x7fffffu) return u2f((u | 0x400000u) & 0xffff0000u);
    return x;
  }
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return u2f(u & 0xffff0000u);
}

/* ------------------------------------------------------------------ */
/* src/scalar.rs                                                       */
/* ------------------------------------------------------------------ */

/* src/scalar.rs:3-18: c[i,j] = 0; for p: c[i,j] += a[i,p] * b[p,j].  The
 * rows are independent and each element keeps its ascending-p order. */
void vko_gemm_f32(size_t m, size_t n, size_t k, const float* a, const float* b, float* c) {
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < m; ++i) {
    float* ci = c + i * n;
    for (size_t j = 0; j < n; ++j) ci[j] = 0.0f;
    for (size_t p = 0; p < k; ++p) {
      const float aip = a[i * k + p];
      const float* bp = b + p * n;
      for (size_t j = 0; j < n; ++j) ci[j] += aip * bp[j];
    }
  }
}

/* src/scalar.rs:25-56: acc += d_a * d_b * isum over ascending blocks. */
void vko_gemm_q8_0(size_t m, size_t n, size_t k, const vko_block_q8_0* a_q,
                   const vko_block_q8_0* b_q, float* c) {
  const size_t nb = k / VKO_QK8_0;
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < m; ++i) {
    const vko_block_q8_0* ar = a_q + i * nb;
    for (size_t j = 0; j < n; ++j) {
      const vko_block_q8_0* br = b_q + j * nb;
      float acc = 0.0f;
      for (size_t bi = 0; bi < nb; ++bi) {
        int32_t isum = 0;
        for (int l = 0; l < VKO_QK8_0; ++l) isum += (int32_t)ar[bi].qs[l] * (int32_t)br[bi].qs[l];
        acc += vko_f16_to_f32(ar[bi].d) * vko_f16_to_f32(br[bi].d) * (float)isum;
      }
      c[i * n + j] = acc;
    }
  }
}

void vko_q8_0_block_dots(size_t m, size_t n, size_t k, const vko_block_q8_0* a_q,
                         const vko_block_q8_0* b_q, int32_t* out) {
  const size_t nb = k / VKO_QK8_0;
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < m; ++i)
    for (size_t j = 0; j < n; ++j)
      for (size_t bi = 0; bi < nb; ++bi) {
        int32_t isum = 0;
        for (int l = 0; l < VKO_QK8_0; ++l)
          isum += (int32_t)a_q[i * nb + bi].qs[l] * (int32_t)b_q[j * nb + bi].qs[l];
        out[(i * n + j) * nb + bi] = isum;
      }
}

/* src/lib.rs:42-50 */
void vko_dequantize_q8_0(const vko_block_q8_0* blocks, size_t nblocks, float* out) {
  for (size_t b = 0; b < nblocks; ++b) {
    const float scale = vko_f16_to_f32(blocks[b].d);
    for (int l = 0; l < VKO_QK8_0; ++l) out[b * VKO_QK8_0 + l] = scale * (float)blocks[b].qs[l];
  }
}

/* Rust f32::max: returns the non-NaN operand when one is NaN. */
static inline float rs_max(float a, float b) { return fmaxf(a, b); }

/* src/q8_0_dot.rs:27-46.  amax folds from 0 with f32::max; d = amax / 127;
 * inv_d is computed from the f32 d (not the rounded f16); round() is
 * half-away-from-zero (C roundf); clamp to [-127, 127] then truncate to i8. */
void vko_quantize_row_q8_0(const float* x, size_t nblocks, vko_block_q8_0* out) {
  for (size_t bi = 0; bi < nblocks; ++bi) {
    const float* src = x + bi * VKO_QK8_0;
    float amax = 0.0f;
    for (int j = 0; j < VKO_QK8_0; ++j) amax = rs_max(amax, fabsf(src[j]));
    const float d = amax / 127.0f;
    const float inv_d = (d != 0.0f) ? 1.0f / d : 0.0f;
    out[bi].d = vko_f16_from_f32(d);
    for (int j = 0; j < VKO_QK8_0; ++j) {
      float q = roundf(src[j] * inv_d);
      if (q < -127.0f) q = -127.0f;
      if (q > 127.0f) q = 127.0f;
      out[bi].qs[j] = (int8_t)q;
    }
  }
}

/* src/scalar.rs:58-63 */
void vko_add(float* dst, const float* src, size_t n) {
  for (size_t i = 0; i < n; ++i) dst[i] += src[i];
}

/* src/scalar.rs:65-81 */
void vko_add_bias_rows(float* x, size_t rows, size_t cols, const float* bias) {
#pragma omp parallel for schedule(static)
  for (size_t r = 0; r < rows; ++r)
    for (size_t c = 0; c < cols; ++c) x[r * cols + c] += bias[c];
}

/* src/scalar.rs:97-114 */
static void layernorm_row(float* row, size_t cols, const float* gamma, const float* beta,
                          float eps) {
  float s = -0.0f;
  for (size_t c = 0; c < cols; ++c) s += row[c];
  const float mean = s / (float)cols;
  float v = -0.0f;
  for (size_t c = 0; c < cols; ++c) {
    const float d = row[c] - mean;
    v += d * d;
  }
  const float var = v / (float)cols;
  const float inv = 1.0f / sqrtf(var + eps);
  for (size_t c = 0; c < cols; ++c) row[c] = (row[c] - mean) * inv * gamma[c] + beta[c];
}

/* src/scalar.rs:83-95 */
void vko_layernorm(float* x, size_t rows, size_t cols, const float* gamma, const float* beta,
                   float eps) {
#pragma omp parallel for schedule(static)
  for (size_t r = 0; r < rows; ++r) layernorm_row(x + r * cols, cols, gamma, beta, eps);
}

/* src/scalar.rs:124-134: Abramowitz-Stegun 7.1.26.  Rust's signum is +1 for
 * +0.0 and -1 for -0.0. */
float vko_erf(float x) {
  const float s = signbit(x) ? -1.0f : 1.0f;
  x = fabsf(x);
  const float t = 1.0f / (1.0f + 0.3275911f * x);
  const float poly =
      ((((1.0614054f * t - 1.453152f) * t) + 1.4214137f) * t - 0.28449674f) * t + 0.2548296f;
  const float y = 1.0f - poly * t * expf(-x * x);
  return s * y;
}

/* src/scalar.rs:116-121 */
void vko_gelu(float* x, size_t n) {
  const float inv_sqrt2 = 0.70710678118654752440f; /* std::f32::consts::FRAC_1_SQRT_2 */
  for (size_t i = 0; i < n; ++i) {
    const float v = x[i];
    x[i] = 0.5f * v * (1.0f + vko_erf(v * inv_sqrt2));
  }
}

/* src/scalar.rs:139-155 */
void vko_layerscale(float* x, size_t rows, size_t cols, const float* gamma) {
  for (size_t r = 0; r < rows; ++r)
    for (size_t c = 0; c < cols; ++c) x[r * cols + c] *= gamma[c];
}

/* src/scalar.rs:157-172 */
void vko_softmax_rows(float* x, size_t rows, size_t cols) {
  for (size_t r = 0; r < rows; ++r) {
    float* row = x + r * cols;
    float m = -INFINITY;
    for (size_t c = 0; c < cols; ++c) m = rs_max(m, row[c]);
    float sum = 0.0f;
    for (size_t c = 0; c < cols; ++c) {
      row[c] = expf(row[c] - m);
      sum += row[c];
    }
    const float inv = 1.0f / sum;
    for (size_t c = 0; c < cols; ++c) row[c] *= inv;
  }
}

/* ------------------------------------------------------------------ */
/* src/attention.rs                                                    */
/* ------------------------------------------------------------------ */

static inline float dot_seq(const float* a, const float* b, size_t n) {
  float s = -0.0f;
  for (size_t i = 0; i < n; ++i) s += a[i] * b[i];
  return s;
}

/* src/attention.rs:10-59.  Rows are independent; each keeps the reference
 * order (scores, max, exp and sum over all n keys, then weighted V sum). */
void vko_attention_naive(const float* q, const float* k, const float* v, size_t heads, size_t n,
                         size_t head_dim, float* out) {
  const float scale = 1.0f / sqrtf((float)head_dim);
#pragma omp parallel
  {
    float* scores = (float*)malloc(sizeof(float) * (n ? n : 1));
#pragma omp for schedule(static)
    for (size_t row = 0; row < heads * n; ++row) {
      const size_t h = row / n, i = row % n;
      const float* qh = q + h * n * head_dim;
      const float* kh = k + h * n * head_dim;
      const float* vh = v + h * n * head_dim;
      const float* qi = qh + i * head_dim;
      float max_score = -INFINITY;
      for (size_t j = 0; j < n; ++j) {
        const float s = dot_seq(qi, kh + j * head_dim, head_dim) * scale;
        scores[j] = s;
        if (s > max_score) max_score = s;
      }
      float sum = 0.0f;
      for (size_t j = 0; j < n; ++j) {
        scores[j] = expf(scores[j] - max_score);
        sum += scores[j];
      }
      const float inv_sum = 1.0f / sum;
      float* oi = out + row * head_dim;
      for (size_t d = 0; d < head_dim; ++d) oi[d] = 0.0f;
      for (size_t j = 0; j < n; ++j) {
        const float w = scores[j] * inv_sum;
        const float* vj = vh + j * head_dim;
        for (size_t d = 0; d < head_dim; ++d) oi[d] += w * vj[d];
      }
    }
    free(scores);
  }
}

#define VKO_KV_TILE 64

/* src/attention.rs:111-201 with use_avx512 == false. */
static void attention_row(const float* qh, const float* kh, const float* vh, size_t i, size_t n,
                          size_t head_dim, float scale, float* acc, float* oi) {
  const float* qi = qh + i * head_dim;
  float running_max = -INFINITY;
  float running_sum = 0.0f;
  for (size_t d = 0; d < head_dim; ++d) acc[d] = 0.0f;
  size_t j0 = 0;
  while (j0 < n) {
    const size_t j1 = (j0 + VKO_KV_TILE < n) ? j0 + VKO_KV_TILE : n;
    float local[VKO_KV_TILE];
    float tile_max = -INFINITY;
    for (size_t j = j0; j < j1; ++j) {
      const float score = dot_seq(qi, kh + j * head_dim, head_dim) * scale;
      local[j - j0] = score;
      if (score > tile_max) tile_max = score;
    }
    const float new_max = rs_max(running_max, tile_max);
    const float correction = isfinite(running_max) ? expf(running_max - new_max) : 0.0f;
    running_sum *= correction;
    for (size_t d = 0; d < head_dim; ++d) acc[d] *= correction;
    for (size_t t = 0; t < j1 - j0; ++t) local[t] -= new_max;
    for (size_t t = 0; t < j1 - j0; ++t) local[t] = expf(local[t]);
    for (size_t j = j0; j < j1; ++j) {
      const float p = local[j - j0];
      running_sum += p;
      const float* vj = vh + j * head_dim;
      for (size_t d = 0; d < head_dim; ++d) acc[d] += p * vj[d];
    }
    running_max = new_max;
    j0 = j1;
  }
  const float inv_sum = 1.0f / running_sum;
  for (size_t d = 0; d < head_dim; ++d) oi[d] = acc[d] * inv_sum;
}

/* src/attention.rs:66-108 (the tiled online route). */
void vko_attention(const float* q, const float* k, const float* v, size_t heads, size_t n,
                   size_t head_dim, float* out) {
  const float scale = 1.0f / sqrtf((float)head_dim);
#pragma omp parallel
  {
    float* acc = (float*)malloc(sizeof(float) * (head_dim ? head_dim : 1));
#pragma omp for schedule(static)
    for (size_t row = 0; row < heads * n; ++row) {
      const size_t h = row / n, i = row % n;
      const size_t base = h * n * head_dim;
      attention_row(q + base, k + base, v + base, i, n, head_dim, scale, acc,
                    out + row * head_dim);
    }
    free(acc);
  }
}

/* ------------------------------------------------------------------ */
/* RoPE: src/rope.rs and src/specialized.rs                            */
/* ------------------------------------------------------------------ */

/* src/rope.rs:84-93 */
static void rotate_half(float* slice, size_t quarter, const float* rot) {
  for (size_t i = 0; i < quarter; ++i) {
    const float s = rot[i * 2], c = rot[i * 2 + 1];
    const float a = slice[i], b = slice[i + quarter];
    slice[i] = a * c - b * s;
    slice[i + quarter] = b * c + a * s;
  }
}

/* src/rope.rs:30-81 */
void vko_rope2d(float* x, size_t heads, size_t n, size_t head_dim, const int64_t* pos_yx,
                float freq) {
  const size_t half_dim = head_dim / 2, quarter = half_dim / 2;
  float* inv_freq = (float*)malloc(sizeof(float) * (quarter ? quarter : 1));
  for (size_t i = 0; i < quarter; ++i)
    inv_freq[i] = powf(freq, -2.0f * (float)i / (float)half_dim);
  float* rot = (float*)malloc(sizeof(float) * (quarter ? 4 * quarter : 1));
  for (size_t p = 0; p < n; ++p) {
    const float pos[2] = {(float)pos_yx[2 * p], (float)pos_yx[2 * p + 1]};
    for (int axis = 0; axis < 2; ++axis)
      for (size_t i = 0; i < quarter; ++i) {
        const float ang = pos[axis] * inv_freq[i];
        rot[(axis * quarter + i) * 2] = sinf(ang);
        rot[(axis * quarter + i) * 2 + 1] = cosf(ang);
      }
    for (size_t h = 0; h < heads; ++h) {
      float* base = x + (h * n + p) * head_dim;
      rotate_half(base, quarter, rot);
      rotate_half(base + half_dim, quarter, rot + quarter * 2);
    }
  }
  free(rot);
  free(inv_freq);
}

/* src/specialized.rs:389-410 (QUARTER = 16, HALF_DIM = 32). */
void vko_rope_rotations(const int64_t* pos_yx, size_t tokens, float freq, float* rotations) {
  float inv_freq[16];
  for (int i = 0; i < 16; ++i) inv_freq[i] = powf(freq, -2.0f * (float)i / 32.0f);
  for (size_t t = 0; t < tokens; ++t)
    for (int axis = 0; axis < 2; ++axis) {
      const float pos = (float)pos_yx[2 * t + axis];
      for (int i = 0; i < 16; ++i) {
        const float ang = pos * inv_freq[i];
        const size_t off = (t * 32 + (size_t)axis * 16 + (size_t)i) * 2;
        rotations[off] = sinf(ang);
        rotations[off + 1] = cosf(ang);
      }
    }
}

/* src/specialized.rs:412-454 */
static void normalize_and_rotate(float* values, size_t rows, size_t tokens, const float* gamma,
                                 const float* beta, float eps, const float* rot) {
#pragma omp parallel for schedule(static)
  for (size_t row = 0; row < rows; ++row) {
    float* data = values + row * 64;
    layernorm_row(data, 64, gamma, beta, eps);
    const size_t token = row % tokens;
    for (int axis = 0; axis < 2; ++axis) {
      const float* r = rot + (token * 32 + (size_t)axis * 16) * 2;
      rotate_half(data + axis * 32, 16, r);
    }
  }
}

void vko_qk_norm_rope(float* q, float* k, size_t heads, size_t tokens, const float* q_gamma,
                      const float* q_beta, const float* k_gamma, const float* k_beta,
                      const int64_t* pos_yx, float freq, float eps) {
  float* rot = (float*)malloc(sizeof(float) * tokens * 64);
  vko_rope_rotations(pos_yx, tokens, freq, rot);
  normalize_and_rotate(q, heads * tokens, tokens, q_gamma, q_beta, eps, rot);
  normalize_and_rotate(k, heads * tokens, tokens, k_gamma, k_beta, eps, rot);
  free(rot);
}

void vko_da3_positions(size_t grid_h, size_t grid_w, int64_t* pos_yx) {
  pos_yx[0] = 0;
  pos_yx[1] = 0;
  for (size_t p = 0; p < grid_h * grid_w; ++p) {
    pos_yx[2 * (p + 1)] = (int64_t)(p / grid_w + 1);
    pos_yx[2 * (p + 1) + 1] = (int64_t)(p % grid_w + 1);
  }
}

/* ------------------------------------------------------------------ */
/* Specialised projections (src/specialized.rs)                        */
/* ------------------------------------------------------------------ */

/* The specialised AVX-512 projections accumulate with one FMA per k in
 * ascending order (src/specialized.rs:1133-1148, :943-955), which fmaf
 * restates exactly. */
static void gemm_fma_rows(size_t m, size_t n, size_t k, const float* a, const float* b,
                          float* c) {
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < m; ++i) {
    float* ci = c + i * n;
    for (size_t j = 0; j < n; ++j) ci[j] = 0.0f;
    for (size_t p = 0; p < k; ++p) {
      const float aip = a[i * k + p];
      const float* bp = b + p * n;
      for (size_t j = 0; j < n; ++j) ci[j] = fmaf(aip, bp[j], ci[j]);
    }
  }
}

/* src/specialized.rs:1101-1167: acc + bias, stored head-major. */
void vko_qkv(size_t tokens, size_t heads, const float* x, const float* w, const float* bias,
             float* q, float* k, float* v) {
  const size_t e = heads * 64, n3 = 3 * e;
  float* tmp = (float*)malloc(sizeof(float) * tokens * n3);
  gemm_fma_rows(tokens, n3, e, x, w, tmp);
  for (size_t t = 0; t < tokens; ++t)
    for (size_t col = 0; col < n3; ++col) {
      const size_t g = col / e, h = (col % e) / 64, d = col % 64;
      float* dst = g == 0 ? q : (g == 1 ? k : v);
      dst[(h * tokens + t) * 64 + d] = tmp[t * n3 + col] + bias[col];
    }
  free(tmp);
}

/* src/specialized.rs:880-991: (acc + bias) * scale. */
void vko_linear_bias_scale(size_t m, size_t n, size_t k, const float* a, const float* b,
                           const float* bias, const float* scale, float* c) {
  gemm_fma_rows(m, n, k, a, b, c);
  for (size_t i = 0; i < m; ++i)
    for (size_t j = 0; j < n; ++j) c[i * n + j] = (c[i * n + j] + bias[j]) * scale[j];
}

/* ------------------------------------------------------------------ */
/* Engine-side block composition                                       */
/* ------------------------------------------------------------------ */

static void round_bf16_buf(float* x, size_t n) {
  for (size_t i = 0; i < n; ++i) x[i] = vko_round_bf16(x[i]);
}

static float* copy_maybe_bf16(const float* src, size_t n, int bf16) {
  float* d = (float*)malloc(sizeof(float) * n);
  memcpy(d, src, sizeof(float) * n);
  if (bf16) round_bf16_buf(d, n);
  return d;
}

static void round_f16_buf(float* x, size_t n) {
  for (size_t i = 0; i < n; ++i) x[i] = vko_f16_to_f32(vko_f16_from_f32(x[i]));
}

/* Q8_0 weights as Kernels::gemm_q8_0 takes them: the [K, N] input-major
 * weight transposed to [N, K] rows (src/dispatch.rs:85-90), each row
 * quantised with quantize_row_q8_0 (src/q8_0_dot.rs:27-46). */
static vko_block_q8_0* quantize_weight_q8(const float* w_kn, size_t k, size_t n) {
  float* row = (float*)malloc(sizeof(float) * k);
  vko_block_q8_0* blocks = (vko_block_q8_0*)malloc(sizeof(vko_block_q8_0) * n * (k / VKO_QK8_0));
  for (size_t j = 0; j < n; ++j) {
    for (size_t p = 0; p < k; ++p) row[p] = w_kn[p * n + j];
    vko_quantize_row_q8_0(row, k / VKO_QK8_0, blocks + j * (k / VKO_QK8_0));
  }
  free(row);
  return blocks;
}

/* c [m, n] = gemm_q8_0(quantize(a), wq): activations quantised per 32-block
 * of each row, then the reference's block-ascending f32 fold
 * (src/scalar.rs:25-56). */
static void linear_q8(size_t m, size_t n, size_t k, const float* a, const vko_block_q8_0* wq, float* c) {
  const size_t nb = k / VKO_QK8_0;
  vko_block_q8_0* aq = (vko_block_q8_0*)malloc(sizeof(vko_block_q8_0) * m * nb);
  for (size_t i = 0; i < m; ++i) vko_quantize_row_q8_0(a + i * k, nb, aq + i * nb);
  vko_gemm_q8_0(m, n, k, aq, wq, c);
  free(aq);
}

/* pre-LN -> QKV (+bias) -> 2D RoPE on Q,K (cls at (0,0), so unrotated) ->
 * attention -> out-proj (+bias) * LS1 + residual -> LN -> fc1 (+bias) -> GELU
 * -> fc2 (+bias) * LS2 + residual.  `points` as documented in vk_oracle.h. */
void vko_encoder_layer(float* x, size_t tokens, size_t grid_h, size_t grid_w, size_t embed,
                       size_t heads, size_t ffn, const vko_layer* w, float eps, float rope_freq,
                       int points) {
  const size_t T = tokens, E = embed, F = ffn;
  const int bf16 = points == VKO_POINTS_BF16, q8 = points == VKO_POINTS_Q8_0;
  float* h = (float*)malloc(sizeof(float) * T * E);
  float* q = (float*)malloc(sizeof(float) * T * E);
  float* k = (float*)malloc(sizeof(float) * T * E);
  float* v = (float*)malloc(sizeof(float) * T * E);
  float* att = (float*)malloc(sizeof(float) * T * E);
  float* tok = (float*)malloc(sizeof(float) * T * E);
  float* o = (float*)malloc(sizeof(float) * T * E);
  float* f = (float*)malloc(sizeof(float) * T * F);
  int64_t* pos = (int64_t*)malloc(sizeof(int64_t) * 2 * T);
  /* tokens may span several views of one raster (global cross-view layers,
   * src/specialized.rs:720-757): each view keeps its own RoPE positions and
   * attention runs over all of them */
  const size_t TV = grid_h * grid_w + 1;
  vko_da3_positions(grid_h, grid_w, pos);
  for (size_t t = TV; t < T; ++t) {
    pos[2 * t] = pos[2 * (t % TV)];
    pos[2 * t + 1] = pos[2 * (t % TV) + 1];
  }

  float *wqkv = NULL, *wo = NULL, *w1 = NULL, *w2 = NULL;
  vko_block_q8_0 *qqkv = NULL, *qo = NULL, *q1 = NULL, *q2 = NULL;
  if (q8) {
    qqkv = quantize_weight_q8(w->qkv_w, E, 3 * E);
    qo = quantize_weight_q8(w->proj_w, E, E);
    q1 = quantize_weight_q8(w->fc1_w, E, F);
    q2 = quantize_weight_q8(w->fc2_w, F, E);
  } else {
    wqkv = copy_maybe_bf16(w->qkv_w, E * 3 * E, bf16);
    wo = copy_maybe_bf16(w->proj_w, E * E, bf16);
    w1 = copy_maybe_bf16(w->fc1_w, E * F, bf16);
    w2 = copy_maybe_bf16(w->fc2_w, F * E, bf16);
  }

  memcpy(h, x, sizeof(float) * T * E);
  vko_layernorm(h, T, E, w->ln1_g, w->ln1_b, eps);
  if (bf16) round_bf16_buf(h, T * E);
  if (q8) {
    float* tmp = (float*)malloc(sizeof(float) * T * 3 * E);
    linear_q8(T, 3 * E, E, h, qqkv, tmp);
    for (size_t t = 0; t < T; ++t)
      for (size_t col = 0; col < 3 * E; ++col) {
        const size_t g = col / E, hh = (col % E) / 64, d = col % 64;
        float* dst = g == 0 ? q : (g == 1 ? k : v);
        dst[(hh * T + t) * 64 + d] = tmp[t * 3 * E + col] + w->qkv_b[col];
      }
    free(tmp);
  } else {
    vko_qkv(T, heads, h, wqkv, w->qkv_b, q, k, v);
  }
  if (w->qn_g != NULL) {
    vko_qk_norm_rope(q, k, heads, T, w->qn_g, w->qn_b, w->kn_g, w->kn_b, pos, rope_freq, eps);
  } else {
    vko_rope2d(q, heads, T, 64, pos, rope_freq);
    vko_rope2d(k, heads, T, 64, pos, rope_freq);
  }
  if (bf16 || q8) {
    round_bf16_buf(q, T * E);
    round_bf16_buf(k, T * E);
    round_f16_buf(v, T * E);
  }
  vko_attention_naive(q, k, v, heads, T, 64, att);
  for (size_t hh = 0; hh < heads; ++hh)
    for (size_t t = 0; t < T; ++t)
      for (size_t d = 0; d < 64; ++d) tok[t * E + hh * 64 + d] = att[(hh * T + t) * 64 + d];
  if (bf16) round_bf16_buf(tok, T * E);
  if (q8) {
    linear_q8(T, E, E, tok, qo, o);
    for (size_t i = 0; i < T; ++i)
      for (size_t j = 0; j < E; ++j) o[i * E + j] = (o[i * E + j] + w->proj_b[j]) * w->ls1[j];
  } else {
    vko_linear_bias_scale(T, E, E, tok, wo, w->proj_b, w->ls1, o);
  }
  vko_add(x, o, T * E);

  memcpy(h, x, sizeof(float) * T * E);
  vko_layernorm(h, T, E, w->ln2_g, w->ln2_b, eps);
  if (bf16) round_bf16_buf(h, T * E);
  if (q8)
    linear_q8(T, F, E, h, q1, f);
  else
    gemm_fma_rows(T, F, E, h, w1, f);
  vko_add_bias_rows(f, T, F, w->fc1_b);
  vko_gelu(f, T * F);
  if (bf16) round_bf16_buf(f, T * F);
  if (q8) {
    linear_q8(T, E, F, f, q2, o);
    for (size_t i = 0; i < T; ++i)
      for (size_t j = 0; j < E; ++j) o[i * E + j] = (o[i * E + j] + w->fc2_b[j]) * w->ls2[j];
  } else {
    vko_linear_bias_scale(T, E, F, f, w2, w->fc2_b, w->ls2, o);
  }
  vko_add(x, o, T * E);

  free(wqkv); free(wo); free(w1); free(w2);
  free(qqkv); free(qo); free(q1); free(q2);
  free(h); free(q); free(k); free(v); free(att); free(tok); free(o); free(f); free(pos);
}

/* ------------------------------------------------ DPT head consumers */

/* src/cuda.rs:278-291 vestra_token_to_chw_f32 */
void vko_token_to_chw(const float* token_major, size_t tokens, size_t channels, float* chw) {
  for (size_t t = 0; t < tokens; ++t)
    for (size_t c = 0; c < channels; ++c) chw[c * tokens + t] = token_major[t * channels + c];
}

/* src/resample.rs:82-99 src_coord (half-pixel centres) */
static void hp_coord(size_t dst, float scale, size_t len_in, size_t* i0, size_t* i1, float* frac) {
  const float src = ((float)dst + 0.5f) * scale - 0.5f;
  const float sc = src > 0.0f ? src : 0.0f;
  size_t a = (size_t)floorf(sc);
  const size_t last = len_in > 0 ? len_in - 1 : 0;
  if (a > last) a = last;
  size_t b = a + 1 > last ? last : a + 1;
  float f = b == a ? 0.0f : sc - (float)a;
  f = f < 0.0f ? 0.0f : (f > 1.0f ? 1.0f : f);
  *i0 = a;
  *i1 = b;
  *frac = f;
}

/* src/resample.rs:151-167 src_coord_align_corners (and the identical
 * closure of src/conv.rs:320-336) */
static void ac_coord(size_t dst, size_t len_in, size_t len_out, size_t* i0, size_t* i1, float* frac) {
  if (len_in <= 1) {
    *i0 = 0;
    *i1 = 0;
    *frac = 0.0f;
    return;
  }
  float src = len_out <= 1 ? 0.0f : (float)dst * (float)(len_in - 1) / (float)(len_out - 1);
  const float hi = (float)(len_in - 1);
  src = src < 0.0f ? 0.0f : (src > hi ? hi : src);
  size_t a = (size_t)floorf(src);
  if (a > len_in - 1) a = len_in - 1;
  const size_t b = a + 1 > len_in - 1 ? len_in - 1 : a + 1;
  float f = b == a ? 0.0f : src - (float)a;
  f = f < 0.0f ? 0.0f : (f > 1.0f ? 1.0f : f);
  *i0 = a;
  *i1 = b;
  *frac = f;
}

/* the blend of src/resample.rs:66-71 / 240-245 */
static float blend(const float* plane, size_t iw, size_t y0, size_t y1, float fy, size_t x0, size_t x1, float fx) {
  const float top = plane[y0 * iw + x0] * (1.0f - fx) + plane[y0 * iw + x1] * fx;
  const float bot = plane[y1 * iw + x0] * (1.0f - fx) + plane[y1 * iw + x1] * fx;
  return top * (1.0f - fy) + bot * fy;
}

/* src/resample.rs:10-78 */
void vko_bilinear_resize(const float* input, size_t c, size_t ih, size_t iw, size_t oh, size_t ow, float* out) {
  if (ih == 0 || iw == 0 || oh == 0 || ow == 0) return;
  const float sy = (float)ih / (float)oh, sx = (float)iw / (float)ow;
  for (size_t ch = 0; ch < c; ++ch)
    for (size_t y = 0; y < oh; ++y) {
      size_t y0, y1;
      float fy;
      hp_coord(y, sy, ih, &y0, &y1, &fy);
      for (size_t x = 0; x < ow; ++x) {
        size_t x0, x1;
        float fx;
        hp_coord(x, sx, iw, &x0, &x1, &fx);
        out[(ch * oh + y) * ow + x] = blend(input + ch * ih * iw, iw, y0, y1, fy, x0, x1, fx);
      }
    }
}

/* src/resample.rs:184-249 */
void vko_bilinear_resize_align_corners(const float* input, size_t c, size_t ih, size_t iw, size_t oh, size_t ow,
                                       float* out) {
  if (ih == 0 || iw == 0 || oh == 0 || ow == 0) return;
  for (size_t ch = 0; ch < c; ++ch)
    for (size_t y = 0; y < oh; ++y) {
      size_t y0, y1;
      float fy;
      ac_coord(y, ih, oh, &y0, &y1, &fy);
      for (size_t x = 0; x < ow; ++x) {
        size_t x0, x1;
        float fx;
        ac_coord(x, iw, ow, &x0, &x1, &fx);
        out[(ch * oh + y) * ow + x] = blend(input + ch * ih * iw, iw, y0, y1, fy, x0, x1, fx);
      }
    }
}

/* src/conv.rs:136-160: U = G g G^T per (oc, ic), stored [position][ic][oc] */
void vko_winograd_f2_filter(const float* weight, size_t in_c, size_t out_c, float* u) {
  for (size_t oc = 0; oc < out_c; ++oc)
    for (size_t ic = 0; ic < in_c; ++ic) {
      const float* g = weight + (oc * in_c + ic) * 9;
      float t[4][3], uu[16];
      for (int j = 0; j < 3; ++j) {
        const float a = g[j], b = g[3 + j], c = g[6 + j];
        t[0][j] = a;
        t[1][j] = 0.5f * (a + b + c);
        t[2][j] = 0.5f * (a - b + c);
        t[3][j] = c;
      }
      for (int i = 0; i < 4; ++i) {
        const float a = t[i][0], b = t[i][1], c = t[i][2];
        uu[i * 4] = a;
        uu[i * 4 + 1] = 0.5f * (a + b + c);
        uu[i * 4 + 2] = 0.5f * (a - b + c);
        uu[i * 4 + 3] = c;
      }
      for (int p = 0; p < 16; ++p) u[(p * in_c + ic) * out_c + oc] = uu[p];
    }
}

/* The input transform B^T d B of one 4x4 patch (src/conv.rs:382-405). */
static void winograd_input_tf(const float d[16], float v[16]) {
  float col[16];
  for (int j = 0; j < 4; ++j) {
    const float a = d[j], b = d[4 + j], c = d[8 + j], e = d[12 + j];
    col[j] = a - c;
    col[4 + j] = b + c;
    col[8 + j] = c - b;
    col[12 + j] = b - e;
  }
  for (int i = 0; i < 4; ++i) {
    const float a = col[i * 4], b = col[i * 4 + 1], c = col[i * 4 + 2], e = col[i * 4 + 3];
    v[i * 4] = a - c;
    v[i * 4 + 1] = b + c;
    v[i * 4 + 2] = c - b;
    v[i * 4 + 3] = b - e;
  }
}

/* The transform-domain products and the output transform A^T M A of one
 * tile for every oc (src/conv.rs:407-481): v [16][in_c] of the tile. */
static void winograd_tile_out(const float* v, const float* u, size_t in_c, size_t out_c, const float* bias,
                              size_t ty, size_t tx, size_t oh, size_t ow, float* out) {
  for (size_t oc = 0; oc < out_c; ++oc) {
    float m[16];
    for (int p = 0; p < 16; ++p) {
      float sum = 0.0f;
      for (size_t ic = 0; ic < in_c; ++ic) sum += u[(p * in_c + ic) * out_c + oc] * v[p * in_c + ic];
      m[p] = sum;
    }
    float q[8];
    for (int j = 0; j < 4; ++j) {
      q[j] = m[j] + m[4 + j] + m[8 + j];
      q[4 + j] = m[4 + j] - m[8 + j] - m[12 + j];
    }
    const float b = bias ? bias[oc] : 0.0f;
    const float val[4] = {q[0] + q[1] + q[2] + b, q[1] - q[2] - q[3] + b, q[4] + q[5] + q[6] + b,
                          q[5] - q[6] - q[7] + b};
    for (size_t dy = 0; dy < 2; ++dy)
      for (size_t dx = 0; dx < 2; ++dx) {
        const size_t y = ty * 2 + dy, x = tx * 2 + dx;
        if (y < oh && x < ow) out[(oc * oh + y) * ow + x] = val[dy * 2 + dx];
      }
  }
}

/* src/conv.rs:681-831 */
void vko_conv3x3_winograd_f2(const float* input, size_t in_c, size_t ih, size_t iw, const float* u, size_t out_c,
                             const float* bias, int relu_input, float* out) {
  const size_t tiles_y = (ih + 1) / 2, tiles_x = (iw + 1) / 2;
#pragma omp parallel for schedule(dynamic, 4)
  for (size_t tile = 0; tile < tiles_y * tiles_x; ++tile) {
    const size_t ty = tile / tiles_x, tx = tile % tiles_x;
    float* v = (float*)malloc(sizeof(float) * 16 * in_c);
    for (size_t ic = 0; ic < in_c; ++ic) {
      float d[16], t[16];
      for (int dy = 0; dy < 4; ++dy)
        for (int dx = 0; dx < 4; ++dx) {
          const long sy = (long)(ty * 2) + dy - 1, sx = (long)(tx * 2) + dx - 1;
          float s = (sy >= 0 && sy < (long)ih && sx >= 0 && sx < (long)iw) ? input[(ic * ih + sy) * iw + sx] : 0.0f;
          d[dy * 4 + dx] = relu_input ? (s > 0.0f ? s : 0.0f) : s;
        }
      winograd_input_tf(d, t);
      for (int p = 0; p < 16; ++p) v[p * in_c + ic] = t[p];
    }
    winograd_tile_out(v, u, in_c, out_c, bias, ty, tx, ih, iw, out);
    free(v);
  }
}

/* src/conv.rs:304-484 */
void vko_conv3x3_winograd_f2_resize_ac(const float* input, size_t in_c, size_t ih, size_t iw, size_t oh, size_t ow,
                                       const float* add, const float* u, size_t out_c, const float* bias, float* out) {
  const size_t tiles_y = (oh + 1) / 2, tiles_x = (ow + 1) / 2;
#pragma omp parallel for schedule(dynamic, 4)
  for (size_t tile = 0; tile < tiles_y * tiles_x; ++tile) {
    const size_t ty = tile / tiles_x, tx = tile % tiles_x;
    float* v = (float*)malloc(sizeof(float) * 16 * in_c);
    for (size_t ic = 0; ic < in_c; ++ic) {
      float d[16], t[16];
      for (int dy = 0; dy < 4; ++dy)
        for (int dx = 0; dx < 4; ++dx) {
          const long y = (long)(ty * 2) + dy - 1, x = (long)(tx * 2) + dx - 1;
          float s = 0.0f;
          if (y >= 0 && y < (long)oh && x >= 0 && x < (long)ow) {
            size_t y0, y1, x0, x1;
            float fy, fx;
            ac_coord((size_t)y, ih, oh, &y0, &y1, &fy);
            ac_coord((size_t)x, iw, ow, &x0, &x1, &fx);
            const float* plane = input + ic * ih * iw;
            const float top = plane[y0 * iw + x0] * (1.0f - fx) + plane[y0 * iw + x1] * fx;
            const float bot = plane[y1 * iw + x0] * (1.0f - fx) + plane[y1 * iw + x1] * fx;
            s = top * (1.0f - fy) + bot * fy + (add ? add[(ic * oh + y) * ow + x] : 0.0f);
          }
          d[dy * 4 + dx] = s;
        }
      winograd_input_tf(d, t);
      for (int p = 0; p < 16; ++p) v[p * in_c + ic] = t[p];
    }
    winograd_tile_out(v, u, in_c, out_c, bias, ty, tx, oh, ow, out);
    free(v);
  }
}

/* src/conv.rs:950-1000 */
void vko_conv2d_naive(const float* input, size_t in_c, size_t ih, size_t iw, const float* weight, size_t out_c,
                      size_t kh, size_t kw, size_t stride, size_t pad, const float* bias, float* out) {
  const size_t oh = (ih + 2 * pad - kh) / stride + 1, ow = (iw + 2 * pad - kw) / stride + 1;
  for (size_t oc = 0; oc < out_c; ++oc)
    for (size_t y = 0; y < oh; ++y)
      for (size_t x = 0; x < ow; ++x) {
        float acc = 0.0f;
        for (size_t ic = 0; ic < in_c; ++ic)
          for (size_t ky = 0; ky < kh; ++ky) {
            const long iy = (long)(y * stride + ky) - (long)pad;
            if (iy < 0 || iy >= (long)ih) continue;
            for (size_t kx = 0; kx < kw; ++kx) {
              const long ix = (long)(x * stride + kx) - (long)pad;
              if (ix < 0 || ix >= (long)iw) continue;
              acc += input[(ic * ih + iy) * iw + ix] * weight[((oc * in_c + ic) * kh + ky) * kw + kx];
            }
          }
        if (bias) acc += bias[oc];
        out[(oc * oh + y) * ow + x] = acc;
      }
}
