/*
 * vk_cpu_ref.h -- the reference's timed CPU fast path, restated in C with
 * AVX-512 intrinsics and OpenMP (in place of rayon).
 *
 * TEST / BENCHMARK INFRASTRUCTURE ONLY: bench.py times it as the CPU
 * baseline ("port" of the reference's AVX-512 path); the product never links
 * it.  Each function cites the reference code it restates.
 */
#ifndef VK_CPU_REF_H
#define VK_CPU_REF_H

#include <stddef.h>
#include <stdint.h>

#include "vk_oracle.h"

#ifdef __cplusplus
extern "C" {
#endif

/* src/specialized.rs:1101-1167 qkv_avx512_column_split (any token count). */
void vkr_qkv(size_t tokens, const float* x, const float* w, const float* bias, float* q, float* k,
             float* v);
/* src/specialized.rs:1171-1300 linear_avx512_column_split. */
void vkr_linear(size_t m, size_t n, size_t k, const float* a, const float* b, float* c);
/* src/specialized.rs:836-878 linear_bias_scale_avx512_rows::<6>. */
void vkr_linear_bias_scale(size_t m, size_t n, size_t k, const float* a, const float* b,
                           const float* bias, const float* scale, float* c);
/* src/specialized.rs:1906-2258 + 1400-1562 flash_attention_avx512 (QT8 tiles,
 * 64-key panels, Cephes exp), head_dim 64. */
void vkr_flash_attention(const float* q, const float* k, const float* v, size_t heads,
                         size_t tokens, float* out);
/* src/simd_avx512.rs:183-209 gelu_avx512 (parallel 4096-element chunks,
 * src/dispatch.rs:68-69). */
void vkr_gelu(float* x, size_t n);
/* src/simd_avx512.rs:215-235 add_avx512. */
void vkr_add(float* dst, const float* src, size_t n);

/* One DA3-BASE block on the fast path, as the engine composes it. */
void vkr_encoder_layer(float* x, size_t tokens, size_t grid_h, size_t grid_w, const vko_layer* w,
                       float eps, float rope_freq);

#ifdef __cplusplus
}
#endif
#endif
