/*
 * vk_oracle.h -- CPU restatement of the vestra-kernels reference arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * B200 kernels: only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs may load it.  The product path
 * (vestra-kernels_b200/) never links or calls it.
 *
 * Every function restates one reference function; the citation beside each
 * declaration is the reference file:line it follows (paths are relative to
 * the vestra-kernels crate root).  Evaluation order, rounding points and
 * constants follow the reference so that outputs are bit-identical to the
 * reference's scalar path on the same inputs (the reference crate cannot be
 * built here: no Rust toolchain, and its registry dependencies are not
 * vendored; see the "parity pin" notes in the test files).
 */
#ifndef VK_ORACLE_H
#define VK_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VKO_QK8_0 32

/* BlockQ8_0 {d: f16, qs: [i8;32]}, #[repr(C)], 34 bytes (src/lib.rs:33-38). */
typedef struct __attribute__((packed)) {
  uint16_t d;
  int8_t qs[VKO_QK8_0];
} vko_block_q8_0;

/* IEEE binary16 round-to-nearest-even, as half::f16::from_f32 (half 2.7.1). */
uint16_t vko_f16_from_f32(float x);
float vko_f16_to_f32(uint16_t h);
/* bfloat16 round-to-nearest-even (the rounding the B200 kernels apply). */
float vko_round_bf16(float x);

/* src/scalar.rs:3-18 */
void vko_gemm_f32(size_t m, size_t n, size_t k, const float* a, const float* b, float* c);
/* src/scalar.rs:25-56 */
void vko_gemm_q8_0(size_t m, size_t n, size_t k, const vko_block_q8_0* a_q,
                   const vko_block_q8_0* b_q, float* c);
/* The int32 block dot of src/scalar.rs:47-50, exposed so the int32 sums can
 * be checked bit for bit: out[(i*n+j)*nb + b] = sum_l qa*qb. */
void vko_q8_0_block_dots(size_t m, size_t n, size_t k, const vko_block_q8_0* a_q,
                         const vko_block_q8_0* b_q, int32_t* out);
/* src/lib.rs:42-50 */
void vko_dequantize_q8_0(const vko_block_q8_0* blocks, size_t nblocks, float* out);
/* src/q8_0_dot.rs:27-46 */
void vko_quantize_row_q8_0(const float* x, size_t nblocks, vko_block_q8_0* out);

/* src/scalar.rs:58-63 */
void vko_add(float* dst, const float* src, size_t n);
/* src/scalar.rs:65-81 */
void vko_add_bias_rows(float* x, size_t rows, size_t cols, const float* bias);
/* src/scalar.rs:83-114 */
void vko_layernorm(float* x, size_t rows, size_t cols, const float* gamma, const float* beta,
                   float eps);
/* src/scalar.rs:116-134 */
void vko_gelu(float* x, size_t n);
float vko_erf(float x);
/* src/scalar.rs:139-155 */
void vko_layerscale(float* x, size_t rows, size_t cols, const float* gamma);
/* src/scalar.rs:157-172 */
void vko_softmax_rows(float* x, size_t rows, size_t cols);

/* src/attention.rs:10-59 */
void vko_attention_naive(const float* q, const float* k, const float* v, size_t heads, size_t n,
                         size_t head_dim, float* out);
/* src/attention.rs:66-201, scalar route (use_avx512 == false, as attention_serial) */
void vko_attention(const float* q, const float* k, const float* v, size_t heads, size_t n,
                   size_t head_dim, float* out);

/* src/rope.rs:30-93 */
void vko_rope2d(float* x, size_t heads, size_t n, size_t head_dim, const int64_t* pos_yx,
                float freq);
/* src/specialized.rs:389-410: rotations[(t*2*16 + axis*16 + i)*2 + {0:sin,1:cos}] */
void vko_rope_rotations(const int64_t* pos_yx, size_t tokens, float freq, float* rotations);
/* src/specialized.rs:278-318, 412-454 (generalised over token count) */
void vko_qk_norm_rope(float* q, float* k, size_t heads, size_t tokens, const float* q_gamma,
                      const float* q_beta, const float* k_gamma, const float* k_beta,
                      const int64_t* pos_yx, float freq, float eps);
/* DA3 position layout, src/specialized.rs:359-366 generalised to a grid of
 * width grid_w: cls token (0,0), patch p -> (p / grid_w + 1, p % grid_w + 1). */
void vko_da3_positions(size_t grid_h, size_t grid_w, int64_t* pos_yx);

/* src/specialized.rs:996-1167: q/k/v[h,t,:] = x[t,:] . W[:, g*768 + h*64 ..] + b,
 * generalised to `tokens` rows and `heads` x 64 columns per group. */
void vko_qkv(size_t tokens, size_t heads, const float* x, const float* w, const float* bias,
             float* q, float* k, float* v);
/* src/specialized.rs:811-991: c = (a.b + bias) * scale */
void vko_linear_bias_scale(size_t m, size_t n, size_t k, const float* a, const float* b,
                           const float* bias, const float* scale, float* c);

/* One DA3-BASE ViT block composed from the restated operators (the engine's
 * composition, which is not in the reference crate).  `points` selects the
 * arithmetic at the points where the B200 kernels store narrow types:
 *   VKO_POINTS_F32   all f32;
 *   VKO_POINTS_BF16  the inputs of every matrix product and the stored
 *                    activations rounded to bf16 (v to f16, the type of the
 *                    attention P V product);
 *   VKO_POINTS_Q8_0  projections through gemm_q8_0 on Q8_0 weights and
 *                    Q8_0-quantised activations (src/scalar.rs:25-56,
 *                    src/q8_0_dot.rs:27-46); q, k bf16 and v f16. */
#define VKO_POINTS_F32 0
#define VKO_POINTS_BF16 1
#define VKO_POINTS_Q8_0 2
typedef struct {
  const float *ln1_g, *ln1_b;
  const float *qkv_w, *qkv_b;   /* [E, 3E], [3E] */
  const float *proj_w, *proj_b; /* [E, E], [E] */
  const float* ls1;             /* [E] */
  const float *ln2_g, *ln2_b;
  const float *fc1_w, *fc1_b;   /* [E, F], [F] */
  const float *fc2_w, *fc2_b;   /* [F, E], [E] */
  const float* ls2;             /* [E] */
  /* optional Q/K LayerNorm before RoPE (qk_norm_rope_f32_da3_base,
   * src/specialized.rs:278-454): [64] each, or all NULL */
  const float *qn_g, *qn_b, *kn_g, *kn_b;
} vko_layer;

/* tokens = views * (grid_h * grid_w + 1): with views > 1 the block attends
 * across all views (a global cross-view layer); RoPE positions repeat per
 * view. */
void vko_encoder_layer(float* x, size_t tokens, size_t grid_h, size_t grid_w, size_t embed,
                       size_t heads, size_t ffn, const vko_layer* w, float eps, float rope_freq,
                       int points);

/* src/cuda.rs:295-316 vestra_patchify_nchw_f32: image [channels, height,
 * width] -> patches [(height/patch)(width/patch), channels * patch^2], each
 * row in (channel, patch_y, patch_x) order.  Returns 0, or -1 on an invalid
 * shape (src/cuda.rs:1081-1093). */
int vko_patchify_nchw(const float* image, size_t height, size_t width, size_t patch, size_t channels,
                      float* patches);
/* src/cuda.rs:321-334 vestra_prepend_cls_add_pos_f32: tokens [patch_count + 1,
 * embed] = [cls; patches] + position. */
void vko_prepend_cls_add_pos(const float* patches, const float* cls, const float* position, size_t patch_count,
                             size_t embed, float* tokens);

/* ---- DPT head consumers: the step after the encoder ---- */
/* src/cuda.rs:278-291 vestra_token_to_chw_f32: token-major [tokens,
 * channels] -> CHW [channels, tokens]. */
void vko_token_to_chw(const float* token_major, size_t tokens, size_t channels, float* chw);
/* src/resample.rs:10-99 bilinear_resize: half-pixel centres, clamp to edge;
 * input [c, ih, iw] -> out [c, oh, ow]; any zero size leaves out untouched. */
void vko_bilinear_resize(const float* input, size_t c, size_t ih, size_t iw, size_t oh, size_t ow, float* out);
/* src/resample.rs:151-249 bilinear_resize_align_corners. */
void vko_bilinear_resize_align_corners(const float* input, size_t c, size_t ih, size_t iw, size_t oh, size_t ow,
                                       float* out);
/* src/conv.rs:121-171 transformed_winograd_filter: OIHW [out_c, in_c, 3, 3]
 * -> U [16][in_c][out_c] (F(2x2, 3x3), G g G^T). */
void vko_winograd_f2_filter(const float* weight, size_t in_c, size_t out_c, float* u);
/* src/conv.rs:681-831 conv3x3_winograd_f2_impl: stride 1, pad 1, output
 * [out_c, ih, iw]; relu_input applies max(x, 0) to every loaded sample;
 * bias may be NULL.  The transform-domain sums run over ascending ic with
 * separately rounded products, as the scalar fallback. */
void vko_conv3x3_winograd_f2(const float* input, size_t in_c, size_t ih, size_t iw, const float* u, size_t out_c,
                             const float* bias, int relu_input, float* out);
/* src/conv.rs:304-484 conv3x3_winograd_f2_prepared_resize_align_corners: the
 * input is resized (align corners) to [in_c, oh, ow], plus `add` (NULL or
 * [in_c, oh, ow]), then convolved; output [out_c, oh, ow]. */
void vko_conv3x3_winograd_f2_resize_ac(const float* input, size_t in_c, size_t ih, size_t iw, size_t oh, size_t ow,
                                       const float* add, const float* u, size_t out_c, const float* bias, float* out);
/* src/conv.rs:950-1000 conv2d_naive: direct convolution, OIHW weights. */
void vko_conv2d_naive(const float* input, size_t in_c, size_t ih, size_t iw, const float* weight, size_t out_c,
                      size_t kh, size_t kw, size_t stride, size_t pad, const float* bias, float* out);

/* Threads used by the parallel loops (rows are independent and each keeps
 * the scalar reduction order, so results do not depend on this). */
void vko_set_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
