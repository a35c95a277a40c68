/*
 * vestra_b200.h -- C ABI of the B200 (sm_100a) DA3-BASE encoder hot path.
 *
 * Drop-in for the primitive-buffer API of the vestra-kernels crate
 * (API.md:1-16, src/lib.rs:1-132).  Conventions:
 *  - every entry point returns an int status; VK_UNSUPPORTED_SHAPE plays the
 *    role of the reference's `false` ("shape unsupported, use your
 *    fallback") and leaves outputs untouched; vk_last_error() describes the
 *    last failure of the calling thread;
 *  - buffers are caller-owned plain pointers with explicit dimensions;
 *    "dev" pointers are device memory of the context's GPU, "host" pointers
 *    host memory (pageable or pinned);
 *  - operations are enqueued on the context's stream (vk_stream_set) and
 *    are asynchronous; vk_synchronize() waits and reports device-side
 *    timeouts (VK_ERR_TIMEOUT);
 *  - one context per GPU; a context is not shared between threads without
 *    external synchronisation;
 *  - weights use the reference layout: [K, N] row-major, input-major
 *    (src/specialized.rs:1058, b[kk * n + col]).
 * Nothing in this header uses C++ or CUDA types.
 */
#ifndef VESTRA_B200_H
#define VESTRA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VK_OK 0
#define VK_UNSUPPORTED_SHAPE 1
#define VK_ERR_INVALID_ARGUMENT 2
#define VK_ERR_CUDA 3
#define VK_ERR_TIMEOUT 4
#define VK_ERR_NO_DEVICE 5
#define VK_ERR_OUT_OF_MEMORY 6

/* Arithmetic of the f32-interface operators and of an encoder. */
#define VK_MATH_F32 0  /* f32 in, f32 arithmetic (CUDA cores), f32 out      */
#define VK_MATH_BF16 1 /* bf16 tensor-core products, f32 accumulation        */
#define VK_MATH_Q8_0 2 /* Q8_0 weights and activations, int8 tensor cores   */

typedef struct vk_ctx vk_ctx;
typedef struct vk_linear vk_linear;
typedef struct vk_encoder vk_encoder;

/* 34-byte Q8_0 record, identical to BlockQ8_0 {d: f16, qs: [i8; 32]}
 * (#[repr(C)], src/lib.rs:33-38). */
#define VK_QK8_0 32
typedef struct {
  uint16_t d;
  int8_t qs[VK_QK8_0];
} vk_block_q8_0;

/* ---------------------------------------------------------------- lifecycle */
/* Context on CUDA device `device` (one per GPU).  Replaces CudaRuntime::new
 * (src/cuda.rs:383-443). */
int vk_init(int device, vk_ctx** out);
int vk_destroy(vk_ctx* ctx);
/* Use this cudaStream_t for later calls (NULL = the context's own stream,
 * a non-blocking stream created by vk_init). */
int vk_stream_set(vk_ctx* ctx, void* stream);
/* Arithmetic of the f32-interface operators below (default VK_MATH_F32). */
int vk_set_math(vk_ctx* ctx, int math);
/* Waits for the context's stream; VK_ERR_TIMEOUT if a kernel gave up a wait. */
int vk_synchronize(vk_ctx* ctx);
const char* vk_last_error(void);
const char* vk_version(void);

/* ------------------------------------------- DA3-BASE specialised operators
 * Device pointers.  These replace the five `*_da3_base` functions of
 * src/lib.rs.  The reference gates them to 865 tokens; here any token count
 * >= 1 is accepted (the 3457-token configuration included).  Like the
 * reference's functions they take the f32 weight on every call; under
 * VK_MATH_BF16 / VK_MATH_Q8_0 that means a conversion of the weight per call.
 * A caller that runs the same weight repeatedly prepares it once with
 * vk_prepare_linear and calls vk_linear_run (the reference's prepared-value
 * route, CudaLinearF32), which converts nothing per call. */

/* src/lib.rs:52 qkv_f32_da3_base: input [tokens, 768], weight [768, 2304],
 * bias [2304] -> q, k, v [12, tokens, 64] head-major (bias added, no RoPE). */
int vk_qkv_f32_da3_base(vk_ctx* ctx, size_t tokens, const float* input, const float* weight,
                        const float* bias, float* q, float* k, float* v);

/* src/lib.rs:67 linear_f32_da3_base: output[m, n] = input[m, k] . weight[k, n].
 * (k, n) must be a DA3-BASE projection: (768, 2304), (768, 768), (768, 3072)
 * or (3072, 768). */
int vk_linear_f32_da3_base(vk_ctx* ctx, size_t m, size_t n, size_t k, const float* input,
                           const float* weight, float* output);

/* src/lib.rs:94 linear_bias_scale_f32_da3_base: c = (a . b + bias) * scale,
 * (k, n) in {(768, 768), (3072, 768)}. */
int vk_linear_bias_scale_f32_da3_base(vk_ctx* ctx, size_t m, size_t n, size_t k, const float* a,
                                      const float* b, const float* bias, const float* scale,
                                      float* c);

/* src/lib.rs:82 flash_attention_f32_da3_base: q, k, v, out [heads, tokens, 64]. */
int vk_flash_attention_f32_da3_base(vk_ctx* ctx, const float* query, const float* key,
                                    const float* value, size_t heads, size_t tokens,
                                    float* output);

/* src/lib.rs:108 qk_norm_rope_f32_da3_base: in place on q, k [heads, tokens, 64];
 * gamma/beta [64]; positions_yx int64 [tokens, 2] (device). */
int vk_qk_norm_rope_f32_da3_base(vk_ctx* ctx, float* q, float* k, size_t heads, size_t tokens,
                                 const float* q_gamma, const float* q_beta, const float* k_gamma,
                                 const float* k_beta, const int64_t* positions_yx,
                                 float frequency, float epsilon);

/* ------------------------------------------------------ generic operators */
/* src/attention.rs:66 attention: q, k, v, out [heads, n, head_dim]; head_dim
 * in {8, 16, 32, 64} (64 follows vk_set_math, others are f32). */
int vk_attention(vk_ctx* ctx, const float* q, const float* k, const float* v, size_t heads,
                 size_t n, size_t head_dim, float* out);
/* src/rope.rs:30 rope2d, in place on x [heads, n, head_dim], head_dim % 4 == 0,
 * pos_yx int64 [n, 2] (device). */
int vk_rope2d(vk_ctx* ctx, float* x, size_t heads, size_t n, size_t head_dim,
              const int64_t* pos_yx, float freq);
/* src/scalar.rs:83 layernorm, in place on x [rows, cols]. */
int vk_layernorm(vk_ctx* ctx, float* x, size_t rows, size_t cols, const float* gamma,
                 const float* beta, float eps);
/* src/dispatch.rs:56 Kernels::gelu (exact-erf GELU, A&S 7.1.26), in place. */
int vk_gelu(vk_ctx* ctx, float* x, size_t n);
/* src/dispatch.rs:77 Kernels::add: dst += src. */
int vk_add(vk_ctx* ctx, float* dst, const float* src, size_t n);
/* src/scalar.rs:65 add_bias_rows, src/scalar.rs:139 layerscale. */
int vk_add_bias_rows(vk_ctx* ctx, float* x, size_t rows, size_t cols, const float* bias);
int vk_layerscale(vk_ctx* ctx, float* x, size_t rows, size_t cols, const float* gamma);
/* src/q8_0_dot.rs:27 quantize_row_q8_0: x [nblocks * 32] -> out [nblocks]. */
int vk_quantize_row_q8_0(vk_ctx* ctx, const float* x, size_t nblocks, vk_block_q8_0* out);
/* src/dispatch.rs:91 Kernels::gemm_q8_0: a_q [m, k/32], b_q [n, k/32]
 * (B pre-transposed, as in the reference), c [m, n] f32.  k % 128 == 0,
 * n % 128 == 0. */
int vk_gemm_q8_0(vk_ctx* ctx, size_t m, size_t n, size_t k, const vk_block_q8_0* a_q,
                 const vk_block_q8_0* b_q, float* c);
/* The int32 block dot products of the same kernel, out [m, n, k/32]
 * (src/scalar.rs:47-50), for bit-exact verification. */
int vk_gemm_q8_0_block_dots(vk_ctx* ctx, size_t m, size_t n, size_t k,
                            const vk_block_q8_0* a_q, const vk_block_q8_0* b_q, int32_t* dots);

/* vk_gemm_q8_0 for callers that cannot allocate device memory (hosts whose
 * device memory is budgeted up front, plugins inside an engine that owns
 * every allocation).  It has no counterpart in the reference.  It takes no
 * context and unpacks the blocks into a fixed 8 MiB array inside the library
 * instead of a cudaMalloc'd workspace: (m + n) * k + (m + n) * (k / 32) * 2
 * bytes must fit (VK_UNSUPPORTED_SHAPE otherwise).  The first call on a
 * device loads the module and should come before any stream capture; calls
 * that overlap on the GPU share the array and race.  `stream` is a
 * cudaStream_t of the current device (NULL = legacy default stream;
 * another device's stream is VK_ERR_INVALID_ARGUMENT); a_q, b_q, c as in
 * vk_gemm_q8_0.  Device-side wait timeouts are not reported (there is no
 * context to carry them): c may then be partly written. */
int vk_gemm_q8_0_noalloc(void* stream, size_t m, size_t n, size_t k, const vk_block_q8_0* a_q,
                         const vk_block_q8_0* b_q, float* c);

/* ------------------------------------------------- patch embedding
 * The step before the encoder.  src/cuda.rs:295-316 vestra_patchify_nchw_f32
 * / CudaRuntime::patchify_nchw_f32 (src/cuda.rs:1073): image [channels,
 * height, width] (device) -> patches [(height/patch) * (width/patch),
 * channels * patch * patch], each row in (channel, patch_y, patch_x) order.
 * Invalid shapes (zero sizes, height or width not a multiple of patch) are
 * VK_ERR_INVALID_ARGUMENT, as the reference's CudaError::Kernel. */
int vk_patchify_nchw_f32(vk_ctx* ctx, const float* image, size_t height, size_t width, size_t patch,
                         size_t channels, float* patches);
/* src/cuda.rs:321-334 vestra_prepend_cls_add_pos_f32 /
 * CudaRuntime::prepend_cls_add_pos_f32 (src/cuda.rs:1130): tokens
 * [patch_count + 1, embed] = [cls; patches] + position (device). */
int vk_prepend_cls_add_pos_f32(vk_ctx* ctx, const float* patches, const float* cls, const float* position,
                               size_t patch_count, size_t embed, float* tokens);

/* Batched patch embedding as one call: tokens[b] = [cls; patchify(image[b])
 * . weight + bias] + position.  weight_host [channels * patch * patch, embed]
 * (the OIHW convolution weight flattened input-major), bias / cls [embed]
 * (host); math VK_MATH_F32 (FMA projection, bit-exact with the f32
 * operators) or VK_MATH_BF16 (tensor cores; embed % 128 == 0). */
typedef struct vk_patch_embed vk_patch_embed;
int vk_patch_embed_prepare(vk_ctx* ctx, size_t channels, size_t patch, size_t embed, const float* weight_host,
                           const float* bias_host, const float* cls_host, int math, vk_patch_embed** out);
/* images_dev [images, channels, height, width]; position_dev [tokens, embed]
 * with tokens = (height/patch) * (width/patch) + 1; tokens_dev [images,
 * tokens, embed] (position and tokens 16-byte aligned). */
int vk_patch_embed_forward(vk_ctx* ctx, const vk_patch_embed* pe, size_t images, size_t height, size_t width,
                           const float* images_dev, const float* position_dev, float* tokens_dev);
int vk_patch_embed_release(vk_patch_embed* pe);

/* --------------------------------------------------------- prepared values
 * Mirrors the prepared-value objects of the reference (CudaLinearF32,
 * src/cuda.rs:1233-1334): weights are converted and laid out once. */
/* weight_host [k, n] f32, bias_host / scale_host [n] or NULL; math selects
 * the stored form (f32, bf16, or Q8_0 quantised per 32 along k). */
int vk_prepare_linear(vk_ctx* ctx, size_t k, size_t n, const float* weight_host,
                      const float* bias_host, const float* scale_host, int math,
                      vk_linear** out);
/* Q8_0 weights given as blocks [n, k/32] (host). */
int vk_prepare_linear_q8_0(vk_ctx* ctx, size_t k, size_t n, const vk_block_q8_0* blocks_host,
                           const float* bias_host, const float* scale_host, vk_linear** out);
/* output[m, n] = (input[m, k] . W + bias) * scale, device pointers. */
int vk_linear_run(vk_ctx* ctx, const vk_linear* lin, size_t m, const float* input, float* output);
int vk_release_linear(vk_linear* lin);

/* ------------------------------------------------------------- encoder
 * DA3-BASE ViT encoder: pre-LN -> QKV -> 2D RoPE on Q, K (cls unrotated) ->
 * attention -> out-proj + LayerScale + residual -> LN -> fc1 + GELU -> fc2 +
 * LayerScale + residual, for `layers` blocks (the composition the engine
 * performs with the operators above). */
typedef struct {
  const float *ln1_gamma, *ln1_beta;     /* [E]            */
  const float *qkv_weight, *qkv_bias;    /* [E, 3E], [3E]  */
  const float *proj_weight, *proj_bias;  /* [E, E], [E]    */
  const float* ls1;                      /* [E]            */
  const float *ln2_gamma, *ln2_beta;     /* [E]            */
  const float *fc1_weight, *fc1_bias;    /* [E, F], [F]    */
  const float *fc2_weight, *fc2_bias;    /* [F, E], [E]    */
  const float* ls2;                      /* [E]            */
  /* Optional Q/K LayerNorm before RoPE (DA3's late blocks;
   * qk_norm_rope_f32_da3_base, src/specialized.rs:278-454): [64] each, all
   * four set or all NULL; eps = the encoder's eps.  bf16 and f32 math. */
  const float *q_norm_gamma, *q_norm_beta, *k_norm_gamma, *k_norm_beta;
} vk_layer_weights;

typedef struct {
  int layers;      /* 12 for DA3-BASE                */
  int heads;       /* 12; embed = heads * 64         */
  int ffn;         /* 3072                           */
  float eps;       /* LayerNorm epsilon, 1e-6        */
  float rope_freq; /* 100                            */
  int math;        /* VK_MATH_BF16, VK_MATH_Q8_0 or VK_MATH_F32 */
  /* Multi-view inputs (global cross-view layers, the reference's flash
   * attention over views * tokens, src/specialized.rs:720-757): bit l of
   * global_layers makes layer l attend across each group of `views`
   * consecutive images (one sequence of views * tokens; RoPE positions repeat
   * per view).  views <= 1 or global_layers == 0: every layer attends within
   * its image.  With global layers, `images` must be a multiple of views. */
  int views;
  uint64_t global_layers;
} vk_encoder_config;

/* layers_host[cfg->layers], host f32 in the reference layout. */
int vk_encoder_prepare(vk_ctx* ctx, const vk_encoder_config* cfg,
                       const vk_layer_weights* layers_host, vk_encoder** out);
/* tokens / out: [images, 1 + grid_h * grid_w, E] f32, device pointers (may
 * alias).  Token 0 of each image is the cls token at RoPE position (0, 0);
 * patch p sits at (p / grid_w + 1, p % grid_w + 1). */
int vk_encoder_forward(vk_ctx* ctx, vk_encoder* enc, size_t images, size_t grid_h, size_t grid_w,
                       const float* tokens_dev, float* out_dev);
/* Same with host buffers: the copies in and out are pipelined with the
 * compute in image chunks (the end-to-end entry point). */
int vk_encoder_forward_host(vk_ctx* ctx, vk_encoder* enc, size_t images, size_t grid_h,
                            size_t grid_w, const float* tokens_host, float* out_host);
/* As vk_encoder_forward_host but returns once the work is enqueued: the
 * result is in out_host after vk_synchronize(ctx) (or any later work on the
 * context stream).  Back-to-back calls overlap one call's copies with the
 * neighbouring calls' compute.  Both host buffers must stay valid and
 * tokens_host unmodified until then; pinned host memory is needed for the
 * copies to overlap.  Work enqueued on the context stream before the call is
 * not waited for (vk_synchronize first if it must be). */
int vk_encoder_forward_host_async(vk_ctx* ctx, vk_encoder* enc, size_t images, size_t grid_h,
                                  size_t grid_w, const float* tokens_host, float* out_host);
/* One eager forward with CUDA events between kernels: ms_per_slot[i] sums
 * the device time of the i-th kernel of every block (slots >= 7 for bf16 /
 * Q8_0, >= 10 for f32; order as in the block description above). */
int vk_encoder_profile(vk_ctx* ctx, vk_encoder* enc, size_t images, size_t grid_h, size_t grid_w,
                       const float* tokens_dev, float* out_dev, float* ms_per_slot, int slots);
/* Kernels launched by the last vk_encoder_forward (for accounting). */
int vk_encoder_last_launches(const vk_encoder* enc);
int vk_encoder_release(vk_encoder* enc);

/* ------------------------------------------------- DPT head consumers
 * The step after the encoder: token-major features to CHW maps, bilinear
 * resizes and the 3x3 convolutions of the DPT head, all f32 on device
 * buffers, batch 1 as the reference (plus batched conveniences). */

/* src/cuda.rs:278-291 vestra_token_to_chw_f32 / CudaRuntime::token_to_chw_f32
 * (src/cuda.rs:1032-1068): token_major [tokens, channels] -> chw [channels,
 * tokens].  tokens or channels == 0 is VK_ERR_INVALID_ARGUMENT, as the
 * reference's CudaError::LengthMismatch. */
int vk_token_to_chw_f32(vk_ctx* ctx, const float* token_major, size_t tokens, size_t channels, float* chw);
/* `images` [tokens, channels] matrices back to back -> `images` CHW maps. */
int vk_token_to_chw_f32_batched(vk_ctx* ctx, const float* token_major, size_t images, size_t tokens,
                                size_t channels, float* chw);
/* src/resample.rs:10-78 bilinear_resize (half-pixel centres, clamp to edge):
 * input [c, ih, iw] -> out [c, oh, ow].  Any zero size is a no-op, as the
 * reference's early return.  Bit-exact with the reference's f32 arithmetic. */
int vk_bilinear_resize_f32(vk_ctx* ctx, const float* input, size_t c, size_t ih, size_t iw, size_t oh, size_t ow,
                           float* out);
/* src/resample.rs:184-249 bilinear_resize_align_corners; as above. */
int vk_bilinear_resize_align_corners_f32(vk_ctx* ctx, const float* input, size_t c, size_t ih, size_t iw, size_t oh,
                                         size_t ow, float* out);

/* A prepared 3x3 convolution filter: WinogradF2Filter
 * (prepare_winograd_f2_filter, src/conv.rs:175-178; the transform of
 * src/conv.rs:136-160) held on the device as U [16][in_c][out_c]. */
typedef struct vk_conv3x3 vk_conv3x3;
/* weight_host: OIHW [out_c, in_c, 3, 3] f32. */
int vk_conv3x3_prepare(vk_ctx* ctx, const float* weight_host, size_t in_c, size_t out_c, vk_conv3x3** out);
/* As vk_conv3x3_prepare with a math mode: VK_MATH_F32 (the reference's
 * Winograd F(2x2, 3x3) arithmetic) or VK_MATH_BF16 -- the convolution as an
 * implicit GEMM on the tensor cores over bf16 inputs and weights with f32
 * accumulation (1e-2 relative L2 bar, the precision class of the encoder's
 * bf16 math).  bf16 math uses the context's workspace for a channels-last
 * copy of the input (images * h * w * in_c rounded up to 64, bf16). */
int vk_conv3x3_prepare_math(vk_ctx* ctx, const float* weight_host, size_t in_c, size_t out_c, int math,
                            vk_conv3x3** out);
/* conv3x3_winograd_f2_prepared / _prepared_relu_input (src/conv.rs:282-302,
 * 667-679): stride 1, pad 1, input [in_c, ih, iw] -> out [out_c, ih, iw];
 * bias [out_c] or NULL (device); relu_input != 0 applies max(x, 0) to every
 * input sample.  in_c / out_c must match the filter (VK_ERR_INVALID_ARGUMENT).
 * The transforms follow the reference's F(2x2, 3x3) arithmetic; the
 * transform-domain sums run over ascending in_c with fused multiply-adds. */
int vk_conv3x3_forward(vk_ctx* ctx, const vk_conv3x3* conv, const float* input, size_t in_c, size_t ih, size_t iw,
                       size_t out_c, const float* bias, int relu_input, float* out);
/* conv3x3_winograd_f2_prepared_resize_align_corners (src/conv.rs:304-484):
 * input [in_c, ih, iw] resized (align corners) to [in_c, oh, ow], plus `add`
 * ([in_c, oh, ow] or NULL), then convolved -> out [out_c, oh, ow].  Equal
 * bit for bit to vk_bilinear_resize_align_corners_f32, the add, and
 * vk_conv3x3_forward in sequence (which is how it runs: the resized map,
 * images * in_c * oh * ow floats, lives in the context's workspace). */
int vk_conv3x3_resize_ac_forward(vk_ctx* ctx, const vk_conv3x3* conv, const float* input, size_t in_c, size_t ih,
                                 size_t iw, size_t oh, size_t ow, const float* add, size_t out_c, const float* bias,
                                 float* out);
/* Batched forms: `images` inputs / outputs back to back; `add` is shared by
 * all images (the DPT UV embedding depends on the size only). */
int vk_conv3x3_forward_batched(vk_ctx* ctx, const vk_conv3x3* conv, size_t images, const float* input, size_t ih,
                               size_t iw, const float* bias, int relu_input, float* out);
int vk_conv3x3_resize_ac_forward_batched(vk_ctx* ctx, const vk_conv3x3* conv, size_t images, const float* input,
                                         size_t ih, size_t iw, size_t oh, size_t ow, const float* add,
                                         const float* bias, float* out);
int vk_conv3x3_release(vk_conv3x3* conv);

#ifdef __cplusplus
}
#endif
#endif
