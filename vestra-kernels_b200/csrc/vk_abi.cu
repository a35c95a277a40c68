// vk_abi.cu -- the C ABI (include/vestra_b200.h): contexts, the operator
// entry points of the reference's public API, prepared linears.  The encoder
// driver lives in vk_encoder.cu.
#include <cstring>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <string>
#include <vector>

#include "vestra_b200.h"
#include "vk_abi_internal.h"
#include "vk_internal.h"

using namespace vk;

// ------------------------------------------------------------------ errors
static thread_local std::string g_last_error;

int vk_fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int vk_cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return VK_OK;
  if (e == cudaErrorMemoryAllocation) return vk_fail(VK_ERR_OUT_OF_MEMORY, "%s: %s", what, cudaGetErrorString(e));
  return vk_fail(VK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

extern "C" const char* vk_last_error(void) { return g_last_error.c_str(); }
extern "C" const char* vk_version(void) { return "vestra-b200 0.1.0 (sm_100a)"; }

// ------------------------------------------------------------------ context
int ctx_reserve(vk_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->ws_bytes) return VK_OK;
  cudaError_t e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return vk_cuda_status(e, "workspace sync");
  if (ctx->ws) cudaFree(ctx->ws);
  ctx->ws = nullptr;
  ctx->ws_bytes = 0;
  size_t want = bytes + (bytes >> 2);
  e = cudaMalloc(&ctx->ws, want);
  if (e != cudaSuccess) return vk_cuda_status(e, "workspace allocation");
  ctx->ws_bytes = want;
  return VK_OK;
}

extern "C" int vk_init(int device, vk_ctx** out) {
  if (out == nullptr) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_init: out is NULL");
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return vk_fail(VK_ERR_NO_DEVICE, "vk_init: no CUDA device");
  if (device < 0 || device >= n) return vk_fail(VK_ERR_NO_DEVICE, "vk_init: device %d of %d", device, n);
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return vk_cuda_status(e, "cudaSetDevice");
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return vk_cuda_status(e, "cudaGetDeviceProperties");
  if (prop.major != 10) return vk_fail(VK_ERR_NO_DEVICE, "vk_init: device %d is sm_%d%d, this library is sm_100a", device, prop.major, prop.minor);
  vk_ctx* ctx = new vk_ctx();
  ctx->device = device;
  e = cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&ctx->d_err, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(ctx->d_err, 0, sizeof(int));
  if (e != cudaSuccess) {
    if (ctx->d_err) cudaFree(ctx->d_err);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return vk_cuda_status(e, "vk_init");
  }
  ctx->stream = ctx->own_stream;
  *out = ctx;
  return VK_OK;
}

extern "C" int vk_destroy(vk_ctx* ctx) {
  if (ctx == nullptr) return VK_OK;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (ctx->ws) cudaFree(ctx->ws);
  if (ctx->d_err) cudaFree(ctx->d_err);
  for (auto& l : ctx->rope_luts) cudaFree(l.lut);
  if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
  delete ctx;
  return VK_OK;
}

extern "C" int vk_stream_set(vk_ctx* ctx, void* stream) {
  if (ctx == nullptr) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_stream_set: NULL context");
  ctx->stream = stream ? static_cast<cudaStream_t>(stream) : ctx->own_stream;
  return VK_OK;
}

extern "C" int vk_set_math(vk_ctx* ctx, int math) {
  if (ctx == nullptr) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_set_math: NULL context");
  if (math != VK_MATH_F32 && math != VK_MATH_BF16 && math != VK_MATH_Q8_0)
    return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_set_math: unknown math %d", math);
  ctx->math = math;
  return VK_OK;
}

extern "C" int vk_synchronize(vk_ctx* ctx) {
  if (ctx == nullptr) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_synchronize: NULL context");
  cudaSetDevice(ctx->device);
  cudaError_t e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return vk_cuda_status(e, "vk_synchronize");
  int flag = 0;
  e = cudaMemcpy(&flag, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return vk_cuda_status(e, "vk_synchronize: error word");
  if (flag != 0) {
    cudaMemset(ctx->d_err, 0, sizeof(int));
    return vk_fail(VK_ERR_TIMEOUT, "a kernel gave up a bounded wait (device code 0x%x)", flag);
  }
  return VK_OK;
}

// Bump allocator over the context workspace (256-byte aligned slices).
void* Arena::take(size_t bytes) {
  size_t o = (off + 255) & ~size_t(255);
  off = o + bytes;
  return base ? static_cast<char*>(base) + o : nullptr;
}

// ------------------------------------------------------------------ helpers
// Rotation table of the reference (src/rope.rs:42-60, src/specialized.rs:389-410),
// computed on the host with the same f32 powf / sinf / cosf calls so the
// values are bit-identical: rot[(p * 2q + axis * q + i) * 2 + {0: sin, 1: cos}],
// q = head_dim / 4.
void host_rotations(const int64_t* pos, size_t n, size_t head_dim, float freq, std::vector<float>& rot) {
  const size_t half = head_dim / 2, quarter = half / 2;
  std::vector<float> inv(quarter);
  for (size_t i = 0; i < quarter; ++i) inv[i] = powf(freq, -2.0f * static_cast<float>(i) / static_cast<float>(half));
  rot.assign(n * 4 * quarter, 0.0f);
  for (size_t p = 0; p < n; ++p)
    for (size_t axis = 0; axis < 2; ++axis) {
      const float position = static_cast<float>(pos[2 * p + axis]);
      for (size_t i = 0; i < quarter; ++i) {
        const float ang = position * inv[i];
        const size_t off = (p * 2 * quarter + axis * quarter + i) * 2;
        rot[off] = sinf(ang);
        rot[off + 1] = cosf(ang);
      }
    }
}

// Per-token rotations of device positions, built on the device without a
// host round trip: the context keeps, per (head_dim, freq), a lookup table
// of the host's f32 sin / cos for integer positions [0, 4096) (built and
// uploaded once, on the first call), which the table kernel indexes.  Grid
// coordinates of any DA3 image size fall in that range; a position outside
// it takes sin / cos in double precision rounded to f32 (within an ulp of
// the host's f32 functions).
// head_dim above 128 (more than 32 frequencies): the positions are read back
// and the table built on the host, with two synchronisations.
static int rotations_via_host(vk_ctx* ctx, const int64_t* pos_dev, size_t n, size_t head_dim, float freq,
                              float* rot_dev) {
  std::vector<int64_t> pos(2 * n);
  VK_TRY_CUDA(cudaMemcpyAsync(pos.data(), pos_dev, pos.size() * sizeof(int64_t), cudaMemcpyDeviceToHost, ctx->stream),
              "positions download");
  VK_TRY_CUDA(cudaStreamSynchronize(ctx->stream), "positions download");
  std::vector<float> rot;
  host_rotations(pos.data(), n, head_dim, freq, rot);
  VK_TRY_CUDA(cudaMemcpyAsync(rot_dev, rot.data(), rot.size() * sizeof(float), cudaMemcpyHostToDevice, ctx->stream),
              "rotation upload");
  VK_TRY_CUDA(cudaStreamSynchronize(ctx->stream), "rotation upload");  // the host vector goes out of scope
  return VK_OK;
}

static int rotations_from_device_positions(vk_ctx* ctx, const int64_t* pos_dev, size_t n, size_t head_dim,
                                           float freq, float* rot_dev) {
  const size_t half = head_dim / 2, quarter = half / 2;
  if (quarter > 32) return rotations_via_host(ctx, pos_dev, n, head_dim, freq, rot_dev);
  uint32_t fbits;
  std::memcpy(&fbits, &freq, 4);
  vk_ctx::RopeLut* hit = nullptr;
  for (auto& l : ctx->rope_luts)
    if (l.quarter == quarter && l.freq_bits == fbits) hit = &l;
  if (hit == nullptr) {
    vk_ctx::RopeLut l{};
    l.quarter = quarter;
    l.freq_bits = fbits;
    std::vector<int64_t> pos(2 * VK_ROPE_LUT_POSITIONS);
    for (int p = 0; p < VK_ROPE_LUT_POSITIONS; ++p) pos[2 * p] = pos[2 * p + 1] = p;
    std::vector<float> rot;  // [p][axis][i][2]; the table keeps axis 0
    host_rotations(pos.data(), VK_ROPE_LUT_POSITIONS, head_dim, freq, rot);
    std::vector<float> lut(static_cast<size_t>(VK_ROPE_LUT_POSITIONS) * quarter * 2);
    for (size_t p = 0; p < static_cast<size_t>(VK_ROPE_LUT_POSITIONS); ++p)
      std::memcpy(&lut[p * quarter * 2], &rot[p * quarter * 4], quarter * 2 * sizeof(float));
    for (size_t i = 0; i < quarter; ++i) l.inv[i] = powf(freq, -2.0f * static_cast<float>(i) / static_cast<float>(half));
    VK_TRY_CUDA(cudaMalloc(&l.lut, lut.size() * sizeof(float)), "RoPE table");
    VK_TRY_CUDA(cudaMemcpy(l.lut, lut.data(), lut.size() * sizeof(float), cudaMemcpyHostToDevice), "RoPE table");
    ctx->rope_luts.push_back(l);
    hit = &ctx->rope_luts.back();
  }
  RopeInv inv{};
  for (size_t i = 0; i < quarter; ++i) inv.v[i] = hit->inv[i];
  VK_TRY_CUDA(rope_rotations_device(pos_dev, static_cast<int>(n), static_cast<int>(quarter), inv, hit->lut, rot_dev,
                                    ctx->stream),
              "RoPE rotations");
  return VK_OK;
}

static bool da3_projection(size_t k, size_t n) {
  return (k == 768 && (n == 2304 || n == 768 || n == 3072)) || (k == 3072 && n == 768);
}

#define VK_CTX_CHECK(ctx, name)                                                           \
  do {                                                                                    \
    if ((ctx) == nullptr) return vk_fail(VK_ERR_INVALID_ARGUMENT, name ": NULL context"); \
    cudaSetDevice((ctx)->device);                                                         \
  } while (0)

// One projection C = A[m,k] . W[k,n] with an epilogue, in the context's math.
// W is given in the reference layout [k, n] f32 and converted per call.
static int projection_raw(vk_ctx* ctx, size_t m, size_t n, size_t k, const float* a, const float* w, int mode,
                          GemmEpi epi, const char* name) {
  cudaStream_t s = ctx->stream;
  if (ctx->math == VK_MATH_F32) {
    if (mode == EPI_QKV_BF16) mode = EPI_QKV_F32;
    return vk_cuda_status(gemm_f32_simt(a, w, (int)m, (int)n, (int)k, mode, epi, s), name);
  }
  auto layout = [&](Arena& ar, void** p) {
    if (ctx->math == VK_MATH_BF16) {
      p[0] = ar.get<__nv_bfloat16>(m * k);
      p[1] = ar.get<__nv_bfloat16>(n * k);
    } else {
      p[0] = ar.get<int8_t>(m * k);
      p[1] = ar.get<__half>(m * k / 32);
      p[2] = ar.get<float>(n * k);
      p[3] = ar.get<int8_t>(n * k);
      p[4] = ar.get<__half>(n * k / 32);
    }
  };
  void* p[5] = {};
  Arena sizing;
  layout(sizing, p);
  VK_TRY(ctx_reserve(ctx, sizing.off + 256));
  Arena ar{ctx->ws, 0};
  layout(ar, p);
  if (ctx->math == VK_MATH_BF16) {
    auto* a16 = static_cast<__nv_bfloat16*>(p[0]);
    auto* w16 = static_cast<__nv_bfloat16*>(p[1]);
    VK_TRY_CUDA(cast_f32_bf16(a, a16, m * k, s), name);
    VK_TRY_CUDA(transpose_cast_bf16(w, w16, (int)k, (int)n, s), name);
    return vk_cuda_status(gemm_bf16_tc(a16, w16, (int)m, (int)n, (int)k, mode, epi, ctx->d_err, s), name);
  }
  auto* aq = static_cast<int8_t*>(p[0]);
  auto* ad = static_cast<__half*>(p[1]);
  auto* wt = static_cast<float*>(p[2]);
  auto* wq = static_cast<int8_t*>(p[3]);
  auto* wd = static_cast<__half*>(p[4]);
  VK_TRY_CUDA(quantize_q8_0(a, m * k / 32, aq, ad, s), name);
  VK_TRY_CUDA(transpose_f32(w, wt, (int)k, (int)n, s), name);
  VK_TRY_CUDA(quantize_q8_0(wt, n * k / 32, wq, wd, s), name);
  return vk_cuda_status(gemm_q8_tc(aq, ad, wq, wd, (int)m, (int)n, (int)k, mode, epi, nullptr, ctx->d_err, s), name);
}

// ------------------------------------------------------------------ DA3 specialised
extern "C" int vk_qkv_f32_da3_base(vk_ctx* ctx, size_t tokens, const float* input, const float* weight,
                                   const float* bias, float* q, float* k, float* v) {
  VK_CTX_CHECK(ctx, "vk_qkv_f32_da3_base");
  if (tokens == 0) return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_qkv_f32_da3_base: tokens == 0");
  VK_TRY(vk_dims_fit("vk_qkv_f32_da3_base", {tokens}));
  if (!input || !weight || !bias || !q || !k || !v)
    return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_qkv_f32_da3_base: NULL buffer");
  GemmEpi epi;
  epi.bias = bias;
  epi.q = q;
  epi.k = k;
  epi.v = v;
  epi.tokens = static_cast<int>(tokens);
  epi.heads = 12;
  return projection_raw(ctx, tokens, 2304, 768, input, weight, EPI_QKV_F32, epi, "vk_qkv_f32_da3_base");
}

extern "C" int vk_linear_f32_da3_base(vk_ctx* ctx, size_t m, size_t n, size_t k, const float* input,
                                      const float* weight, float* output) {
  VK_CTX_CHECK(ctx, "vk_linear_f32_da3_base");
  if (m == 0 || !da3_projection(k, n))
    return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_linear_f32_da3_base: (m=%zu, k=%zu, n=%zu) is not a DA3-BASE projection", m, k, n);
  VK_TRY(vk_dims_fit("vk_linear_f32_da3_base", {m}));
  if (!input || !weight || !output) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_linear_f32_da3_base: NULL buffer");
  GemmEpi epi;
  epi.out = output;
  epi.ldo = static_cast<int64_t>(n);
  return projection_raw(ctx, m, n, k, input, weight, EPI_F32, epi, "vk_linear_f32_da3_base");
}

extern "C" int vk_linear_bias_scale_f32_da3_base(vk_ctx* ctx, size_t m, size_t n, size_t k, const float* a,
                                                 const float* b, const float* bias, const float* scale, float* c) {
  VK_CTX_CHECK(ctx, "vk_linear_bias_scale_f32_da3_base");
  if (m == 0 || !((k == 768 && n == 768) || (k == 3072 && n == 768)))
    return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_linear_bias_scale_f32_da3_base: (k=%zu, n=%zu) unsupported", k, n);
  VK_TRY(vk_dims_fit("vk_linear_bias_scale_f32_da3_base", {m}));
  if (!a || !b || !bias || !scale || !c) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_linear_bias_scale_f32_da3_base: NULL buffer");
  GemmEpi epi;
  epi.bias = bias;
  epi.scale = scale;
  epi.out = c;
  epi.ldo = static_cast<int64_t>(n);
  return projection_raw(ctx, m, n, k, a, b, EPI_F32, epi, "vk_linear_bias_scale_f32_da3_base");
}

static int attention64(vk_ctx* ctx, const float* q, const float* k, const float* v, size_t heads, size_t tokens,
                       float* out, const char* name) {
  cudaStream_t s = ctx->stream;
  if (ctx->math == VK_MATH_F32)
    return vk_cuda_status(attention_f32(q, k, v, (int)heads, (int)tokens, 64, out, s), name);
  const size_t n = heads * tokens * 64;
  VK_TRY(ctx_reserve(ctx, 3 * n * sizeof(__nv_bfloat16) + 1024));
  Arena ar{ctx->ws, 0};
  auto* q16 = ar.get<__nv_bfloat16>(n);
  auto* k16 = ar.get<__nv_bfloat16>(n);
  auto* v16 = ar.get<__half>(n);  // V in f16, the type of the P V product
  VK_TRY_CUDA(cast_f32_bf16(q, q16, n, s), name);
  VK_TRY_CUDA(cast_f32_bf16(k, k16, n, s), name);
  VK_TRY_CUDA(cast_f32_f16(v, v16, n, s), name);
  return vk_cuda_status(attention_bf16(q16, k16, v16, 1, (int)heads, (int)tokens, ATTN_OUT_HEAD_F32, out, nullptr, ctx->d_err, s), name);
}

extern "C" int vk_flash_attention_f32_da3_base(vk_ctx* ctx, const float* query, const float* key, const float* value,
                                               size_t heads, size_t tokens, float* output) {
  VK_CTX_CHECK(ctx, "vk_flash_attention_f32_da3_base");
  if (heads == 0 || tokens == 0) return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_flash_attention_f32_da3_base: empty shape");
  VK_TRY(vk_dims_fit("vk_flash_attention_f32_da3_base", {heads, tokens}));
  if (!query || !key || !value || !output) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_flash_attention_f32_da3_base: NULL buffer");
  return attention64(ctx, query, key, value, heads, tokens, output, "vk_flash_attention_f32_da3_base");
}

extern "C" int vk_qk_norm_rope_f32_da3_base(vk_ctx* ctx, float* q, float* k, size_t heads, size_t tokens,
                                            const float* q_gamma, const float* q_beta, const float* k_gamma,
                                            const float* k_beta, const int64_t* positions_yx, float frequency,
                                            float epsilon) {
  VK_CTX_CHECK(ctx, "vk_qk_norm_rope_f32_da3_base");
  if (heads == 0 || tokens == 0) return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_qk_norm_rope_f32_da3_base: empty shape");
  VK_TRY(vk_dims_fit("vk_qk_norm_rope_f32_da3_base", {heads, tokens}));
  if (!q || !k || !q_gamma || !q_beta || !k_gamma || !k_beta || !positions_yx)
    return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_qk_norm_rope_f32_da3_base: NULL buffer");
  VK_TRY(ctx_reserve(ctx, tokens * 64 * sizeof(float) + 256));
  float* rot = static_cast<float*>(ctx->ws);
  VK_TRY(rotations_from_device_positions(ctx, positions_yx, tokens, 64, frequency, rot));
  return vk_cuda_status(qk_norm_rope_f32(q, k, (int)heads, (int)tokens, q_gamma, q_beta, k_gamma, k_beta, rot, epsilon,
                                         ctx->stream),
                        "vk_qk_norm_rope_f32_da3_base");
}

// ------------------------------------------------------------------ generic operators
extern "C" int vk_attention(vk_ctx* ctx, const float* q, const float* k, const float* v, size_t heads, size_t n,
                            size_t head_dim, float* out) {
  VK_CTX_CHECK(ctx, "vk_attention");
  if (heads == 0 || n == 0) return VK_OK;
  if (!q || !k || !v || !out) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_attention: NULL buffer");
  VK_TRY(vk_dims_fit("vk_attention", {heads, n}));
  if (head_dim == 64) return attention64(ctx, q, k, v, heads, n, out, "vk_attention");
  if (head_dim != 8 && head_dim != 16 && head_dim != 32)
    return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_attention: head_dim %zu (supported: 8, 16, 32, 64)", head_dim);
  return vk_cuda_status(attention_f32(q, k, v, (int)heads, (int)n, (int)head_dim, out, ctx->stream), "vk_attention");
}

extern "C" int vk_rope2d(vk_ctx* ctx, float* x, size_t heads, size_t n, size_t head_dim, const int64_t* pos_yx,
                         float freq) {
  VK_CTX_CHECK(ctx, "vk_rope2d");
  if (head_dim % 4 != 0) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_rope2d: head_dim must be divisible by 4, got %zu", head_dim);
  if (heads == 0 || n == 0 || head_dim == 0) return VK_OK;
  if (!x || !pos_yx) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_rope2d: NULL buffer");
  VK_TRY(vk_dims_fit("vk_rope2d", {heads, n, head_dim}));
  VK_TRY(ctx_reserve(ctx, n * head_dim * sizeof(float) + 256));
  float* rot = static_cast<float*>(ctx->ws);
  VK_TRY(rotations_from_device_positions(ctx, pos_yx, n, head_dim, freq, rot));
  return vk_cuda_status(rope2d_f32(x, (int)heads, (int)n, (int)head_dim, rot, ctx->stream), "vk_rope2d");
}

extern "C" int vk_layernorm(vk_ctx* ctx, float* x, size_t rows, size_t cols, const float* gamma, const float* beta,
                            float eps) {
  VK_CTX_CHECK(ctx, "vk_layernorm");
  if (rows == 0 || cols == 0) return VK_OK;
  if (!x || !gamma || !beta) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_layernorm: NULL buffer");
  VK_TRY(vk_dims_fit("vk_layernorm", {rows, cols}));
  return vk_cuda_status(layernorm_f32(x, x, nullptr, nullptr, nullptr, (int)rows, (int)cols, gamma, beta, eps, ctx->stream),
                        "vk_layernorm");
}

extern "C" int vk_gelu(vk_ctx* ctx, float* x, size_t n) {
  VK_CTX_CHECK(ctx, "vk_gelu");
  if (n && !x) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_gelu: NULL buffer");
  return vk_cuda_status(gelu_f32(x, n, ctx->stream), "vk_gelu");
}

extern "C" int vk_add(vk_ctx* ctx, float* dst, const float* src, size_t n) {
  VK_CTX_CHECK(ctx, "vk_add");
  if (n && (!dst || !src)) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_add: NULL buffer");
  return vk_cuda_status(add_f32(dst, src, n, ctx->stream), "vk_add");
}

extern "C" int vk_add_bias_rows(vk_ctx* ctx, float* x, size_t rows, size_t cols, const float* bias) {
  VK_CTX_CHECK(ctx, "vk_add_bias_rows");
  if (rows * cols && (!x || !bias)) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_add_bias_rows: NULL buffer");
  return vk_cuda_status(add_bias_rows_f32(x, rows, cols, bias, ctx->stream), "vk_add_bias_rows");
}

extern "C" int vk_layerscale(vk_ctx* ctx, float* x, size_t rows, size_t cols, const float* gamma) {
  VK_CTX_CHECK(ctx, "vk_layerscale");
  if (rows * cols && (!x || !gamma)) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_layerscale: NULL buffer");
  return vk_cuda_status(layerscale_f32(x, rows, cols, gamma, ctx->stream), "vk_layerscale");
}

extern "C" int vk_quantize_row_q8_0(vk_ctx* ctx, const float* x, size_t nblocks, vk_block_q8_0* out) {
  VK_CTX_CHECK(ctx, "vk_quantize_row_q8_0");
  if (nblocks == 0) return VK_OK;
  if (!x || !out) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_quantize_row_q8_0: NULL buffer");
  if (reinterpret_cast<uintptr_t>(x) % 16 != 0)
    return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_quantize_row_q8_0: x must be 16-byte aligned");
  Arena sizing;
  sizing.get<int8_t>(nblocks * 32);
  sizing.get<__half>(nblocks);
  VK_TRY(ctx_reserve(ctx, sizing.off + 256));
  Arena ar{ctx->ws, 0};
  auto* qs = ar.get<int8_t>(nblocks * 32);
  auto* d = ar.get<__half>(nblocks);
  VK_TRY_CUDA(quantize_q8_0(x, nblocks, qs, d, ctx->stream), "vk_quantize_row_q8_0");
  return vk_cuda_status(pack_blocks_q8_0(qs, d, nblocks, out, ctx->stream), "vk_quantize_row_q8_0");
}

static int gemm_q8_blocks(vk_ctx* ctx, size_t m, size_t n, size_t k, const vk_block_q8_0* a_q,
                          const vk_block_q8_0* b_q, float* c, int32_t* dots, const char* name) {
  if (ctx == nullptr) return vk_fail(VK_ERR_INVALID_ARGUMENT, "%s: NULL context", name);
  cudaSetDevice(ctx->device);
  if (m == 0 || n == 0) return VK_OK;
  if (k == 0 || k % 128 != 0 || n % 128 != 0)
    return vk_fail(VK_UNSUPPORTED_SHAPE, "%s: needs k %% 128 == 0 and n %% 128 == 0 (k=%zu, n=%zu)", name, k, n);
  if (!a_q || !b_q || (!c && !dots)) return vk_fail(VK_ERR_INVALID_ARGUMENT, "%s: NULL buffer", name);
  VK_TRY(vk_dims_fit(name, {m, n, k}));
  const size_t nb = k / 32;
  auto layout = [&](Arena& ar, void** p) {
    p[0] = ar.get<int8_t>(m * k);
    p[1] = ar.get<__half>(m * nb);
    p[2] = ar.get<int8_t>(n * k);
    p[3] = ar.get<__half>(n * nb);
    p[4] = ar.get<float>(dots ? m * n : 0);
  };
  void* p[5];
  Arena sizing;
  layout(sizing, p);
  VK_TRY(ctx_reserve(ctx, sizing.off + 256));
  Arena ar{ctx->ws, 0};
  layout(ar, p);
  cudaStream_t s = ctx->stream;
  VK_TRY_CUDA(unpack_blocks_q8_0(a_q, m * nb, static_cast<int8_t*>(p[0]), static_cast<__half*>(p[1]), s), name);
  VK_TRY_CUDA(unpack_blocks_q8_0(b_q, n * nb, static_cast<int8_t*>(p[2]), static_cast<__half*>(p[3]), s), name);
  GemmEpi epi;
  epi.out = dots ? p[4] : c;
  epi.ldo = static_cast<int64_t>(n);
  return vk_cuda_status(gemm_q8_tc(static_cast<int8_t*>(p[0]), static_cast<__half*>(p[1]), static_cast<int8_t*>(p[2]),
                                   static_cast<__half*>(p[3]), (int)m, (int)n, (int)k, EPI_F32, epi, dots, ctx->d_err, s),
                        name);
}

extern "C" int vk_gemm_q8_0(vk_ctx* ctx, size_t m, size_t n, size_t k, const vk_block_q8_0* a_q,
                            const vk_block_q8_0* b_q, float* c) {
  return gemm_q8_blocks(ctx, m, n, k, a_q, b_q, c, nullptr, "vk_gemm_q8_0");
}

extern "C" int vk_gemm_q8_0_block_dots(vk_ctx* ctx, size_t m, size_t n, size_t k, const vk_block_q8_0* a_q,
                                       const vk_block_q8_0* b_q, int32_t* dots) {
  return gemm_q8_blocks(ctx, m, n, k, a_q, b_q, nullptr, dots, "vk_gemm_q8_0_block_dots");
}

// ------------------------------------------------------------------ prepared linears
static int upload(void** dst, const void* src, size_t bytes, std::vector<void*>* track) {
  VK_TRY_CUDA(cudaMalloc(dst, bytes), "weight allocation");
  if (track) track->push_back(*dst);
  VK_TRY_CUDA(cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice), "weight upload");
  return VK_OK;
}

// Converts a host [k, n] f32 weight into the device form of `math`.
int prepare_weight(size_t k, size_t n, const float* w_host, int math, float** w32, __nv_bfloat16** w16, int8_t** wq,
                   __half** wd, std::vector<void*>* track) {
  float* tmp = nullptr;
  VK_TRY(upload(reinterpret_cast<void**>(&tmp), w_host, k * n * sizeof(float), nullptr));
  int st = VK_OK;
  if (math == VK_MATH_F32) {
    *w32 = tmp;
    if (track) track->push_back(tmp);
    return VK_OK;
  }
  if (math == VK_MATH_BF16) {
    cudaError_t e = cudaMalloc(w16, n * k * sizeof(__nv_bfloat16));
    if (e == cudaSuccess) {
      if (track) track->push_back(*w16);
      e = transpose_cast_bf16(tmp, *w16, (int)k, (int)n, 0);
    }
    st = vk_cuda_status(e, "bf16 weight preparation");
  } else {
    float* wt = nullptr;
    cudaError_t e = cudaMalloc(&wt, n * k * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(wq, n * k);
    if (e == cudaSuccess) {
      if (track) track->push_back(*wq);
      e = cudaMalloc(wd, n * k / 32 * sizeof(__half));
    }
    if (e == cudaSuccess) {
      if (track) track->push_back(*wd);
      e = transpose_f32(tmp, wt, (int)k, (int)n, 0);
    }
    if (e == cudaSuccess) e = quantize_q8_0(wt, n * k / 32, *wq, *wd, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (wt) cudaFree(wt);
    st = vk_cuda_status(e, "Q8_0 weight preparation");
  }
  cudaDeviceSynchronize();
  cudaFree(tmp);
  return st;
}

static void free_linear(vk_linear* l) {
  if (!l) return;
  cudaSetDevice(l->device);
  for (void* p : {static_cast<void*>(l->w_f32), static_cast<void*>(l->w_bf16), static_cast<void*>(l->w_q),
                  static_cast<void*>(l->w_d), static_cast<void*>(l->bias), static_cast<void*>(l->scale)})
    if (p) cudaFree(p);
  delete l;
}

static int prepare_vectors(vk_linear* l, const float* bias, const float* scale) {
  if (bias) VK_TRY(upload(reinterpret_cast<void**>(&l->bias), bias, l->n * sizeof(float), nullptr));
  if (scale) VK_TRY(upload(reinterpret_cast<void**>(&l->scale), scale, l->n * sizeof(float), nullptr));
  return VK_OK;
}

extern "C" int vk_prepare_linear(vk_ctx* ctx, size_t k, size_t n, const float* weight_host, const float* bias_host,
                                 const float* scale_host, int math, vk_linear** out) {
  VK_CTX_CHECK(ctx, "vk_prepare_linear");
  if (!out || !weight_host) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_prepare_linear: NULL argument");
  *out = nullptr;
  if (k == 0 || n == 0) return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_prepare_linear: empty weight");
  if (math == VK_MATH_BF16 && (k % 64 != 0 || n % 128 != 0))
    return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_prepare_linear: bf16 needs k %% 64 == 0 and n %% 128 == 0");
  if (math == VK_MATH_Q8_0 && (k % 128 != 0 || n % 128 != 0))
    return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_prepare_linear: Q8_0 needs k %% 128 == 0 and n %% 128 == 0");
  if (math != VK_MATH_F32 && math != VK_MATH_BF16 && math != VK_MATH_Q8_0)
    return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_prepare_linear: unknown math %d", math);
  vk_linear* l = new vk_linear();
  l->device = ctx->device;
  l->math = math;
  l->k = k;
  l->n = n;
  int st = prepare_weight(k, n, weight_host, math, &l->w_f32, &l->w_bf16, &l->w_q, &l->w_d, nullptr);
  if (st == VK_OK) st = prepare_vectors(l, bias_host, scale_host);
  if (st != VK_OK) {
    free_linear(l);
    return st;
  }
  *out = l;
  return VK_OK;
}

extern "C" int vk_prepare_linear_q8_0(vk_ctx* ctx, size_t k, size_t n, const vk_block_q8_0* blocks_host,
                                      const float* bias_host, const float* scale_host, vk_linear** out) {
  VK_CTX_CHECK(ctx, "vk_prepare_linear_q8_0");
  if (!out || !blocks_host) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_prepare_linear_q8_0: NULL argument");
  *out = nullptr;
  if (k == 0 || n == 0 || k % 128 != 0 || n % 128 != 0)
    return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_prepare_linear_q8_0: needs k %% 128 == 0 and n %% 128 == 0");
  vk_linear* l = new vk_linear();
  l->device = ctx->device;
  l->math = VK_MATH_Q8_0;
  l->k = k;
  l->n = n;
  const size_t nblocks = n * k / 32;
  void* tmp = nullptr;
  int st = upload(&tmp, blocks_host, nblocks * sizeof(vk_block_q8_0), nullptr);
  cudaError_t e = cudaSuccess;
  if (st == VK_OK) e = cudaMalloc(&l->w_q, n * k);
  if (st == VK_OK && e == cudaSuccess) e = cudaMalloc(&l->w_d, nblocks * sizeof(__half));
  if (st == VK_OK && e == cudaSuccess) e = unpack_blocks_q8_0(tmp, nblocks, l->w_q, l->w_d, 0);
  if (st == VK_OK && e == cudaSuccess) e = cudaDeviceSynchronize();
  if (tmp) cudaFree(tmp);
  if (st == VK_OK) st = vk_cuda_status(e, "vk_prepare_linear_q8_0");
  if (st == VK_OK) st = prepare_vectors(l, bias_host, scale_host);
  if (st != VK_OK) {
    free_linear(l);
    return st;
  }
  *out = l;
  return VK_OK;
}

extern "C" int vk_linear_run(vk_ctx* ctx, const vk_linear* lin, size_t m, const float* input, float* output) {
  VK_CTX_CHECK(ctx, "vk_linear_run");
  if (!lin || !input || !output) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_linear_run: NULL argument");
  VK_TRY(vk_dims_fit("vk_linear_run", {m}));
  if (m == 0) return VK_OK;
  const size_t k = lin->k, n = lin->n;
  GemmEpi epi;
  epi.bias = lin->bias;
  epi.scale = lin->scale;
  epi.out = output;
  epi.ldo = static_cast<int64_t>(n);
  cudaStream_t s = ctx->stream;
  if (lin->math == VK_MATH_F32)
    return vk_cuda_status(gemm_f32_simt(input, lin->w_f32, (int)m, (int)n, (int)k, EPI_F32, epi, s), "vk_linear_run");
  if (lin->math == VK_MATH_BF16) {
    VK_TRY(ctx_reserve(ctx, m * k * sizeof(__nv_bfloat16) + 256));
    auto* a16 = static_cast<__nv_bfloat16*>(ctx->ws);
    VK_TRY_CUDA(cast_f32_bf16(input, a16, m * k, s), "vk_linear_run");
    return vk_cuda_status(gemm_bf16_tc(a16, lin->w_bf16, (int)m, (int)n, (int)k, EPI_F32, epi, ctx->d_err, s),
                          "vk_linear_run");
  }
  Arena sizing;
  sizing.get<int8_t>(m * k);
  sizing.get<__half>(m * k / 32);
  VK_TRY(ctx_reserve(ctx, sizing.off + 256));
  Arena ar{ctx->ws, 0};
  auto* aq = ar.get<int8_t>(m * k);
  auto* ad = ar.get<__half>(m * k / 32);
  VK_TRY_CUDA(quantize_q8_0(input, m * k / 32, aq, ad, s), "vk_linear_run");
  return vk_cuda_status(gemm_q8_tc(aq, ad, lin->w_q, lin->w_d, (int)m, (int)n, (int)k, EPI_F32, epi, nullptr, ctx->d_err, s),
                        "vk_linear_run");
}

extern "C" int vk_release_linear(vk_linear* lin) {
  free_linear(lin);
  return VK_OK;
}
