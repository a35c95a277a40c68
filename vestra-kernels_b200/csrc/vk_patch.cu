// vk_patch.cu -- DA3 patch embedding and token assembly: the step before the
// encoder.
//
// Operators with the reference's semantics (src/cuda.rs:295-334 kernels,
// CudaRuntime::patchify_nchw_f32 / prepend_cls_add_pos_f32 at
// src/cuda.rs:1073-1175):
//   vk_patchify_nchw_f32       NCHW image -> [patches, C * p * p] rows, the
//                              row index following the OIHW inner order
//                              (channel, patch_y, patch_x)
//   vk_prepend_cls_add_pos_f32 tokens = [cls; patches] + position
// and the batched embedding the engine composes from them, as one call:
//   vk_patch_embed_forward     tokens[b] = [cls; patchify(image[b]) . W + bias] + position
// f32 math runs the ascending-K FMA GEMM (bit-exact with the reference's f32
// projection arithmetic); bf16 math patchifies straight into a K-padded bf16
// operand (C * p * p = 588 -> 640, zeros) for the tensor-core GEMM.
#include "vestra_b200.h"
#include "vk_abi_internal.h"
#include "vk_common.cuh"
#include "vk_internal.h"

using namespace vk;

namespace {

constexpr int PT_THREADS = 256;

// One thread per output element, in output order (coalesced writes; the
// reads walk image rows patch-width at a time).
__global__ void k_patchify_f32(const float* __restrict__ image, float* __restrict__ patches, int images, int height,
                               int width, int patch, int channels) {
  const int gw = width / patch, gh = height / patch;
  const int row_width = channels * patch * patch;
  const size_t per_image = static_cast<size_t>(gh) * gw * row_width;
  const size_t total = per_image * images;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t b = i / per_image;
    const size_t r = i - b * per_image;
    const int p = static_cast<int>(r / row_width);
    const int w = static_cast<int>(r - static_cast<size_t>(p) * row_width);
    const int c = w / (patch * patch), s = w - c * patch * patch;
    const int y = (p / gw) * patch + s / patch, x = (p % gw) * patch + s % patch;
    patches[i] = image[((b * channels + c) * height + y) * width + x];
  }
}

// As k_patchify_f32 into bf16 rows of `kpad` >= C * p * p columns (the tail
// zero), the A operand of the tensor-core GEMM.  Driven by the input: block
// row blockIdx.y is one image row (b, c, y), read coalesced, one thread per
// pixel; pixel x lands in patch x / p at column c p^2 + (y % p) p + x % p,
// so each patch receives a contiguous run of p values.  The padding columns
// are zeroed by k_patch_pad.
__global__ void k_patchify_bf16(const float* __restrict__ image, __nv_bfloat16* __restrict__ patches, int images,
                                int height, int width, int patch, int channels, int kpad) {
  const int gw = width / patch, gh = height / patch;
  const int x = blockIdx.x * blockDim.x + threadIdx.x;
  const int rows = images * channels * height;
  for (int rid = blockIdx.y; rid < rows; rid += gridDim.y) {
    if (x >= width) continue;
    const int y = rid % height, bc = rid / height, c = bc % channels, b = bc / channels;
    const float v = image[static_cast<size_t>(rid) * width + x];
    const int px = x / patch, sx = x - px * patch, gy = y / patch, sy = y - gy * patch;
    const size_t prow = static_cast<size_t>(b) * gh * gw + static_cast<size_t>(gy) * gw + px;
    patches[prow * kpad + (c * patch + sy) * patch + sx] = __float2bfloat16_rn(v);
  }
}
__global__ void k_patch_pad(__nv_bfloat16* __restrict__ patches, size_t rows, int row_width, int kpad) {
  const int pad = kpad - row_width;
  const size_t total = rows * pad;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t r = i / pad;
    patches[r * kpad + row_width + (i - r * pad)] = __float2bfloat16_rn(0.0f);
  }
}

// tokens[b][0] = cls + position[0] for every image (the bf16 path, whose
// GEMM epilogue writes the patch rows).
__global__ void k_cls_rows(const float* __restrict__ cls, const float* __restrict__ position, float* __restrict__ tokens,
                           int images, int patch_count, int embed) {
  const int e4 = embed / 4;
  const size_t total = static_cast<size_t>(images) * e4;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t b = i / e4;
    const int c = static_cast<int>(i - b * e4);
    const float4 v = reinterpret_cast<const float4*>(cls)[c], q = reinterpret_cast<const float4*>(position)[c];
    reinterpret_cast<float4*>(tokens)[b * (static_cast<size_t>(patch_count) + 1) * e4 + c] =
        make_float4(v.x + q.x, v.y + q.y, v.z + q.z, v.w + q.w);
  }
}

// tokens[b][0] = cls + position[0]; tokens[b][t] = projected[b][t - 1] + position[t]
// (value + position, as the reference kernel).  float4 per thread.
__global__ void k_assemble_tokens(const float* __restrict__ projected, const float* __restrict__ cls,
                                  const float* __restrict__ position, float* __restrict__ tokens, int images,
                                  int patch_count, int embed) {
  const int e4 = embed / 4;
  const size_t per_image = static_cast<size_t>(patch_count + 1) * e4;
  const size_t total = per_image * images;
  const float4* proj4 = reinterpret_cast<const float4*>(projected);
  const float4* cls4 = reinterpret_cast<const float4*>(cls);
  const float4* pos4 = reinterpret_cast<const float4*>(position);
  float4* out4 = reinterpret_cast<float4*>(tokens);
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t b = i / per_image;
    const size_t r = i - b * per_image;
    const size_t t = r / e4;
    const int c = static_cast<int>(r - t * e4);
    const float4 v = t == 0 ? cls4[c] : proj4[(b * patch_count + (t - 1)) * e4 + c];
    const float4 p = pos4[r];
    out4[i] = make_float4(v.x + p.x, v.y + p.y, v.z + p.z, v.w + p.w);
  }
}

// Scalar form of the same (any embed width): the single-image reference operator.
__global__ void k_prepend_cls_add_pos(const float* __restrict__ patches, const float* __restrict__ cls,
                                      const float* __restrict__ position, float* __restrict__ tokens,
                                      int patch_count, int embed) {
  const size_t total = static_cast<size_t>(patch_count + 1) * embed;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t t = i / embed;
    const size_t c = i - t * embed;
    const float v = t == 0 ? cls[c] : patches[(t - 1) * embed + c];
    tokens[i] = v + position[i];
  }
}

int grid_for(size_t n) {
  const size_t g = (n + PT_THREADS - 1) / PT_THREADS;
  const size_t cap = static_cast<size_t>(num_sms()) * 16;
  return static_cast<int>(g < cap ? (g > 0 ? g : 1) : cap);
}

bool patch_shape_ok(size_t height, size_t width, size_t patch, size_t channels) {
  return height > 0 && width > 0 && patch > 0 && channels > 0 && height % patch == 0 && width % patch == 0 &&
         height <= (1u << 20) && width <= (1u << 20);
}

}  // namespace

struct vk_patch_embed {
  int device = 0;
  int math = VK_MATH_F32;
  size_t channels = 0, patch = 0, embed = 0, k = 0, kpad = 0;
  float* w_f32 = nullptr;          // [k, embed] (f32 math)
  __nv_bfloat16* w_bf16 = nullptr; // [embed, kpad] (bf16 math, zero-padded K)
  float* bias = nullptr;           // [embed]
  float* cls = nullptr;            // [embed]
};

int prepare_weight(size_t k, size_t n, const float* w_host, int math, float** w32, __nv_bfloat16** w16, int8_t** wq,
                   __half** wd, std::vector<void*>* track);

extern "C" int vk_patchify_nchw_f32(vk_ctx* ctx, const float* image, size_t height, size_t width, size_t patch,
                                    size_t channels, float* patches) {
  if (!ctx) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_patchify_nchw_f32: NULL context");
  cudaSetDevice(ctx->device);
  if (!image || !patches) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_patchify_nchw_f32: NULL buffer");
  if (!patch_shape_ok(height, width, patch, channels))
    return vk_fail(VK_ERR_INVALID_ARGUMENT,
                   "vk_patchify_nchw_f32: invalid NCHW patchify shape channels=%zu height=%zu width=%zu patch=%zu",
                   channels, height, width, patch);
  const size_t n = channels * height * width;
  k_patchify_f32<<<grid_for(n), PT_THREADS, 0, ctx->stream>>>(image, patches, 1, (int)height, (int)width, (int)patch,
                                                               (int)channels);
  return vk_cuda_status(cudaGetLastError(), "vk_patchify_nchw_f32");
}

extern "C" int vk_prepend_cls_add_pos_f32(vk_ctx* ctx, const float* patches, const float* cls, const float* position,
                                          size_t patch_count, size_t embed, float* tokens) {
  if (!ctx) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_prepend_cls_add_pos_f32: NULL context");
  cudaSetDevice(ctx->device);
  if (!cls || !position || !tokens || (patch_count > 0 && !patches))
    return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_prepend_cls_add_pos_f32: NULL buffer");
  if (embed == 0) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_prepend_cls_add_pos_f32: embed == 0");
  const size_t n = (patch_count + 1) * embed;
  k_prepend_cls_add_pos<<<grid_for(n), PT_THREADS, 0, ctx->stream>>>(patches, cls, position, tokens,
                                                                      (int)patch_count, (int)embed);
  return vk_cuda_status(cudaGetLastError(), "vk_prepend_cls_add_pos_f32");
}

static void free_patch_embed(vk_patch_embed* pe) {
  if (!pe) return;
  cudaSetDevice(pe->device);
  for (void* p : {static_cast<void*>(pe->w_f32), static_cast<void*>(pe->w_bf16), static_cast<void*>(pe->bias),
                  static_cast<void*>(pe->cls)})
    if (p) cudaFree(p);
  delete pe;
}

extern "C" int vk_patch_embed_prepare(vk_ctx* ctx, size_t channels, size_t patch, size_t embed,
                                      const float* weight_host, const float* bias_host, const float* cls_host, int math,
                                      vk_patch_embed** out) {
  if (!ctx) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_patch_embed_prepare: NULL context");
  cudaSetDevice(ctx->device);
  if (!out || !weight_host || !bias_host || !cls_host)
    return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_patch_embed_prepare: NULL argument");
  *out = nullptr;
  if (channels == 0 || patch == 0 || embed == 0 || embed % 4 != 0)
    return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_patch_embed_prepare: needs embed %% 4 == 0");
  if (math == VK_MATH_BF16 && embed % 128 != 0)
    return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_patch_embed_prepare: bf16 needs embed %% 128 == 0");
  if (math != VK_MATH_F32 && math != VK_MATH_BF16)
    return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_patch_embed_prepare: math must be f32 or bf16");
  vk_patch_embed* pe = new vk_patch_embed();
  pe->device = ctx->device;
  pe->math = math;
  pe->channels = channels;
  pe->patch = patch;
  pe->embed = embed;
  pe->k = channels * patch * patch;
  pe->kpad = (pe->k + 63) / 64 * 64;
  int st = VK_OK;
  if (math == VK_MATH_F32) {
    st = prepare_weight(pe->k, embed, weight_host, VK_MATH_F32, &pe->w_f32, nullptr, nullptr, nullptr, nullptr);
  } else {
    std::vector<float> padded(pe->kpad * embed, 0.0f);  // zero rows beyond K
    std::copy(weight_host, weight_host + pe->k * embed, padded.begin());
    st = prepare_weight(pe->kpad, embed, padded.data(), VK_MATH_BF16, nullptr, &pe->w_bf16, nullptr, nullptr, nullptr);
  }
  auto up = [&](float** dst, const float* src) -> int {
    VK_TRY_CUDA(cudaMalloc(dst, embed * sizeof(float)), "vk_patch_embed_prepare");
    VK_TRY_CUDA(cudaMemcpy(*dst, src, embed * sizeof(float), cudaMemcpyHostToDevice), "vk_patch_embed_prepare");
    return VK_OK;
  };
  if (st == VK_OK) st = up(&pe->bias, bias_host);
  if (st == VK_OK) st = up(&pe->cls, cls_host);
  if (st != VK_OK) {
    free_patch_embed(pe);
    return st;
  }
  *out = pe;
  return VK_OK;
}

extern "C" int vk_patch_embed_forward(vk_ctx* ctx, const vk_patch_embed* pe, size_t images, size_t height,
                                      size_t width, const float* images_dev, const float* position_dev,
                                      float* tokens_dev) {
  if (!ctx || !pe) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_patch_embed_forward: NULL context or embedding");
  cudaSetDevice(ctx->device);
  if (images == 0) return VK_OK;
  if (!images_dev || !position_dev || !tokens_dev)
    return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_patch_embed_forward: NULL buffer");
  if (!patch_shape_ok(height, width, pe->patch, pe->channels))
    return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_patch_embed_forward: %zux%zu is not a multiple of the %zu-pixel patch",
                   height, width, pe->patch);
  if (reinterpret_cast<uintptr_t>(position_dev) % 16 != 0 || reinterpret_cast<uintptr_t>(tokens_dev) % 16 != 0)
    return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_patch_embed_forward: position and tokens must be 16-byte aligned");
  VK_TRY(vk_dims_fit("vk_patch_embed_forward", {images * pe->channels * height, width, images * (height / pe->patch) *
                                                 (width / pe->patch)}));
  const size_t np = (height / pe->patch) * (width / pe->patch), E = pe->embed;
  const size_t rows = images * np;
  cudaStream_t s = ctx->stream;
  Arena sizing;
  if (pe->math == VK_MATH_F32) {
    sizing.get<float>(rows * pe->k);
    sizing.get<float>(rows * E);  // the projection, assembled into tokens after
  } else {
    sizing.get<__nv_bfloat16>(rows * pe->kpad);
  }
  VK_TRY(ctx_reserve(ctx, sizing.off + 256));
  Arena ar{ctx->ws, 0};
  GemmEpi epi;
  epi.bias = pe->bias;
  epi.ldo = static_cast<int64_t>(E);
  if (pe->math == VK_MATH_F32) {
    float* a = ar.get<float>(rows * pe->k);
    float* proj = ar.get<float>(rows * E);
    k_patchify_f32<<<grid_for(rows * pe->k), PT_THREADS, 0, s>>>(images_dev, a, (int)images, (int)height, (int)width,
                                                                  (int)pe->patch, (int)pe->channels);
    VK_TRY_CUDA(cudaGetLastError(), "vk_patch_embed_forward: patchify");
    epi.out = proj;
    VK_TRY_CUDA(gemm_f32_simt(a, pe->w_f32, (int)rows, (int)E, (int)pe->k, EPI_F32, epi, s),
                "vk_patch_embed_forward: projection");
    k_assemble_tokens<<<grid_for((np + 1) * (E / 4) * images), PT_THREADS, 0, s>>>(proj, pe->cls, position_dev, tokens_dev,
                                                                                  (int)images, (int)np, (int)E);
  } else {
    auto* a = ar.get<__nv_bfloat16>(rows * pe->kpad);
    {
      const int in_rows = static_cast<int>(images * pe->channels * height);
      const dim3 grid(static_cast<unsigned>((width + PT_THREADS - 1) / PT_THREADS),
                      static_cast<unsigned>(in_rows < 65535 ? in_rows : 65535));
      k_patchify_bf16<<<grid, PT_THREADS, 0, s>>>(images_dev, a, (int)images, (int)height, (int)width, (int)pe->patch,
                                                  (int)pe->channels, (int)pe->kpad);
      const int row_width = static_cast<int>(pe->channels * pe->patch * pe->patch);
      if (static_cast<int>(pe->kpad) > row_width)
        k_patch_pad<<<grid_for(rows * (pe->kpad - row_width)), PT_THREADS, 0, s>>>(a, rows, row_width, (int)pe->kpad);
    }
    VK_TRY_CUDA(cudaGetLastError(), "vk_patch_embed_forward: patchify");
    // the GEMM's epilogue adds the positions and writes each patch straight
    // to its token row (1 + p of its image); the cls rows come from a small
    // kernel
    epi.out = tokens_dev;
    epi.tokens = static_cast<int>(np);
    epi.pos = position_dev;
    VK_TRY_CUDA(gemm_bf16_tc(a, pe->w_bf16, (int)rows, (int)E, (int)pe->kpad, EPI_TOKENS, epi, ctx->d_err, s),
                "vk_patch_embed_forward: projection");
    k_cls_rows<<<grid_for(images * (E / 4)), PT_THREADS, 0, s>>>(pe->cls, position_dev, tokens_dev, (int)images,
                                                                  (int)np, (int)E);
  }
  return vk_cuda_status(cudaGetLastError(), "vk_patch_embed_forward: assembly");
}

extern "C" int vk_patch_embed_release(vk_patch_embed* pe) {
  free_patch_embed(pe);
  return VK_OK;
}
