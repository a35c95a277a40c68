// vk_dpt.cu -- the DPT head's consumers of the encoder output: the step after
// the encoder.
//
//   vk_token_to_chw_f32        [tokens, channels] -> [channels, tokens]
//                              (src/cuda.rs:278-291), a 32 x 32 tiled
//                              transpose through shared memory
//   vk_bilinear_resize_f32     half-pixel centres (src/resample.rs:10-99)
//   vk_bilinear_resize_align_corners_f32 (src/resample.rs:151-249)
//   vk_conv3x3_*               the Winograd F(2x2, 3x3) convolutions
//                              (src/conv.rs:121-171, 304-484, 681-831)
//
// Resizes are one thread per output sample, with the reference's f32
// operations in its order (explicit round-to-nearest intrinsics, so nothing
// is contracted into an FMA): bit-exact.
//
// The convolution is one fused kernel per (32 tiles of 2x2 outputs, 32
// output channels).  Per 16-channel slice it builds the transformed input
// V = B^T d B of its tiles in shared memory (sampling through the fused
// align-corners resize and add, or ReLU, where asked), stages the matching
// slice of the prepared filter U, and accumulates the 16 transform-domain
// products M_p = V_p U_p in registers: each thread owns one of the 16
// positions for 8 tiles x 8 channels.  The output transform A^T M A then
// runs from shared memory and writes the 2x2 outputs with the bias.
#include "vestra_b200.h"
#include "vk_abi_internal.h"
#include "vk_common.cuh"
#include "vk_internal.h"

using namespace vk;

struct vk_conv3x3 {
  int device = 0;
  size_t in_c = 0, out_c = 0;
  float* u = nullptr;  // [16][in_c][out_c]
};

namespace {

constexpr int DT_THREADS = 256;

// ---------------------------------------------------------------- layout
__global__ void k_token_to_chw(const float* __restrict__ tm, float* __restrict__ chw, int tokens, int channels) {
  __shared__ float tile[32][33];
  const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  const size_t off = static_cast<size_t>(blockIdx.z) * tokens * channels;  // image
  tm += off;
  chw += off;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
  for (int r = ty; r < 32; r += 8) {
    const int t = t0 + r, c = c0 + tx;
    if (t < tokens && c < channels) tile[r][tx] = tm[static_cast<size_t>(t) * channels + c];
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    const int c = c0 + r, t = t0 + tx;
    if (t < tokens && c < channels) chw[static_cast<size_t>(c) * tokens + t] = tile[tx][r];
  }
}

// ---------------------------------------------------------------- resize
struct Coord {
  int i0, i1;
  float f;
};

// src/resample.rs:82-99 src_coord
__device__ __forceinline__ Coord hp_coord(int dst, float scale, int len_in) {
  const float src = __fsub_rn(__fmul_rn(__fadd_rn(static_cast<float>(dst), 0.5f), scale), 0.5f);
  const float sc = src > 0.0f ? src : 0.0f;
  int a = static_cast<int>(floorf(sc));
  a = a < len_in - 1 ? a : len_in - 1;
  const int b = a + 1 < len_in - 1 ? a + 1 : len_in - 1;
  float f = b == a ? 0.0f : __fsub_rn(sc, static_cast<float>(a));
  f = fminf(fmaxf(f, 0.0f), 1.0f);
  return {a, b, f};
}

// src/resample.rs:151-167 src_coord_align_corners (= the closure of
// src/conv.rs:320-336)
__device__ __forceinline__ Coord ac_coord(int dst, int len_in, int len_out) {
  if (len_in <= 1) return {0, 0, 0.0f};
  float src = len_out <= 1 ? 0.0f
                           : __fdiv_rn(__fmul_rn(static_cast<float>(dst), static_cast<float>(len_in - 1)),
                                       static_cast<float>(len_out - 1));
  src = fminf(fmaxf(src, 0.0f), static_cast<float>(len_in - 1));
  int a = static_cast<int>(floorf(src));
  a = a < len_in - 1 ? a : len_in - 1;
  const int b = a + 1 < len_in - 1 ? a + 1 : len_in - 1;
  float f = b == a ? 0.0f : __fsub_rn(src, static_cast<float>(a));
  f = fminf(fmaxf(f, 0.0f), 1.0f);
  return {a, b, f};
}

// top = r0[x0](1 - fx) + r0[x1] fx, bot likewise, top (1 - fy) + bot fy
// (src/resample.rs:66-71)
__device__ __forceinline__ float blend(const float* __restrict__ plane, int iw, const Coord& y, const Coord& x) {
  const float gx = __fsub_rn(1.0f, x.f), gy = __fsub_rn(1.0f, y.f);
  const float* r0 = plane + static_cast<size_t>(y.i0) * iw;
  const float* r1 = plane + static_cast<size_t>(y.i1) * iw;
  const float top = __fadd_rn(__fmul_rn(__ldg(r0 + x.i0), gx), __fmul_rn(__ldg(r0 + x.i1), x.f));
  const float bot = __fadd_rn(__fmul_rn(__ldg(r1 + x.i0), gx), __fmul_rn(__ldg(r1 + x.i1), x.f));
  return __fadd_rn(__fmul_rn(top, gy), __fmul_rn(bot, y.f));
}

// One CTA per (64 columns of an output row, 8 channels): the row's source
// coordinate once, the thread's column once, then the channels' samples,
// unrolled so that their gathers are in flight together (stores coalesce
// along the row).
constexpr int RS_CH = 8, RS_X = 64;
template <bool AC>
__global__ void __launch_bounds__(RS_X) k_bilinear(const float* __restrict__ in, float* __restrict__ out, int c,
                                                   int ih, int iw, int oh, int ow) {
  const int x = blockIdx.x * RS_X + threadIdx.x, y = blockIdx.y;
  const int c0 = blockIdx.z * RS_CH;
  if (x >= ow) return;
  const Coord cy = AC ? ac_coord(y, ih, oh) : hp_coord(y, __fdiv_rn(static_cast<float>(ih), static_cast<float>(oh)), ih);
  const Coord cx = AC ? ac_coord(x, iw, ow) : hp_coord(x, __fdiv_rn(static_cast<float>(iw), static_cast<float>(ow)), iw);
#pragma unroll
  for (int k = 0; k < RS_CH; ++k) {
    const int ch = c0 + k;
    if (ch < c)
      out[(static_cast<size_t>(ch) * oh + y) * ow + x] = blend(in + static_cast<size_t>(ch) * ih * iw, iw, cy, cx);
  }
}

// ---------------------------------------------------------------- filter
// U = G g G^T, G = [1 0 0; 1/2 1/2 1/2; 1/2 -1/2 1/2; 0 0 1], stored
// [position][ic][oc] (src/conv.rs:136-160).
__global__ void k_winograd_filter(const float* __restrict__ w, float* __restrict__ u, int in_c, int out_c) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= in_c * out_c) return;
  const int oc = i / in_c, ic = i - oc * in_c;
  const float* g = w + static_cast<size_t>(i) * 9;
  float t[4][3];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const float a = g[j], b = g[3 + j], c = g[6 + j];
    t[0][j] = a;
    t[1][j] = __fmul_rn(0.5f, __fadd_rn(__fadd_rn(a, b), c));
    t[2][j] = __fmul_rn(0.5f, __fadd_rn(__fsub_rn(a, b), c));
    t[3][j] = c;
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const float a = t[r][0], b = t[r][1], c = t[r][2];
    const float v[4] = {a, __fmul_rn(0.5f, __fadd_rn(__fadd_rn(a, b), c)),
                        __fmul_rn(0.5f, __fadd_rn(__fsub_rn(a, b), c)), c};
#pragma unroll
    for (int k = 0; k < 4; ++k) u[(static_cast<size_t>(r * 4 + k) * in_c + ic) * out_c + oc] = v[k];
  }
}

}  // namespace

namespace {

// ---------------------------------------------------------------- conv
constexpr int CT = 32;                 // 2x2 output tiles per CTA
constexpr int CO = 32;                 // output channels per CTA
constexpr int KC = 16;                 // input channels per shared-memory slice
constexpr int PV = KC * CT + 4;        // floats per position plane of V (padded: no bank clash across planes)
constexpr int PU = KC * CO + 4;        // likewise for U
constexpr int PM = CT * (CO + 1);      // per position plane of the products
constexpr int CONV_THREADS = 256;      // 16 positions x (4 tile groups x 4 channel groups)
constexpr int TBY = 4, TBX = 8;        // the CTA's tiles: 4 rows x 8 columns (CT)
constexpr int PR = 2 * TBY + 2, PC = 2 * TBX + 2;  // its input patch: 10 x 18 samples per channel
constexpr int A_FLOATS = 16 * PM > 16 * (PV + PU) ? 16 * PM : 16 * (PV + PU);
enum { CONV_PLAIN = 0, CONV_RELU = 1, CONV_RESIZE_AC = 2 };
template <int MODE>
constexpr size_t conv_smem() {  // the resized patch and its coordinates only where the resize is fused
  return sizeof(float) * A_FLOATS + (MODE == CONV_RESIZE_AC ? sizeof(float) * KC * PR * PC + sizeof(int4) * (PR + PC) : 0);
}
static_assert(TBY * TBX == CT, "tile block");


// The input transform B^T d B of one 4x4 patch (src/conv.rs:382-405).
__device__ __forceinline__ void input_transform(const float (&d)[16], float (&v)[16]) {
  float col[16];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float a = d[j], b = d[4 + j], c = d[8 + j], e = d[12 + j];
    col[j] = __fsub_rn(a, c);
    col[4 + j] = __fadd_rn(b, c);
    col[8 + j] = __fsub_rn(c, b);
    col[12 + j] = __fsub_rn(b, e);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a = col[i * 4], b = col[i * 4 + 1], c = col[i * 4 + 2], e = col[i * 4 + 3];
    v[i * 4] = __fsub_rn(a, c);
    v[i * 4 + 1] = __fadd_rn(b, c);
    v[i * 4 + 2] = __fsub_rn(c, b);
    v[i * 4 + 3] = __fsub_rn(b, e);
  }
}

// input [images][in_c][ih][iw]; out [images][out_c][oh][ow] (oh, ow = ih, iw
// unless MODE is CONV_RESIZE_AC); add [in_c][oh][ow] or null; u
// [16][in_c][out_c]; bias [out_c] or null.
template <int MODE>
__global__ void __launch_bounds__(CONV_THREADS) k_conv3x3_wino(const float* __restrict__ input,
                                                               const float* __restrict__ add,
                                                               const float* __restrict__ u,
                                                               const float* __restrict__ bias, float* __restrict__ out,
                                                               int in_c, int ih, int iw, int oh, int ow, int out_c) {
  extern __shared__ float4 smem4[];
  float* sV = reinterpret_cast<float*>(smem4);
  float* sU = sV + 16 * PV;
  float* sM = sV;                 // reused after the last slice
  float* sIn = sV + A_FLOATS;     // [KC][PR][PC] input patch of the slice
  int4* sCoord = reinterpret_cast<int4*>(sIn + KC * PR * PC);  // resize: rows [PR], then columns [PC]
  const int tid = threadIdx.x;
  const int tiles_x = (ow + 1) / 2, tiles_y = (oh + 1) / 2;
  const int nbx = (tiles_x + TBX - 1) / TBX;
  const int bty = (blockIdx.x / nbx) * TBY, btx = (blockIdx.x % nbx) * TBX;  // first tile row / column
  const int py0 = bty * 2 - 1, px0 = btx * 2 - 1;                            // patch origin (pad 1)
  const int oc0 = blockIdx.y * CO;
  const float* in_img = input + static_cast<size_t>(blockIdx.z) * in_c * ih * iw;
  if constexpr (MODE == CONV_RESIZE_AC) {
    // source coordinates of the patch's rows and columns (align corners)
    if (tid < PR + PC) {
      const bool row = tid < PR;
      const int d = row ? py0 + tid : px0 + tid - PR;
      const int lim = row ? oh : ow;
      const Coord c = row ? ac_coord(min(max(d, 0), lim - 1), ih, oh) : ac_coord(min(max(d, 0), lim - 1), iw, ow);
      sCoord[tid] = make_int4(c.i0, c.i1, __float_as_int(c.f), 0);
    }
  }

  // this thread's tile for the input transform (fixed across slices)
  const int tt = tid & (CT - 1);
  const int tyl = tt / TBX, txl = tt % TBX;
  const bool tile_ok = bty + tyl < tiles_y && btx + txl < tiles_x;
  const int oy0 = py0 + 2 * tyl, ox0 = px0 + 2 * txl;  // the tile's 4x4 patch origin

  // products: position p, tiles [tg * 8, +8), channels [og * 8, +8)
  const int p = tid >> 4, tg = (tid >> 2) & 3, og = tid & 3;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

  for (int ic0 = 0; ic0 < in_c; ic0 += KC) {
    __syncthreads();  // the previous slice has been consumed
    if constexpr (MODE == CONV_RESIZE_AC) {
      // the slice's resized patch, each sample computed once; zero padding
#pragma unroll 4
      for (int e = tid; e < KC * PR * PC; e += CONV_THREADS) {
        const int icl = e / (PR * PC), r = (e / PC) % PR, c = e % PC;
        const int ic = ic0 + icl, y = py0 + r, x = px0 + c;
        float s = 0.0f;
        if (ic < in_c && y >= 0 && y < oh && x >= 0 && x < ow) {
          const int4 a = sCoord[r], b = sCoord[PR + c];
          s = __fadd_rn(blend(in_img + static_cast<size_t>(ic) * ih * iw, iw, Coord{a.x, a.y, __int_as_float(a.z)},
                              Coord{b.x, b.y, __int_as_float(b.z)}),
                        add ? __ldg(add + (static_cast<size_t>(ic) * oh + y) * ow + x) : 0.0f);
        }
        sIn[e] = s;
      }
      __syncthreads();
    }
    // V of (tile tt, channels ic0 + icl) for icl = tid / 32 + {0, 8}
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int icl = (tid >> 5) + h * 8, ic = ic0 + icl;
      float d[16];
      if constexpr (MODE == CONV_RESIZE_AC) {
        const float* src = sIn + icl * PR * PC + (2 * tyl) * PC + 2 * txl;
#pragma unroll
        for (int dy = 0; dy < 4; ++dy)
#pragma unroll
          for (int dx = 0; dx < 4; ++dx) d[dy * 4 + dx] = src[dy * PC + dx];
      } else {
#pragma unroll
        for (int k = 0; k < 16; ++k) d[k] = 0.0f;
        if (ic < in_c) {
          const float* plane = in_img + static_cast<size_t>(ic) * ih * iw;
#pragma unroll
          for (int dy = 0; dy < 4; ++dy) {
            const int y = oy0 + dy;
            if (y < 0 || y >= oh) continue;
#pragma unroll
            for (int dx = 0; dx < 4; ++dx) {
              const int x = ox0 + dx;
              if (x < 0 || x >= ow) continue;
              float s = __ldg(plane + static_cast<size_t>(y) * iw + x);
              if constexpr (MODE == CONV_RELU) s = fmaxf(s, 0.0f);
              d[dy * 4 + dx] = s;
            }
          }
        }
      }
      float v[16];
      input_transform(d, v);
#pragma unroll
      for (int q = 0; q < 16; ++q) sV[q * PV + icl * CT + tt] = v[q];
    }
    // U slice [16][KC][CO]
#pragma unroll 4
    for (int e = tid; e < 16 * KC * CO; e += CONV_THREADS) {
      const int o = e & (CO - 1), k = (e / CO) & (KC - 1), q = e / (CO * KC);
      const int ic = ic0 + k, oc = oc0 + o;
      sU[q * PU + k * CO + o] =
          (ic < in_c && oc < out_c) ? __ldg(u + (static_cast<size_t>(q) * in_c + ic) * out_c + oc) : 0.0f;
    }
    __syncthreads();
    const float* vp = sV + p * PV + tg * 8;
    const float* up = sU + p * PU + og * 8;
#pragma unroll 4
    for (int k = 0; k < KC; ++k) {
      const float4 a0 = *reinterpret_cast<const float4*>(vp + k * CT);
      const float4 a1 = *reinterpret_cast<const float4*>(vp + k * CT + 4);
      const float4 b0 = *reinterpret_cast<const float4*>(up + k * CO);
      const float4 b1 = *reinterpret_cast<const float4*>(up + k * CO + 4);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) sM[p * PM + (tg * 8 + i) * (CO + 1) + og * 8 + j] = acc[i][j];
  __syncthreads();

  // output transform A^T M A + bias (src/conv.rs:440-481)
  float* out_img = out + static_cast<size_t>(blockIdx.z) * out_c * oh * ow;
#pragma unroll 1
  for (int q = 0; q < CO / 8; ++q) {
    const int o = (tid >> 5) + q * 8, oc = oc0 + o;
    if (!tile_ok || oc >= out_c) continue;
    float m[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) m[k] = sM[k * PM + tt * (CO + 1) + o];
    float r[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      r[j] = __fadd_rn(__fadd_rn(m[j], m[4 + j]), m[8 + j]);
      r[4 + j] = __fsub_rn(__fsub_rn(m[4 + j], m[8 + j]), m[12 + j]);
    }
    const float b = bias ? __ldg(bias + oc) : 0.0f;
    const float val[4] = {__fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), r[2]), b),
                          __fadd_rn(__fsub_rn(__fsub_rn(r[1], r[2]), r[3]), b),
                          __fadd_rn(__fadd_rn(__fadd_rn(r[4], r[5]), r[6]), b),
                          __fadd_rn(__fsub_rn(__fsub_rn(r[5], r[6]), r[7]), b)};
    float* plane = out_img + static_cast<size_t>(oc) * oh * ow;
#pragma unroll
    for (int dy = 0; dy < 2; ++dy)
#pragma unroll
      for (int dx = 0; dx < 2; ++dx) {
        const int y = oy0 + 1 + dy, x = ox0 + 1 + dx;
        if (y < oh && x < ow) plane[static_cast<size_t>(y) * ow + x] = val[dy * 2 + dx];
      }
  }
}

constexpr size_t DIM_MAX = size_t(1) << 20;

}  // namespace

// ---------------------------------------------------------------- C ABI
extern "C" int vk_token_to_chw_f32_batched(vk_ctx* ctx, const float* token_major, size_t images, size_t tokens,
                                           size_t channels, float* chw) {
  if (!ctx) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_token_to_chw_f32: NULL context");
  cudaSetDevice(ctx->device);
  if (!token_major || !chw) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_token_to_chw_f32: NULL buffer");
  if (tokens == 0 || channels == 0 || tokens * channels >= (size_t(1) << 31) || channels > (size_t(1) << 21))
    return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_token_to_chw_f32: tokens=%zu channels=%zu out of range", tokens,
                   channels);
  if (images > 65535) return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_token_to_chw_f32: more than 65535 images");
  if (images == 0) return VK_OK;
  const dim3 grid(static_cast<unsigned>((tokens + 31) / 32), static_cast<unsigned>((channels + 31) / 32),
                  static_cast<unsigned>(images));
  k_token_to_chw<<<grid, DT_THREADS, 0, ctx->stream>>>(token_major, chw, static_cast<int>(tokens),
                                                       static_cast<int>(channels));
  return vk_cuda_status(cudaGetLastError(), "vk_token_to_chw_f32");
}

extern "C" int vk_token_to_chw_f32(vk_ctx* ctx, const float* token_major, size_t tokens, size_t channels, float* chw) {
  return vk_token_to_chw_f32_batched(ctx, token_major, 1, tokens, channels, chw);
}

static int resize_impl(vk_ctx* ctx, const float* input, size_t c, size_t ih, size_t iw, size_t oh, size_t ow,
                       float* out, bool ac, const char* name) {
  if (!ctx) return vk_fail(VK_ERR_INVALID_ARGUMENT, "%s: NULL context", name);
  cudaSetDevice(ctx->device);
  if (c == 0 || ih == 0 || iw == 0 || oh == 0 || ow == 0) return VK_OK;  // the reference returns early
  if (!input || !out) return vk_fail(VK_ERR_INVALID_ARGUMENT, "%s: NULL buffer", name);
  if (ih > DIM_MAX || iw > DIM_MAX || oh > DIM_MAX || ow > DIM_MAX || c > DIM_MAX)
    return vk_fail(VK_UNSUPPORTED_SHAPE, "%s: dimension above 2^20", name);
  const dim3 grid(static_cast<unsigned>((ow + RS_X - 1) / RS_X), static_cast<unsigned>(oh),
                  static_cast<unsigned>((c + RS_CH - 1) / RS_CH));
  if (grid.y > 65535 || grid.z > 65535) return vk_fail(VK_UNSUPPORTED_SHAPE, "%s: oh or channels out of range", name);
  if (ac)
    k_bilinear<true><<<grid, RS_X, 0, ctx->stream>>>(input, out, (int)c, (int)ih, (int)iw, (int)oh, (int)ow);
  else
    k_bilinear<false><<<grid, RS_X, 0, ctx->stream>>>(input, out, (int)c, (int)ih, (int)iw, (int)oh, (int)ow);
  return vk_cuda_status(cudaGetLastError(), name);
}

extern "C" int vk_bilinear_resize_f32(vk_ctx* ctx, const float* input, size_t c, size_t ih, size_t iw, size_t oh,
                                      size_t ow, float* out) {
  return resize_impl(ctx, input, c, ih, iw, oh, ow, out, false, "vk_bilinear_resize_f32");
}

extern "C" int vk_bilinear_resize_align_corners_f32(vk_ctx* ctx, const float* input, size_t c, size_t ih, size_t iw,
                                                    size_t oh, size_t ow, float* out) {
  return resize_impl(ctx, input, c, ih, iw, oh, ow, out, true, "vk_bilinear_resize_align_corners_f32");
}

extern "C" int vk_conv3x3_prepare(vk_ctx* ctx, const float* weight_host, size_t in_c, size_t out_c, vk_conv3x3** out) {
  if (!ctx) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_conv3x3_prepare: NULL context");
  cudaSetDevice(ctx->device);
  if (!weight_host || !out) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_conv3x3_prepare: NULL argument");
  *out = nullptr;
  if (in_c == 0 || out_c == 0 || in_c * out_c > (size_t(1) << 26))
    return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_conv3x3_prepare: in_c=%zu out_c=%zu", in_c, out_c);
  const size_t wn = out_c * in_c * 9;
  float* w = nullptr;
  vk_conv3x3* cv = new vk_conv3x3();
  cv->device = ctx->device;
  cv->in_c = in_c;
  cv->out_c = out_c;
  cudaError_t e = cudaMalloc(&w, wn * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&cv->u, 16 * in_c * out_c * sizeof(float));
  if (e == cudaSuccess) e = cudaMemcpyAsync(w, weight_host, wn * sizeof(float), cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) {
    const int n = static_cast<int>(in_c * out_c);
    k_winograd_filter<<<(n + DT_THREADS - 1) / DT_THREADS, DT_THREADS, 0, ctx->stream>>>(w, cv->u, (int)in_c,
                                                                                          (int)out_c);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (w) cudaFree(w);
  if (e != cudaSuccess) {
    if (cv->u) cudaFree(cv->u);
    delete cv;
    return vk_cuda_status(e, "vk_conv3x3_prepare");
  }
  *out = cv;
  return VK_OK;
}

extern "C" int vk_conv3x3_release(vk_conv3x3* conv) {
  if (!conv) return VK_OK;
  cudaSetDevice(conv->device);
  if (conv->u) cudaFree(conv->u);
  delete conv;
  return VK_OK;
}

template <int MODE>
static int conv_launch(vk_ctx* ctx, const vk_conv3x3* cv, size_t images, const float* input, size_t ih, size_t iw,
                       size_t oh, size_t ow, const float* add, const float* bias, float* out, const char* name) {
  const size_t blocks = ((oh + 1) / 2 + TBY - 1) / TBY * (((ow + 1) / 2 + TBX - 1) / TBX);
  const void* fn = reinterpret_cast<const void*>(k_conv3x3_wino<MODE>);
  VK_TRY_CUDA(ensure_smem_limit(fn, static_cast<int>(conv_smem<MODE>())), name);
  const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>((cv->out_c + CO - 1) / CO),
                  static_cast<unsigned>(images));
  k_conv3x3_wino<MODE><<<grid, CONV_THREADS, conv_smem<MODE>(), ctx->stream>>>(input, add, cv->u, bias, out, (int)cv->in_c,
                                                                       (int)ih, (int)iw, (int)oh, (int)ow,
                                                                       (int)cv->out_c);
  return vk_cuda_status(cudaGetLastError(), name);
}

static int conv_check(vk_ctx* ctx, const vk_conv3x3* cv, size_t images, const float* input, size_t ih, size_t iw,
                      size_t oh, size_t ow, float* out, const char* name) {
  if (!ctx) return vk_fail(VK_ERR_INVALID_ARGUMENT, "%s: NULL context", name);
  cudaSetDevice(ctx->device);
  if (!cv || !input || !out) return vk_fail(VK_ERR_INVALID_ARGUMENT, "%s: NULL argument", name);
  if (cv->device != ctx->device) return vk_fail(VK_ERR_INVALID_ARGUMENT, "%s: filter of another device", name);
  if (images > 65535 || ih > DIM_MAX || iw > DIM_MAX || oh > DIM_MAX || ow > DIM_MAX ||
      cv->in_c * ih * iw >= (size_t(1) << 31) || cv->out_c * oh * ow >= (size_t(1) << 31))
    return vk_fail(VK_UNSUPPORTED_SHAPE, "%s: shape out of range", name);
  return VK_OK;
}

extern "C" int vk_conv3x3_forward_batched(vk_ctx* ctx, const vk_conv3x3* conv, size_t images, const float* input,
                                          size_t ih, size_t iw, const float* bias, int relu_input, float* out) {
  const char* name = "vk_conv3x3_forward";
  VK_TRY(conv_check(ctx, conv, images, input, ih, iw, ih, iw, out, name));
  if (images == 0 || ih == 0 || iw == 0) return VK_OK;
  return relu_input ? conv_launch<CONV_RELU>(ctx, conv, images, input, ih, iw, ih, iw, nullptr, bias, out, name)
                    : conv_launch<CONV_PLAIN>(ctx, conv, images, input, ih, iw, ih, iw, nullptr, bias, out, name);
}

extern "C" int vk_conv3x3_forward(vk_ctx* ctx, const vk_conv3x3* conv, const float* input, size_t in_c, size_t ih,
                                  size_t iw, size_t out_c, const float* bias, int relu_input, float* out) {
  if (conv && (in_c != conv->in_c || out_c != conv->out_c))
    return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_conv3x3_forward: in_c=%zu out_c=%zu, filter %zu -> %zu", in_c, out_c,
                   conv->in_c, conv->out_c);
  return vk_conv3x3_forward_batched(ctx, conv, 1, input, ih, iw, bias, relu_input, out);
}

extern "C" int vk_conv3x3_resize_ac_forward_batched(vk_ctx* ctx, const vk_conv3x3* conv, size_t images,
                                                    const float* input, size_t ih, size_t iw, size_t oh, size_t ow,
                                                    const float* add, const float* bias, float* out) {
  const char* name = "vk_conv3x3_resize_ac_forward";
  VK_TRY(conv_check(ctx, conv, images, input, ih, iw, oh, ow, out, name));
  if (images == 0 || oh == 0 || ow == 0) return VK_OK;
  if (ih == 0 || iw == 0) return vk_fail(VK_ERR_INVALID_ARGUMENT, "%s: empty input", name);
  return conv_launch<CONV_RESIZE_AC>(ctx, conv, images, input, ih, iw, oh, ow, add, bias, out, name);
}

extern "C" int vk_conv3x3_resize_ac_forward(vk_ctx* ctx, const vk_conv3x3* conv, const float* input, size_t in_c,
                                            size_t ih, size_t iw, size_t oh, size_t ow, const float* add,
                                            size_t out_c, const float* bias, float* out) {
  if (conv && (in_c != conv->in_c || out_c != conv->out_c))
    return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_conv3x3_resize_ac_forward: in_c=%zu out_c=%zu, filter %zu -> %zu",
                   in_c, out_c, conv->in_c, conv->out_c);
  return vk_conv3x3_resize_ac_forward_batched(ctx, conv, 1, input, ih, iw, oh, ow, add, bias, out);
}
