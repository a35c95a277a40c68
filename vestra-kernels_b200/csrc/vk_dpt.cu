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
// The convolution (f32 math) is one kernel per (4 x 8 tiles of 2x2 outputs,
// 32 output channels).  Per 16-channel slice it builds the transformed input
// V = B^T d B of its tiles in shared memory (ReLU on the samples where
// asked), stages the matching slice of the prepared filter U, and
// accumulates the 16 transform-domain products M_p = V_p U_p in registers:
// each thread owns one of the 16 positions for 8 tiles x 8 channels.  The
// output transform A^T M A then runs from shared memory and writes the 2x2
// outputs with the bias.  bf16 math runs the products on the tensor cores
// (k_conv3x3_wino_tc below).  The resize-fused form resizes (and adds) into
// the context workspace with the resize kernel, then convolves.
#include "vestra_b200.h"
#include "vk_abi_internal.h"
#include "vk_common.cuh"
#include "vk_internal.h"

using namespace vk;

struct vk_conv3x3 {
  int device = 0;
  int math = VK_MATH_F32;
  size_t in_c = 0, out_c = 0;
  float* u = nullptr;           // f32 math: [16][in_c][out_c]
  __nv_bfloat16* ub = nullptr;  // bf16 math: [out_c / 32][in_c / 16][16][32 x 16 core-matrix tile]
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

// One CTA per (64 columns of an output row, 8 channels): the source
// coordinates and the four neighbour offsets once per thread, then the
// channels' samples by pointer increments (unrolled, so that several
// channels' gathers are in flight together; stores coalesce along the row).
constexpr int RS_CH = 8, RS_X = 64;
template <bool AC>
__global__ void __launch_bounds__(RS_X) k_bilinear(const float* __restrict__ in, float* __restrict__ out, int c,
                                                   int ih, int iw, int oh, int ow, const float* __restrict__ add,
                                                   int add_c) {
  const int x = blockIdx.x * RS_X + threadIdx.x, y = blockIdx.y;
  const int c0 = blockIdx.z * RS_CH;
  if (x >= ow) return;
  const Coord cy = AC ? ac_coord(y, ih, oh) : hp_coord(y, __fdiv_rn(static_cast<float>(ih), static_cast<float>(oh)), ih);
  const Coord cx = AC ? ac_coord(x, iw, ow) : hp_coord(x, __fdiv_rn(static_cast<float>(iw), static_cast<float>(ow)), iw);
  const int o00 = cy.i0 * iw + cx.i0, o01 = cy.i0 * iw + cx.i1, o10 = cy.i1 * iw + cx.i0, o11 = cy.i1 * iw + cx.i1;
  const float gx = __fsub_rn(1.0f, cx.f), gy = __fsub_rn(1.0f, cy.f);
  const size_t in_plane = static_cast<size_t>(ih) * iw, out_plane = static_cast<size_t>(oh) * ow;
  const float* src = in + c0 * in_plane;
  float* dst = out + c0 * out_plane + static_cast<size_t>(y) * ow + x;
  const int n = min(RS_CH, c - c0);
  const int yx = y * ow + x;
#pragma unroll
  for (int k = 0; k < RS_CH; ++k) {
    if (k >= n) break;
    // top = r0[x0](1 - fx) + r0[x1] fx, bot likewise, top (1 - fy) + bot fy (src/resample.rs:66-71)
    const float top = __fadd_rn(__fmul_rn(__ldg(src + o00), gx), __fmul_rn(__ldg(src + o01), cx.f));
    const float bot = __fadd_rn(__fmul_rn(__ldg(src + o10), gx), __fmul_rn(__ldg(src + o11), cx.f));
    float v = __fadd_rn(__fmul_rn(top, gy), __fmul_rn(bot, cy.f));
    if (add) v = __fadd_rn(v, __ldg(add + ((c0 + k) % add_c) * out_plane + yx));  // shared per image
    *dst = v;
    src += in_plane;
    dst += out_plane;
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
constexpr int A_FLOATS = 16 * PM > 16 * (PV + PU) ? 16 * PM : 16 * (PV + PU);  // V + U slices, then M
enum { CONV_PLAIN = 0, CONV_RELU = 1 };
constexpr size_t CONV_SMEM = sizeof(float) * A_FLOATS;
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

// input [images][in_c][h][w]; out [images][out_c][h][w]; u [16][in_c][out_c];
// bias [out_c] or null.
template <int MODE>
__global__ void __launch_bounds__(CONV_THREADS) k_conv3x3_wino(const float* __restrict__ input,
                                                               const float* __restrict__ u,
                                                               const float* __restrict__ bias, float* __restrict__ out,
                                                               int in_c, int ih, int iw, int oh, int ow, int out_c) {
  extern __shared__ float4 smem4[];
  float* sV = reinterpret_cast<float*>(smem4);
  float* sU = sV + 16 * PV;
  float* sM = sV;                 // reused after the last slice
  const int tid = threadIdx.x;
  const int tiles_x = (ow + 1) / 2, tiles_y = (oh + 1) / 2;
  const int nbx = (tiles_x + TBX - 1) / TBX;
  const int bty = (blockIdx.x / nbx) * TBY, btx = (blockIdx.x % nbx) * TBX;  // first tile row / column
  const int py0 = bty * 2 - 1, px0 = btx * 2 - 1;                            // patch origin (pad 1)
  const int oc0 = blockIdx.y * CO;
  const float* in_img = input + static_cast<size_t>(blockIdx.z) * in_c * ih * iw;

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
    // V of (tile tt, channels ic0 + icl) for icl = tid / 32 + {0, 8}
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int icl = (tid >> 5) + h * 8, ic = ic0 + icl;
      float d[16];
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

// ---------------------------------------------------------------- conv on the tensor cores (bf16 math)
// The 16 position products M_p = V_p U_p run as tcgen05 MMAs: per CTA 128
// tiles (M) x 32 output channels (N) x 16 positions, accumulated in TMEM
// (16 x 32 = all 512 columns).  K runs over 16-channel slices: 256 worker
// threads build the slice's V (bf16, core-matrix K-major layout) in shared
// memory, while one thread streams the prepared bf16 U slices in with bulk
// copies and issues the 16 MMAs of the previous slice.  The epilogue reads
// each tile row's 16 positions from TMEM and applies A^T M A in registers.
namespace {

constexpr int TM = 128;                      // tiles per CTA (MMA M)
constexpr int TN = 32;                       // output channels per CTA (MMA N)
constexpr int TK = 16;                       // input channels per slice (MMA K)
#ifndef VK_CONV_TC_WORKERS
#define VK_CONV_TC_WORKERS 512
#endif
constexpr int TC_WORKERS = VK_CONV_TC_WORKERS;  // transform / epilogue threads (256 or 512)
constexpr int KPT = TK * TM / TC_WORKERS;       // input channels per worker per slice (8 or 4)
constexpr int CPW = TN * 4 * 32 / TC_WORKERS;   // epilogue columns per worker warp (16 or 8)
static_assert(KPT == 8 || KPT == 4, "workers");
constexpr int TC_THREADS = TC_WORKERS + 32;  // + the MMA and copy warp
constexpr int A_POS = TM * TK * 2;           // 4 KB: one position's V slice
constexpr int B_POS = TN * TK * 2;           // 1 KB: one position's U slice
constexpr int A_SLICE = 16 * A_POS, B_SLICE = 16 * B_POS;
constexpr size_t TC_SMEM = 1024 + 2 * (A_SLICE + B_SLICE) + 128;

// K-major operand without swizzle: core matrices of 8 rows x 16 bytes; the
// two along K (a 16-element slice) are 128 bytes apart (LBO), 8-row groups
// 256 bytes apart (SBO).  Row r, element k at (r/8)*256 + (k/8)*128 + (r%8)*16 + (k%8)*2.
__device__ __forceinline__ uint64_t desc_kmajor_core(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(128u >> 4) << 16;  // LBO
  d |= static_cast<uint64_t>(256u >> 4) << 32;  // SBO
  d |= static_cast<uint64_t>(1u) << 46;         // sm_100 descriptor version; layout 0 = no swizzle
  return d;
}
__host__ __device__ constexpr int core_offset(int r, int k) { return (r / 8) * 256 + (k / 8) * 128 + (r % 8) * 16 + (k % 8) * 2; }

// plain bulk copy global -> shared (no tensor map, no multicast)
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// U f32 [16][in_c][out_c] -> bf16 [out_c / 32][slices][16 positions][32 x 16 core-matrix tile], zero-padded
__global__ void k_pack_u_bf16(const float* __restrict__ u, __nv_bfloat16* __restrict__ ub, int in_c, int out_c,
                              int slices, int ocb) {
  const size_t total = static_cast<size_t>(ocb) * slices * 16 * TN * TK;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int k = static_cast<int>(i % TK), n = static_cast<int>((i / TK) % TN);
    const int p = static_cast<int>((i / (TK * TN)) % 16);
    const size_t sb = i / (TK * TN * 16);
    const int s = static_cast<int>(sb % slices), b = static_cast<int>(sb / slices);
    const int ic = s * TK + k, oc = b * TN + n;
    const float v = (ic < in_c && oc < out_c) ? u[(static_cast<size_t>(p) * in_c + ic) * out_c + oc] : 0.0f;
    ub[sb * (16 * TN * TK) + p * (TN * TK) + core_offset(n, k) / 2] = __float2bfloat16_rn(v);
  }
}

template <int MODE>
__global__ void __launch_bounds__(TC_THREADS, 1)
    k_conv3x3_wino_tc(const float* __restrict__ input, const __nv_bfloat16* __restrict__ ub, const float* __restrict__ bias, float* __restrict__ out,
                      int in_c, int ih, int iw, int oh, int ow, int out_c, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                   // [2][16][4 KB]
  uint8_t* sB = smem + 2 * A_SLICE;     // [2][16][1 KB]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + 2 * B_SLICE);
  uint64_t* a_full = bars;              // [2] count TC_WORKERS
  uint64_t* b_full = bars + 2;          // [2] U slice landed
  uint64_t* ab_free = bars + 4;         // [2] the slice's MMAs finished
  uint64_t* acc_done = bars + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 7);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int slices = (in_c + TK - 1) / TK;
  const int tiles_x = (ow + 1) / 2, tiles_y = (oh + 1) / 2;
  const int ocb = blockIdx.y, oc0 = ocb * TN;
  const float* in_img = input + static_cast<size_t>(blockIdx.z) * in_c * ih * iw;
  const __nv_bfloat16* ub_blk = ub + static_cast<size_t>(ocb) * slices * (16 * TN * TK);

  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&a_full[b], TC_WORKERS);
      mbar_init(&b_full[b], 1);
      mbar_init(&ab_free[b], 1);
    }
    mbar_init(acc_done, 1);
    fence_mbar_init();
  }
  if (warp == TC_WORKERS / 32) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == TC_WORKERS / 32) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(TM, TN);
      auto load_u = [&](int s) {
        mbar_arrive_expect_tx(&b_full[s & 1], B_SLICE);
        bulk_load(sB + (s & 1) * B_SLICE, ub_blk + static_cast<size_t>(s) * (16 * TN * TK), B_SLICE, &b_full[s & 1]);
      };
      load_u(0);
      if (slices > 1) load_u(1);
      for (int s = 0; s < slices && ok; ++s) {
        const int b = s & 1;
        const uint32_t ph = (s >> 1) & 1;
        if (!(ok = mbar_wait(&b_full[b], ph, err, VK_DEV_TIMEOUT_MMA))) break;
        if (!(ok = mbar_wait(&a_full[b], ph, err, VK_DEV_TIMEOUT_MMA))) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + b * A_SLICE), b0 = smem_u32(sB + b * B_SLICE);
#pragma unroll
        for (int p = 0; p < 16; ++p)
          umma_f16(tmem + p * TN, desc_kmajor_core(a0 + p * A_POS), desc_kmajor_core(b0 + p * B_POS), idesc,
                   s > 0 ? 1u : 0u);
        umma_commit(&ab_free[b]);
        if (s + 2 < slices) {
          if (!(ok = mbar_wait(&ab_free[b], ph, err, VK_DEV_TIMEOUT_MMA))) break;  // this slice's MMAs read sB[b]
          load_u(s + 2);
        }
      }
      umma_commit(acc_done);
    }
  } else {
    // ---- V slices: thread (tile row m, channel group kh of KPT); the CTA takes 128
    // consecutive tiles in row-major order (rows of consecutive tiles load
    // best straight from global memory; L1 serves the patches' overlap)
    const int m = tid & (TM - 1), kh = tid / TM;
    const int lin_t = blockIdx.x * TM + m;
    const bool lin_ok = lin_t < tiles_x * tiles_y;
    const int lin_ty = lin_ok ? lin_t / tiles_x : 0, lin_tx = lin_ok ? lin_t % tiles_x : 0;
    // the 4x4 patch's offsets in a channel plane (clamped into it) and which samples are inside
    int roff[4], coff[4];
    uint32_t inside = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int y = lin_ty * 2 - 1 + k, x = lin_tx * 2 - 1 + k;
      roff[k] = min(max(y, 0), oh - 1) * iw;
      coff[k] = min(max(x, 0), ow - 1);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int yj = lin_ty * 2 - 1 + j;
        inside |= static_cast<uint32_t>(lin_ok && yj >= 0 && yj < oh && x >= 0 && x < ow) << (j * 4 + k);
      }
    }
    const size_t plane_sz = static_cast<size_t>(ih) * iw;
    for (int s = 0; s < slices && ok; ++s) {
      const int b = s & 1;
      uint32_t packed[16][KPT / 2];
#pragma unroll
      for (int pr = 0; pr < KPT / 2; ++pr) {  // channel pairs of this thread's KPT
        float v2[2][16];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int icl = kh * KPT + pr * 2 + e;
          float d[16];
          const int ic = s * TK + icl;
          const uint32_t live = ic < in_c ? inside : 0u;
          const float* plane = in_img + (ic < in_c ? ic : 0) * plane_sz;
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            float v = __ldg(plane + roff[k >> 2] + coff[k & 3]);  // always inside the plane; zero outside the image
            if constexpr (MODE == CONV_RELU) v = fmaxf(v, 0.0f);
            d[k] = (live >> k) & 1u ? v : 0.0f;
          }
          input_transform(d, v2[e]);
        }
#pragma unroll
        for (int p = 0; p < 16; ++p) packed[p][pr] = pack_bf16x2(v2[0][p], v2[1][p]);
      }
      // the slice's A buffer is free once the MMAs of slice s - 2 have finished
      if (s >= 2 && !(ok = mbar_wait(&ab_free[b], ((s >> 1) - 1) & 1, err, VK_DEV_TIMEOUT_OTHER))) break;
      uint8_t* a = sA + b * A_SLICE + core_offset(m, kh * KPT);
#pragma unroll
      for (int p = 0; p < 16; ++p) {
        if constexpr (KPT == 8)
          *reinterpret_cast<uint4*>(a + p * A_POS) =
              make_uint4(packed[p][0], packed[p][1 % (KPT / 2)], packed[p][2 % (KPT / 2)], packed[p][3 % (KPT / 2)]);
        else
          *reinterpret_cast<uint2*>(a + p * A_POS) = make_uint2(packed[p][0], packed[p][1]);
      }
      fence_proxy_async();  // generic-proxy stores -> visible to the tensor core
      mbar_arrive(&a_full[b]);
    }
    // ---- epilogue: warp w reads lanes (tiles) of quarter w % 4, channels [CPW (w / 4), +CPW)
    if (ok && (ok = mbar_wait(acc_done, 0, err, VK_DEV_TIMEOUT_EPILOGUE))) {
      tc_fence_after();
      const int q = warp & 3, chh = warp >> 2;
      const int mt = q * 32 + lane;
      const int lt = blockIdx.x * TM + mt;
      const int ty = lt / tiles_x, tx = lt % tiles_x;
      float acc[4][CPW];
#pragma unroll
      for (int o = 0; o < 4; ++o)
#pragma unroll
        for (int c = 0; c < CPW; ++c) acc[o][c] = 0.0f;
      constexpr float AT[2][4] = {{1.f, 1.f, 1.f, 0.f}, {0.f, 1.f, -1.f, -1.f}};
#pragma unroll
      for (int p = 0; p < 16; ++p) {
        uint32_t r[CPW];
        if constexpr (CPW == 16)
          tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + p * TN + chh * CPW,
                    *reinterpret_cast<uint32_t(*)[16]>(&r[0]));
        else
          tmem_ld8(tmem + (static_cast<uint32_t>(q * 32) << 16) + p * TN + chh * CPW,
                   *reinterpret_cast<uint32_t(*)[8]>(&r[0]));
        tmem_wait_ld();
        const int i = p >> 2, j = p & 3;
#pragma unroll
        for (int dy = 0; dy < 2; ++dy)
#pragma unroll
          for (int dx = 0; dx < 2; ++dx) {
            const float cf = AT[dy][i] * AT[dx][j];
            if (cf == 0.0f) continue;
#pragma unroll
            for (int c = 0; c < CPW; ++c)
              acc[dy * 2 + dx][c] = cf > 0.0f ? acc[dy * 2 + dx][c] + __uint_as_float(r[c])
                                              : acc[dy * 2 + dx][c] - __uint_as_float(r[c]);
          }
      }
      if (ty < tiles_y && tx < tiles_x) {
        const int ty0 = ty * 2, tx0 = tx * 2;
        float* out_img = out + static_cast<size_t>(blockIdx.z) * out_c * oh * ow;
#pragma unroll
        for (int c = 0; c < CPW; ++c) {
          const int oc = oc0 + chh * CPW + c;
          if (oc >= out_c) break;
          const float bb = bias ? __ldg(bias + oc) : 0.0f;
          float* plane = out_img + static_cast<size_t>(oc) * oh * ow;
#pragma unroll
          for (int dy = 0; dy < 2; ++dy)
#pragma unroll
            for (int dx = 0; dx < 2; ++dx) {
              const int y = ty0 + dy, x = tx0 + dx;
              if (y < oh && x < ow) plane[static_cast<size_t>(y) * ow + x] = acc[dy * 2 + dx][c] + bb;
            }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == TC_WORKERS / 32) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

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

// input [c][ih][iw] -> out [c][oh][ow]; add [add_c][oh][ow] (added to plane ch at ch % add_c) or null
static int resize_launch(vk_ctx* ctx, const float* input, size_t c, size_t ih, size_t iw, size_t oh, size_t ow,
                         const float* add, size_t add_c, float* out, bool ac, const char* name) {
  const dim3 grid(static_cast<unsigned>((ow + RS_X - 1) / RS_X), static_cast<unsigned>(oh),
                  static_cast<unsigned>((c + RS_CH - 1) / RS_CH));
  if (grid.y > 65535 || grid.z > 65535) return vk_fail(VK_UNSUPPORTED_SHAPE, "%s: oh or channels out of range", name);
  if (ac)
    k_bilinear<true><<<grid, RS_X, 0, ctx->stream>>>(input, out, (int)c, (int)ih, (int)iw, (int)oh, (int)ow, add,
                                                     (int)(add_c ? add_c : 1));
  else
    k_bilinear<false><<<grid, RS_X, 0, ctx->stream>>>(input, out, (int)c, (int)ih, (int)iw, (int)oh, (int)ow, add,
                                                      (int)(add_c ? add_c : 1));
  return vk_cuda_status(cudaGetLastError(), name);
}

static int resize_impl(vk_ctx* ctx, const float* input, size_t c, size_t ih, size_t iw, size_t oh, size_t ow,
                       float* out, bool ac, const char* name) {
  if (!ctx) return vk_fail(VK_ERR_INVALID_ARGUMENT, "%s: NULL context", name);
  cudaSetDevice(ctx->device);
  if (c == 0 || ih == 0 || iw == 0 || oh == 0 || ow == 0) return VK_OK;  // the reference returns early
  if (!input || !out) return vk_fail(VK_ERR_INVALID_ARGUMENT, "%s: NULL buffer", name);
  if (ih > DIM_MAX || iw > DIM_MAX || oh > DIM_MAX || ow > DIM_MAX || c > DIM_MAX)
    return vk_fail(VK_UNSUPPORTED_SHAPE, "%s: dimension above 2^20", name);
  return resize_launch(ctx, input, c, ih, iw, oh, ow, nullptr, 0, out, ac, name);
}

extern "C" int vk_bilinear_resize_f32(vk_ctx* ctx, const float* input, size_t c, size_t ih, size_t iw, size_t oh,
                                      size_t ow, float* out) {
  return resize_impl(ctx, input, c, ih, iw, oh, ow, out, false, "vk_bilinear_resize_f32");
}

extern "C" int vk_bilinear_resize_align_corners_f32(vk_ctx* ctx, const float* input, size_t c, size_t ih, size_t iw,
                                                    size_t oh, size_t ow, float* out) {
  return resize_impl(ctx, input, c, ih, iw, oh, ow, out, true, "vk_bilinear_resize_align_corners_f32");
}

extern "C" int vk_conv3x3_prepare_math(vk_ctx* ctx, const float* weight_host, size_t in_c, size_t out_c, int math,
                                       vk_conv3x3** out) {
  if (!ctx) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_conv3x3_prepare: NULL context");
  if (math != VK_MATH_F32 && math != VK_MATH_BF16)
    return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_conv3x3_prepare: math must be f32 or bf16");
  cudaSetDevice(ctx->device);
  if (!weight_host || !out) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_conv3x3_prepare: NULL argument");
  *out = nullptr;
  if (in_c == 0 || out_c == 0 || in_c * out_c > (size_t(1) << 26))
    return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_conv3x3_prepare: in_c=%zu out_c=%zu", in_c, out_c);
  const size_t wn = out_c * in_c * 9;
  float* w = nullptr;
  vk_conv3x3* cv = new vk_conv3x3();
  cv->device = ctx->device;
  cv->math = math;
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
  if (e == cudaSuccess && math == VK_MATH_BF16) {
    const int slices = static_cast<int>((in_c + TK - 1) / TK), ocb = static_cast<int>((out_c + TN - 1) / TN);
    const size_t n = static_cast<size_t>(ocb) * slices * 16 * TN * TK;
    e = cudaMalloc(&cv->ub, n * sizeof(__nv_bfloat16));
    if (e == cudaSuccess) {
      k_pack_u_bf16<<<static_cast<int>((n + DT_THREADS - 1) / DT_THREADS < 4096 ? (n + DT_THREADS - 1) / DT_THREADS : 4096),
                      DT_THREADS, 0, ctx->stream>>>(cv->u, cv->ub, (int)in_c, (int)out_c, slices, ocb);
      e = cudaGetLastError();
    }
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (w) cudaFree(w);
  if (e == cudaSuccess && cv->ub) {  // bf16 math keeps only the packed filter
    cudaFree(cv->u);
    cv->u = nullptr;
  }
  if (e != cudaSuccess) {
    if (cv->u) cudaFree(cv->u);
    if (cv->ub) cudaFree(cv->ub);
    delete cv;
    return vk_cuda_status(e, "vk_conv3x3_prepare");
  }
  *out = cv;
  return VK_OK;
}

extern "C" int vk_conv3x3_prepare(vk_ctx* ctx, const float* weight_host, size_t in_c, size_t out_c, vk_conv3x3** out) {
  return vk_conv3x3_prepare_math(ctx, weight_host, in_c, out_c, VK_MATH_F32, out);
}

extern "C" int vk_conv3x3_release(vk_conv3x3* conv) {
  if (!conv) return VK_OK;
  cudaSetDevice(conv->device);
  if (conv->u) cudaFree(conv->u);
  if (conv->ub) cudaFree(conv->ub);
  delete conv;
  return VK_OK;
}

template <int MODE>
static int conv_launch(vk_ctx* ctx, const vk_conv3x3* cv, size_t images, const float* input, size_t h, size_t w,
                       const float* bias, float* out, const char* name) {
  const size_t tiles = ((h + 1) / 2) * ((w + 1) / 2);
  if (cv->math == VK_MATH_BF16) {
    const void* fn = reinterpret_cast<const void*>(k_conv3x3_wino_tc<MODE>);
    VK_TRY_CUDA(ensure_smem_limit(fn, static_cast<int>(TC_SMEM)), name);
    const dim3 grid(static_cast<unsigned>((tiles + TM - 1) / TM), static_cast<unsigned>((cv->out_c + TN - 1) / TN),
                    static_cast<unsigned>(images));
    k_conv3x3_wino_tc<MODE><<<grid, TC_THREADS, TC_SMEM, ctx->stream>>>(input, cv->ub, bias, out, (int)cv->in_c,
                                                                        (int)h, (int)w, (int)h, (int)w,
                                                                        (int)cv->out_c, ctx->d_err);
    return vk_cuda_status(cudaGetLastError(), name);
  }
  const size_t blocks = ((h + 1) / 2 + TBY - 1) / TBY * (((w + 1) / 2 + TBX - 1) / TBX);
  const void* fn = reinterpret_cast<const void*>(k_conv3x3_wino<MODE>);
  VK_TRY_CUDA(ensure_smem_limit(fn, static_cast<int>(CONV_SMEM)), name);
  const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>((cv->out_c + CO - 1) / CO),
                  static_cast<unsigned>(images));
  k_conv3x3_wino<MODE><<<grid, CONV_THREADS, CONV_SMEM, ctx->stream>>>(input, cv->u, bias, out, (int)cv->in_c, (int)h,
                                                                       (int)w, (int)h, (int)w, (int)cv->out_c);
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
  return relu_input ? conv_launch<CONV_RELU>(ctx, conv, images, input, ih, iw, bias, out, name)
                    : conv_launch<CONV_PLAIN>(ctx, conv, images, input, ih, iw, bias, out, name);
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
  // The resized + added map goes through the context's workspace: a
  // high-occupancy resize kernel and then the plain convolution beat
  // resampling inside the convolution (whose few resident warps cannot hide
  // the gathers).  Same operations in the same order as the reference's
  // fused form, so the result is the one of resize, add, conv in sequence.
  const size_t planes = images * conv->in_c;
  VK_TRY(ctx_reserve(ctx, planes * oh * ow * sizeof(float)));
  float* mid = static_cast<float*>(ctx->ws);
  VK_TRY(resize_launch(ctx, input, planes, ih, iw, oh, ow, add, conv->in_c, mid, true, name));
  return conv_launch<CONV_PLAIN>(ctx, conv, images, mid, oh, ow, bias, out, name);
}

extern "C" int vk_conv3x3_resize_ac_forward(vk_ctx* ctx, const vk_conv3x3* conv, const float* input, size_t in_c,
                                            size_t ih, size_t iw, size_t oh, size_t ow, const float* add,
                                            size_t out_c, const float* bias, float* out) {
  if (conv && (in_c != conv->in_c || out_c != conv->out_c))
    return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_conv3x3_resize_ac_forward: in_c=%zu out_c=%zu, filter %zu -> %zu",
                   in_c, out_c, conv->in_c, conv->out_c);
  return vk_conv3x3_resize_ac_forward_batched(ctx, conv, 1, input, ih, iw, oh, ow, add, bias, out);
}
