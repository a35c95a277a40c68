// vk_elementwise.cu -- the HBM-bound kernels of the path: LayerNorm (with
// bf16 / Q8_0 output fused), RoPE, Q/K-norm+RoPE, Q8_0 quantisation and the
// stand-alone epilogue passes of the reference's f32 API.
//
// Reference functions restated (file:line in the vestra-kernels crate):
//   layernorm            src/scalar.rs:83-114
//   gelu / erf           src/scalar.rs:116-134, src/dispatch.rs:56-73
//   add                  src/dispatch.rs:77, src/scalar.rs:58-63
//   add_bias_rows        src/scalar.rs:65-81
//   layerscale           src/scalar.rs:139-155
//   rope2d               src/rope.rs:30-93
//   qk_norm_rope         src/specialized.rs:278-454
//   quantize_row_q8_0    src/q8_0_dot.rs:27-46
#include "vk_common.cuh"
#include "vk_internal.h"

namespace vk {

namespace {
constexpr int EW_THREADS = 256;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

inline int ew_grid(size_t n) {
  size_t g = (n + EW_THREADS - 1) / EW_THREADS;
  const size_t cap = static_cast<size_t>(num_sms()) * 16;
  return static_cast<int>(g < cap ? (g ? g : 1) : cap);
}
}  // namespace

// ---------------------------------------------------------------- LayerNorm
// One warp per row; the row stays in registers between the two passes (mean,
// then mean of squared deviations, as src/scalar.rs:99-110).  Output f32, bf16
// or Q8_0 blocks (amax over the 8 lanes that hold one 32-block).
template <int VPL>  // float4 vectors per lane; cols == VPL * 128
__global__ void __launch_bounds__(EW_THREADS)
    k_layernorm_vec(const float* __restrict__ x, float* y, __nv_bfloat16* yb, int8_t* yq, __half* yd,
                    int rows, int cols, const float* __restrict__ g, const float* __restrict__ b, float eps) {
  grid_dependency_wait();  // x from the previous kernel is visible from here
  // a small LayerNorm (at most 128 rows per SM: 16 images of 865 tokens)
  // lets the next GEMM set up on the SMs its blocks leave (64 rows per SM
  // before: 16 images went from 4,294-4,300 to 4,327-4,346 images/s)
  if (rows <= 128 * 148) grid_launch_dependents();
  // Rows run from the last to the first: the GEMM that wrote x finished with
  // its last rows, which are the ones still in L2.
  const int warp = rows - 1 - static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (warp < 0) return;
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(warp) * cols);
  float4 v[VPL];
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    v[j] = __ldg(xr + j * 32 + lane);
    s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
  }
  const float mean = warp_sum(s) / static_cast<float>(cols);
  float q = 0.0f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const float a = v[j].x - mean, bb = v[j].y - mean, c = v[j].z - mean, d = v[j].w - mean;
    q += (a * a + bb * bb) + (c * c + d * d);
  }
  const float var = warp_sum(q) / static_cast<float>(cols);
  const float inv = 1.0f / sqrtf(var + eps);
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int c0 = (j * 32 + lane) * 4;
    const float4 gg = __ldg(reinterpret_cast<const float4*>(g + c0));
    const float4 bt = __ldg(reinterpret_cast<const float4*>(b + c0));
    float4 o;
    o.x = (v[j].x - mean) * inv * gg.x + bt.x;
    o.y = (v[j].y - mean) * inv * gg.y + bt.y;
    o.z = (v[j].z - mean) * inv * gg.z + bt.z;
    o.w = (v[j].w - mean) * inv * gg.w + bt.w;
    const size_t off = static_cast<size_t>(warp) * cols + c0;
    if (y != nullptr) *reinterpret_cast<float4*>(y + off) = o;
    if (yb != nullptr) *reinterpret_cast<uint2*>(yb + off) = make_uint2(pack_bf16x2(o.x, o.y), pack_bf16x2(o.z, o.w));
    if (yq != nullptr) {
      // 8 consecutive lanes hold one 32-wide Q8_0 block.
      float amax = fmaxf(fmaxf(fabsf(o.x), fabsf(o.y)), fmaxf(fabsf(o.z), fabsf(o.w)));
#pragma unroll
      for (int m = 1; m < 8; m <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
      const float dd = amax / 127.0f;
      const float id = dd != 0.0f ? 1.0f / dd : 0.0f;
      char4 qq;
      qq.x = static_cast<signed char>(fminf(fmaxf(roundf(o.x * id), -127.0f), 127.0f));
      qq.y = static_cast<signed char>(fminf(fmaxf(roundf(o.y * id), -127.0f), 127.0f));
      qq.z = static_cast<signed char>(fminf(fmaxf(roundf(o.z * id), -127.0f), 127.0f));
      qq.w = static_cast<signed char>(fminf(fmaxf(roundf(o.w * id), -127.0f), 127.0f));
      *reinterpret_cast<char4*>(yq + off) = qq;
      if ((lane & 7) == 0) yd[off / 32] = __float2half_rn(dd);
    }
  }
}

// f32 output (the reference's layernorm operator and f32 math): bit-exact
// with scalar::layernorm (src/scalar.rs:83-114).  The row sum and the sum of
// squared deviations are left folds over ascending columns from -0.0 (Rust's
// f32 Sum), every product and sum separately rounded (no FMA contraction),
// inv = 1 / sqrt with IEEE division and square root, then
// (x - mean) * inv * g + b.  The fold is a serial chain per row, so one
// thread owns one row; its 128-byte lines stay in L1 between the passes.
__global__ void k_layernorm_exact(const float* __restrict__ x, float* y, int rows, int cols,
                                  const float* __restrict__ g, const float* __restrict__ b, float eps) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const float* xr = x + static_cast<size_t>(row) * cols;
  float s = -0.0f;
  for (int c = 0; c < cols; ++c) s = __fadd_rn(s, xr[c]);
  const float mean = __fdiv_rn(s, static_cast<float>(cols));
  float q = -0.0f;
  for (int c = 0; c < cols; ++c) {
    const float d = __fsub_rn(xr[c], mean);
    q = __fadd_rn(q, __fmul_rn(d, d));
  }
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(q, static_cast<float>(cols)), eps)));
  float* yr = y + static_cast<size_t>(row) * cols;
  for (int c = 0; c < cols; ++c) yr[c] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xr[c], mean), inv), g[c]), b[c]);
}

cudaError_t layernorm_f32(const float* x, float* y, __nv_bfloat16* yb, int8_t* yq, __half* yd, int rows, int cols,
                          const float* g, const float* b, float eps, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  const int grid = (rows * 32 + EW_THREADS - 1) / EW_THREADS;
  const bool vec_ok = (cols % 128 == 0) && cols <= 1024 &&
                      (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (reinterpret_cast<uintptr_t>(g) % 16 == 0) &&
                      (reinterpret_cast<uintptr_t>(b) % 16 == 0);
  if (y != nullptr) {  // f32 output: the bit-exact kernel (bf16 / Q8_0 outputs feed rounding anyway)
    if (yb != nullptr || yq != nullptr) return cudaErrorInvalidValue;
    k_layernorm_exact<<<(rows + 127) / 128, 128, 0, s>>>(x, y, rows, cols, g, b, eps);
    return cudaGetLastError();
  }
  if (!vec_ok) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(EW_THREADS);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  switch (cols / 128) {
#define VK_LN_CASE(n) \
  case n: return cudaLaunchKernelEx(&cfg, k_layernorm_vec<n>, x, y, yb, yq, yd, rows, cols, g, b, eps);
    VK_LN_CASE(1) VK_LN_CASE(2) VK_LN_CASE(3) VK_LN_CASE(4) VK_LN_CASE(5) VK_LN_CASE(6) VK_LN_CASE(7)
    VK_LN_CASE(8)
#undef VK_LN_CASE
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------- pointwise
__global__ void k_gelu(float* x, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += static_cast<size_t>(gridDim.x) * blockDim.x)
    x[i] = gelu_erf(x[i]);
}
cudaError_t gelu_f32(float* x, size_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  k_gelu<<<ew_grid(n), EW_THREADS, 0, s>>>(x, n);
  return cudaGetLastError();
}

__global__ void k_add(float* dst, const float* src, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += static_cast<size_t>(gridDim.x) * blockDim.x)
    dst[i] = dst[i] + src[i];
}
cudaError_t add_f32(float* dst, const float* src, size_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  k_add<<<ew_grid(n), EW_THREADS, 0, s>>>(dst, src, n);
  return cudaGetLastError();
}

__global__ void k_bias_rows(float* x, size_t rows, size_t cols, const float* bias) {
  const size_t n = rows * cols;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += static_cast<size_t>(gridDim.x) * blockDim.x)
    x[i] = x[i] + bias[i % cols];
}
cudaError_t add_bias_rows_f32(float* x, size_t rows, size_t cols, const float* bias, cudaStream_t s) {
  if (rows * cols == 0) return cudaSuccess;
  k_bias_rows<<<ew_grid(rows * cols), EW_THREADS, 0, s>>>(x, rows, cols, bias);
  return cudaGetLastError();
}

__global__ void k_layerscale(float* x, size_t rows, size_t cols, const float* g) {
  const size_t n = rows * cols;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += static_cast<size_t>(gridDim.x) * blockDim.x)
    x[i] = x[i] * g[i % cols];
}
cudaError_t layerscale_f32(float* x, size_t rows, size_t cols, const float* g, cudaStream_t s) {
  if (rows * cols == 0) return cudaSuccess;
  k_layerscale<<<ew_grid(rows * cols), EW_THREADS, 0, s>>>(x, rows, cols, g);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- RoPE
__global__ void k_rope_rotations(const int64_t* __restrict__ pos, int n, int quarter, RopeInv inv,
                                 const float* __restrict__ lut, float* rot) {
  const int total = n * 2 * quarter;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += gridDim.x * blockDim.x) {
    const int i = idx % quarter, axis = (idx / quarter) & 1, t = idx / (2 * quarter);
    const int64_t p = pos[2 * t + axis];
    float sn, cs;
    if (p >= 0 && p < VK_ROPE_LUT_POSITIONS) {
      const float2 sc = reinterpret_cast<const float2*>(lut)[p * quarter + i];
      sn = sc.x;
      cs = sc.y;
    } else {
      const float ang = __fmul_rn(static_cast<float>(p), inv.v[i]);
      double ds, dc;
      sincos(static_cast<double>(ang), &ds, &dc);
      sn = static_cast<float>(ds);
      cs = static_cast<float>(dc);
    }
    reinterpret_cast<float2*>(rot)[idx] = make_float2(sn, cs);
  }
}
cudaError_t rope_rotations_device(const int64_t* pos, int n, int quarter, RopeInv inv, const float* lut,
                                  float* rot, cudaStream_t s) {
  const size_t total = static_cast<size_t>(n) * 2 * quarter;
  if (total == 0) return cudaSuccess;
  k_rope_rotations<<<ew_grid(total), EW_THREADS, 0, s>>>(pos, n, quarter, inv, lut, rot);
  return cudaGetLastError();
}

// One thread per rotation pair.  rot[(t * 2 * quarter + axis * quarter + i) * 2 + {0: sin, 1: cos}]
// as in src/rope.rs:49-60.  Products and sums are separately rounded (no FMA
// contraction), so the result is bit-identical to the reference's rotate_half.
__global__ void k_rope2d(float* x, int heads, int n, int head_dim, const float* __restrict__ rot, int period) {
  const int quarter = head_dim / 4, half = head_dim / 2;
  const size_t total = static_cast<size_t>(heads) * n * 2 * quarter;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(idx % quarter);
    const int axis = static_cast<int>((idx / quarter) % 2);
    const size_t ht = idx / (2 * quarter);  // h * n + p
    const int p = static_cast<int>(ht % n) % period;  // rotation-table row
    float* base = x + ht * head_dim + axis * half;
    const float sn = rot[(static_cast<size_t>(p) * 2 * quarter + axis * quarter + i) * 2];
    const float cs = rot[(static_cast<size_t>(p) * 2 * quarter + axis * quarter + i) * 2 + 1];
    const float a = base[i], b = base[i + quarter];
    base[i] = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(b, sn));
    base[i + quarter] = __fadd_rn(__fmul_rn(b, cs), __fmul_rn(a, sn));
  }
}
cudaError_t rope2d_f32(float* x, int heads, int n, int head_dim, const float* rot, cudaStream_t s, int period) {
  const size_t total = static_cast<size_t>(heads) * n * (head_dim / 2);
  if (total == 0) return cudaSuccess;
  k_rope2d<<<ew_grid(total), EW_THREADS, 0, s>>>(x, heads, n, head_dim, rot, period > 0 ? period : n);
  return cudaGetLastError();
}

// Fused Q/K LayerNorm (64-wide rows) + axial RoPE, bit-exact with
// normalize_and_rotate (src/specialized.rs:412-454): one thread per row, the
// LayerNorm folds in ascending order as layernorm_row (src/scalar.rs:99-113),
// then rotate_half on each 32-wide axis half (pair (i, i + 16)), every
// product and sum separately rounded.
__global__ void k_qk_norm_rope(float* q, float* k, int rows, int tokens, const float* __restrict__ qg,
                               const float* __restrict__ qb, const float* __restrict__ kg,
                               const float* __restrict__ kb, const float* __restrict__ rot, float eps) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= 2 * rows) return;
  const bool is_k = idx >= rows;
  const int row = is_k ? idx - rows : idx;
  float* data = (is_k ? k : q) + static_cast<size_t>(row) * 64;
  const float* g = is_k ? kg : qg;
  const float* bt = is_k ? kb : qb;
  float v[64];
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    const float4 f = reinterpret_cast<const float4*>(data)[c];
    v[4 * c] = f.x; v[4 * c + 1] = f.y; v[4 * c + 2] = f.z; v[4 * c + 3] = f.w;
  }
  float s = -0.0f;
#pragma unroll
  for (int c = 0; c < 64; ++c) s = __fadd_rn(s, v[c]);
  const float mean = __fdiv_rn(s, 64.0f);
  float sq = -0.0f;
#pragma unroll
  for (int c = 0; c < 64; ++c) {
    const float d = __fsub_rn(v[c], mean);
    sq = __fadd_rn(sq, __fmul_rn(d, d));
  }
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sq, 64.0f), eps)));
#pragma unroll
  for (int c = 0; c < 64; ++c) v[c] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[c], mean), inv), g[c]), bt[c]);
  const int token = row % tokens;
#pragma unroll
  for (int axis = 0; axis < 2; ++axis) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float* r = rot + (static_cast<size_t>(token) * 32 + axis * 16 + i) * 2;
      const float sn = r[0], cs = r[1];
      const float a = v[axis * 32 + i], bb = v[axis * 32 + i + 16];
      v[axis * 32 + i] = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(bb, sn));
      v[axis * 32 + i + 16] = __fadd_rn(__fmul_rn(bb, cs), __fmul_rn(a, sn));
    }
  }
#pragma unroll
  for (int c = 0; c < 16; ++c)
    reinterpret_cast<float4*>(data)[c] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}
cudaError_t qk_norm_rope_f32(float* q, float* k, int heads, int tokens, const float* qg, const float* qb,
                             const float* kg, const float* kb, const float* rot, float eps, cudaStream_t s) {
  const int rows = heads * tokens;
  if (rows == 0) return cudaSuccess;
  const int grid = (2 * rows + 127) / 128;
  k_qk_norm_rope<<<grid, 128, 0, s>>>(q, k, rows, tokens, qg, qb, kg, kb, rot, eps);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- Q8_0
// One thread per 32-block; d = amax / 127 (f32), inv from the f32 d, round
// half away from zero, clamp to +-127 (src/q8_0_dot.rs:34-45).
__global__ void k_quantize_q8_0(const float* __restrict__ x, size_t nblocks, int8_t* qs, __half* d) {
  for (size_t bi = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; bi < nblocks;
       bi += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float4* src = reinterpret_cast<const float4*>(x + bi * 32);
    float v[32];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 f = __ldg(src + j);
      v[4 * j] = f.x; v[4 * j + 1] = f.y; v[4 * j + 2] = f.z; v[4 * j + 3] = f.w;
    }
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
    const float dd = amax / 127.0f;
    const float id = dd != 0.0f ? 1.0f / dd : 0.0f;
    d[bi] = __float2half_rn(dd);
    uint32_t w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint32_t packed = 0;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float qf = fminf(fmaxf(roundf(v[4 * j + t] * id), -127.0f), 127.0f);
        packed |= (static_cast<uint32_t>(static_cast<int32_t>(qf)) & 0xffu) << (8 * t);
      }
      w[j] = packed;
    }
    uint4* dst = reinterpret_cast<uint4*>(qs + bi * 32);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
}
cudaError_t quantize_q8_0(const float* x, size_t nblocks, int8_t* qs, __half* d, cudaStream_t s) {
  if (nblocks == 0) return cudaSuccess;
  k_quantize_q8_0<<<ew_grid(nblocks), EW_THREADS, 0, s>>>(x, nblocks, qs, d);
  return cudaGetLastError();
}

// BlockQ8_0 records (34 bytes: f16 d, then 32 int8) <-> split arrays.
__global__ void k_pack_q8(const int8_t* qs, const __half* d, size_t nblocks, uint8_t* blocks) {
  const size_t total = nblocks * 34;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t b = i / 34, o = i % 34;
    uint8_t val;
    if (o < 2) {
      const uint16_t h = __half_as_ushort(d[b]);
      val = static_cast<uint8_t>(o == 0 ? (h & 0xff) : (h >> 8));
    } else {
      val = static_cast<uint8_t>(qs[b * 32 + (o - 2)]);
    }
    blocks[i] = val;
  }
}
__global__ void k_unpack_q8(const uint8_t* blocks, size_t nblocks, int8_t* qs, __half* d) {
  const size_t total = nblocks * 34;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t b = i / 34, o = i % 34;
    if (o == 0) {
      const uint16_t h = static_cast<uint16_t>(blocks[i]) | (static_cast<uint16_t>(blocks[i + 1]) << 8);
      d[b] = __ushort_as_half(h);
    } else if (o >= 2) {
      qs[b * 32 + (o - 2)] = static_cast<int8_t>(blocks[i]);
    }
  }
}
cudaError_t pack_blocks_q8_0(const int8_t* qs, const __half* d, size_t nblocks, void* blocks, cudaStream_t s) {
  if (nblocks == 0) return cudaSuccess;
  k_pack_q8<<<ew_grid(nblocks * 34), EW_THREADS, 0, s>>>(qs, d, nblocks, static_cast<uint8_t*>(blocks));
  return cudaGetLastError();
}
cudaError_t unpack_blocks_q8_0(const void* blocks, size_t nblocks, int8_t* qs, __half* d, cudaStream_t s) {
  if (nblocks == 0) return cudaSuccess;
  k_unpack_q8<<<ew_grid(nblocks * 34), EW_THREADS, 0, s>>>(static_cast<const uint8_t*>(blocks), nblocks, qs, d);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- layouts
__global__ void k_cast_bf16(const float* x, __nv_bfloat16* y, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += static_cast<size_t>(gridDim.x) * blockDim.x)
    y[i] = __float2bfloat16_rn(x[i]);
}
cudaError_t cast_f32_bf16(const float* x, __nv_bfloat16* y, size_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  k_cast_bf16<<<ew_grid(n), EW_THREADS, 0, s>>>(x, y, n);
  return cudaGetLastError();
}

__global__ void k_cast_f16(const float* x, __half* y, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += static_cast<size_t>(gridDim.x) * blockDim.x)
    y[i] = __float2half_rn(x[i]);
}
cudaError_t cast_f32_f16(const float* x, __half* y, size_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  k_cast_f16<<<ew_grid(n), EW_THREADS, 0, s>>>(x, y, n);
  return cudaGetLastError();
}

// w [K, N] f32 -> wt [N, K] bf16 through a 32 x 33 shared tile.
__global__ void k_transpose_cast(const float* __restrict__ w, __nv_bfloat16* wt, int K, int N) {
  __shared__ float tile[32][33];
  const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int kk = k0 + r, nn = n0 + threadIdx.x;
    tile[r][threadIdx.x] = (kk < K && nn < N) ? w[static_cast<size_t>(kk) * N + nn] : 0.0f;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int nn = n0 + r, kk = k0 + threadIdx.x;
    if (nn < N && kk < K) wt[static_cast<size_t>(nn) * K + kk] = __float2bfloat16_rn(tile[threadIdx.x][r]);
  }
}
cudaError_t transpose_cast_bf16(const float* w, __nv_bfloat16* wt, int K, int N, cudaStream_t s) {
  dim3 grid((N + 31) / 32, (K + 31) / 32), block(32, 8);
  k_transpose_cast<<<grid, block, 0, s>>>(w, wt, K, N);
  return cudaGetLastError();
}

// w [K, N] f32 -> wt [N, K] f32.
__global__ void k_transpose_f32(const float* __restrict__ w, float* wt, int K, int N) {
  __shared__ float tile[32][33];
  const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int kk = k0 + r, nn = n0 + threadIdx.x;
    tile[r][threadIdx.x] = (kk < K && nn < N) ? w[static_cast<size_t>(kk) * N + nn] : 0.0f;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int nn = n0 + r, kk = k0 + threadIdx.x;
    if (nn < N && kk < K) wt[static_cast<size_t>(nn) * K + kk] = tile[threadIdx.x][r];
  }
}
cudaError_t transpose_f32(const float* w, float* wt, int K, int N, cudaStream_t s) {
  dim3 grid((N + 31) / 32, (K + 31) / 32), block(32, 8);
  k_transpose_f32<<<grid, block, 0, s>>>(w, wt, K, N);
  return cudaGetLastError();
}

// [images, heads, tokens, 64] -> [images * tokens, heads * 64]
__global__ void k_hnd_to_token(const float* x, float* y, int images, int heads, int tokens) {
  const size_t total = static_cast<size_t>(images) * heads * tokens * 64;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int d = static_cast<int>(i % 64);
    const size_t r = i / 64;
    const int t = static_cast<int>(r % tokens);
    const size_t ih = r / tokens;
    const int h = static_cast<int>(ih % heads);
    const size_t im = ih / heads;
    y[(im * tokens + t) * (static_cast<size_t>(heads) * 64) + h * 64 + d] = x[i];
  }
}
cudaError_t hnd_to_token_f32(const float* x, float* y, int images, int heads, int tokens, cudaStream_t s) {
  const size_t total = static_cast<size_t>(images) * heads * tokens * 64;
  if (total == 0) return cudaSuccess;
  k_hnd_to_token<<<ew_grid(total), EW_THREADS, 0, s>>>(x, y, images, heads, tokens);
  return cudaGetLastError();
}

}  // namespace vk
