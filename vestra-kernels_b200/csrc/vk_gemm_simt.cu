// vk_gemm_simt.cu -- f32 projection GEMM on the CUDA cores (FFMA).
//
// The f32 API of the reference (linear_f32_da3_base, linear_bias_scale_f32_da3_base,
// qkv_f32_da3_base; src/specialized.rs:770-1167) promises f32 arithmetic.  Each
// output here is a single ascending-K chain of fused multiply-adds, which is
// exactly the accumulation of the reference's 6x64 AVX-512 tiles
// (`acc = fmadd(a, b, acc)` for kk in 0..k), so the raw products match the
// reference bit for bit; the epilogue rounds `(acc + bias) * scale` in the
// reference's order without contraction.
//
// 128 x 128 output tile per 256-thread CTA, 8 x 8 outputs per thread in a
// 2 x 2 arrangement of 4 x 4 blocks, K staged 8 at a time through shared memory.
#include "vk_common.cuh"
#include "vk_internal.h"

namespace vk {

namespace {
constexpr int SB_M = 128, SB_N = 128, SB_K = 8;
}

__device__ __forceinline__ void simt_store(const GemmEpi& p, int mode, int row, int col, float acc) {
  float v = acc;
  if (p.bias != nullptr) v = __fadd_rn(v, p.bias[col]);
  switch (mode) {
    case EPI_F32:
      if (p.scale != nullptr) v = __fmul_rn(v, p.scale[col]);
      static_cast<float*>(p.out)[static_cast<size_t>(row) * p.ldo + col] = v;
      break;
    case EPI_F32_GELU:
      static_cast<float*>(p.out)[static_cast<size_t>(row) * p.ldo + col] = gelu_erf(v);
      break;
    case EPI_RESID: {
      float* r = p.resid + static_cast<size_t>(row) * p.ldo + col;
      *r = __fadd_rn(*r, __fmul_rn(v, p.scale[col]));
      break;
    }
    case EPI_QKV_F32: {
      const int E = p.heads * 64;
      const int g = col / E, rem = col - g * E, head = rem >> 6, d = rem & 63;
      const int image = row / p.tokens, t = row - image * p.tokens;
      float* base = static_cast<float*>(g == 0 ? p.q : (g == 1 ? p.k : p.v));
      base[((static_cast<size_t>(image) * p.heads + head) * p.tokens + t) * 64 + d] = v;
      break;
    }
    default: break;
  }
}

__global__ void __launch_bounds__(256) k_gemm_f32(const float* __restrict__ A, const float* __restrict__ B, int M,
                                                  int N, int K, int mode, const GemmEpi epi) {
  __shared__ __align__(16) float As[2][SB_K][SB_M];
  __shared__ __align__(16) float Bs[2][SB_K][SB_N];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * SB_M, n0 = blockIdx.x * SB_N;

  // loaders: A tile 128 x 8 (each thread 4 values of one row), B tile 8 x 128
  const int a_row = tid >> 1, a_k = (tid & 1) * 4;
  const int b_k = tid >> 5, b_col = (tid & 31) * 4;

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

  auto load = [&](int buf, int k0) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int gr = m0 + a_row, gk = k0 + a_k + t;
      As[buf][a_k + t][a_row] = (gr < M && gk < K) ? A[static_cast<size_t>(gr) * K + gk] : 0.0f;
    }
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int gk = k0 + b_k, gc = n0 + b_col + t;
      Bs[buf][b_k][b_col + t] = (gk < K && gc < N) ? B[static_cast<size_t>(gk) * N + gc] : 0.0f;
    }
  };

  const int ktiles = (K + SB_K - 1) / SB_K;
  load(0, 0);
  __syncthreads();
  for (int kt = 0; kt < ktiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < ktiles) load(buf ^ 1, (kt + 1) * SB_K);
#pragma unroll
    for (int kk = 0; kk < SB_K; ++kk) {
      if (kt * SB_K + kk >= K) break;
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int row = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (row >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int col = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (col < N) simt_store(epi, mode, row, col, acc[i][j]);
    }
  }
}

cudaError_t gemm_f32_simt(const float* A, const float* B, int M, int N, int K, int mode, const GemmEpi& epi,
                          cudaStream_t s) {
  if (M <= 0 || N <= 0 || K <= 0) return cudaErrorInvalidValue;
  if (mode != EPI_F32 && mode != EPI_F32_GELU && mode != EPI_RESID && mode != EPI_QKV_F32)
    return cudaErrorInvalidValue;
  dim3 grid((N + SB_N - 1) / SB_N, (M + SB_M - 1) / SB_M);
  k_gemm_f32<<<grid, 256, 0, s>>>(A, B, M, N, K, mode, epi);
  return cudaGetLastError();
}

}  // namespace vk
