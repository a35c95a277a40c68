// vk_attention.cu -- non-causal online-softmax attention for [heads, tokens, 64].
//
// Replaces flash_attention_f32_da3_base / attention::attention
// (src/specialized.rs:730-765, 1400-1562, 1906-2258; src/attention.rs:66-201).
//
// The bf16 tensor-core kernel is in vk_attention_tc.cu.
//
// attention_f32: the f32 API path.  One thread per (head, query) row keeps
//   the reference's exact per-row order (src/attention.rs:111-201): 64-key
//   panels, dot products summed left to right, tile max, correction
//   exp(m_old - m_new), exp(s - m_new), sequential P.V accumulation.
#include "vk_common.cuh"
#include "vk_internal.h"

namespace vk {


// ------------------------------------------------------------------ f32 path
template <int D>
__global__ void __launch_bounds__(128) k_attention_f32(const float* __restrict__ q, const float* __restrict__ k,
                                                       const float* __restrict__ v, int tokens, float* out) {
  constexpr int KV = 64;
  __shared__ float sK[KV * D];
  __shared__ float sV[KV * D];
  const int bh = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const bool active = i < tokens;
  const size_t base = static_cast<size_t>(bh) * tokens * D;
  const float scale = 1.0f / sqrtf(static_cast<float>(D));
  float qi[D], acc[D];
#pragma unroll
  for (int d = 0; d < D; ++d) {
    qi[d] = active ? q[base + static_cast<size_t>(i) * D + d] : 0.0f;
    acc[d] = 0.0f;
  }
  float running_max = -INFINITY, running_sum = 0.0f;
  for (int j0 = 0; j0 < tokens; j0 += KV) {
    const int cols = min(KV, tokens - j0);
    __syncthreads();
    for (int idx = threadIdx.x; idx < cols * D; idx += blockDim.x) {
      sK[idx] = k[base + static_cast<size_t>(j0) * D + idx];
      sV[idx] = v[base + static_cast<size_t>(j0) * D + idx];
    }
    __syncthreads();
    float sc[KV];
    float tile_max = -INFINITY;
#pragma unroll 4
    for (int j = 0; j < cols; ++j) {
      float dot = -0.0f;
#pragma unroll
      for (int d = 0; d < D; ++d) dot = __fadd_rn(dot, __fmul_rn(qi[d], sK[j * D + d]));
      const float sv = __fmul_rn(dot, scale);
      sc[j] = sv;
      tile_max = fmaxf(tile_max, sv);
    }
    const float new_max = fmaxf(running_max, tile_max);
    const float corr = isfinite(running_max) ? expf(running_max - new_max) : 0.0f;
    running_sum = __fmul_rn(running_sum, corr);
#pragma unroll
    for (int d = 0; d < D; ++d) acc[d] = __fmul_rn(acc[d], corr);
    for (int j = 0; j < cols; ++j) {
      const float pj = expf(__fsub_rn(sc[j], new_max));
      running_sum = __fadd_rn(running_sum, pj);
#pragma unroll
      for (int d = 0; d < D; ++d) acc[d] = __fadd_rn(acc[d], __fmul_rn(pj, sV[j * D + d]));
    }
    running_max = new_max;
  }
  if (active) {
    const float inv = 1.0f / running_sum;
#pragma unroll
    for (int d = 0; d < D; ++d) out[base + static_cast<size_t>(i) * D + d] = __fmul_rn(acc[d], inv);
  }
}

cudaError_t attention_f32(const float* q, const float* k, const float* v, int bh, int tokens, int head_dim,
                          float* out, cudaStream_t s) {
  if (bh <= 0 || tokens <= 0) return cudaErrorInvalidValue;
  dim3 grid((tokens + 127) / 128, bh);
  switch (head_dim) {
    case 8: k_attention_f32<8><<<grid, 128, 0, s>>>(q, k, v, tokens, out); break;
    case 16: k_attention_f32<16><<<grid, 128, 0, s>>>(q, k, v, tokens, out); break;
    case 32: k_attention_f32<32><<<grid, 128, 0, s>>>(q, k, v, tokens, out); break;
    case 64: k_attention_f32<64><<<grid, 128, 0, s>>>(q, k, v, tokens, out); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace vk
