// vk_epilogue.cuh -- the fused GEMM epilogues, applied to 32 consecutive
// output columns of one row held in registers (one tcgen05.ld of TMEM).
//
// epi_math       bias, GELU, LayerScale, RoPE in registers
// epi_direct     the per-row global store (used where a tile chunk cannot go
//                through a TMA store: Q8_0 outputs, image boundaries)
// epilogue_chunk epi_math + epi_direct
#pragma once
#include "vk_common.cuh"
#include "vk_internal.h"

namespace vk {

// Head-major coordinates of a QKV output column chunk.
struct QkvPos {
  int g, head, axis, image, t;
};
__device__ __forceinline__ QkvPos qkv_pos(const GemmEpi& p, int row, int col0) {
  QkvPos q;
  const int E = p.heads * 64;
  q.g = col0 / E;
  const int rem = col0 - q.g * E;
  q.head = rem >> 6;
  q.axis = (rem >> 5) & 1;
  q.image = row / p.tokens;
  q.t = row - q.image * p.tokens;
  return q;
}

// The V third of a bf16 QKV output is stored as IEEE f16: attention runs
// its P V product in f16 (P with a 10-bit mantissa), and one MMA takes A and
// B of the same type.
__device__ __forceinline__ bool qkv_is_v(const GemmEpi& p, int col0) { return col0 >= 2 * p.heads * 64; }

// bias32 / scale32 point at the 32 bias / scale values of this chunk
// (16-byte aligned, global or shared memory) or are null.
template <int MODE, bool FAST_GELU = false>
__device__ __forceinline__ void epi_math(const GemmEpi& p, int row, int col0, float (&v)[32], const float* bias32,
                                         const float* scale32) {
  if (bias32 != nullptr) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 b = reinterpret_cast<const float4*>(bias32)[j];
      v[4 * j] += b.x;
      v[4 * j + 1] += b.y;
      v[4 * j + 2] += b.z;
      v[4 * j + 3] += b.w;
    }
  }
  if constexpr (MODE == EPI_F32 || MODE == EPI_RESID) {
    if (scale32 != nullptr) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 c = reinterpret_cast<const float4*>(scale32)[j];
        v[4 * j] *= c.x;
        v[4 * j + 1] *= c.y;
        v[4 * j + 2] *= c.z;
        v[4 * j + 3] *= c.w;
      }
    }
  } else if constexpr (MODE == EPI_BF16_GELU || MODE == EPI_Q8_GELU) {
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      if constexpr (FAST_GELU) {
        const float2 g = gelu_erf_ex2(make_float2(v[j], v[j + 1]));
        v[j] = g.x;
        v[j + 1] = g.y;
      } else {
        v[j] = gelu_erf(v[j]);
        v[j + 1] = gelu_erf(v[j + 1]);
      }
    }
  } else if constexpr (MODE == EPI_TOKENS) {
    // tokens = projected + position, the projection's (acc + bias) rounded
    // first (vestra_prepend_cls_add_pos_f32, src/cuda.rs:321-334)
    const int t = row % p.tokens;
    const float4* ps = reinterpret_cast<const float4*>(p.pos + static_cast<size_t>(t + 1) * p.ldo + col0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 q4 = __ldg(ps + j);
      v[4 * j] += q4.x;
      v[4 * j + 1] += q4.y;
      v[4 * j + 2] += q4.z;
      v[4 * j + 3] += q4.w;
    }
  } else if constexpr (MODE == EPI_QKV_BF16 || MODE == EPI_QKV_F32) {
    const QkvPos q = qkv_pos(p, row, col0);
    if (p.rope != nullptr && q.g < 2) {
      // Axial RoPE, rotate-half pairing (i, i + 16) inside this 32-wide axis
      // half (src/rope.rs:84-93); the chunk is exactly one axis half.
      // a global cross-view layer's token t sits at view position t % rope_tokens
      const int rt = p.rope_tokens > 0 ? p.rope_tokens : p.tokens;
      const int tr = p.rope_tokens > 0 ? q.t % p.rope_tokens : q.t;
      const float4* r = reinterpret_cast<const float4*>(p.rope) + static_cast<size_t>(q.axis * 8) * rt + tr;
#pragma unroll
      for (int i2 = 0; i2 < 8; ++i2) {
        const float4 sc = __ldg(r + static_cast<size_t>(i2) * rt);  // (sin, cos) of 2 i2, 2 i2 + 1
        const int i = 2 * i2;
        const float a0 = v[i], b0 = v[i + 16], a1 = v[i + 1], b1 = v[i + 17];
        // separately rounded products and sums, as rotate_half computes them
        v[i] = __fsub_rn(__fmul_rn(a0, sc.y), __fmul_rn(b0, sc.x));
        v[i + 16] = __fadd_rn(__fmul_rn(b0, sc.y), __fmul_rn(a0, sc.x));
        v[i + 1] = __fsub_rn(__fmul_rn(a1, sc.w), __fmul_rn(b1, sc.z));
        v[i + 17] = __fadd_rn(__fmul_rn(b1, sc.w), __fmul_rn(a1, sc.z));
      }
    }
  }
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float (&v)[32]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int j = 0; j < 4; ++j)
    d[j] = make_uint4(pack_bf16x2(v[8 * j], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                      pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
}
__device__ __forceinline__ void store_f16x32(__half* dst, const float (&v)[32]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int j = 0; j < 4; ++j)
    d[j] = make_uint4(pack_f16x2(v[8 * j], v[8 * j + 1]), pack_f16x2(v[8 * j + 2], v[8 * j + 3]),
                      pack_f16x2(v[8 * j + 4], v[8 * j + 5]), pack_f16x2(v[8 * j + 6], v[8 * j + 7]));
}
__device__ __forceinline__ void store_f32x32(float* dst, const float (&v)[32]) {
  float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
  for (int j = 0; j < 8; ++j) d[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

template <int MODE>
__device__ __forceinline__ void epi_direct(const GemmEpi& p, int row, int col0, int N, float (&v)[32]) {
  if constexpr (MODE == EPI_F32) {
    store_f32x32(static_cast<float*>(p.out) + row * p.ldo + col0, v);
  } else if constexpr (MODE == EPI_BF16 || MODE == EPI_BF16_GELU) {
    store_bf16x32(static_cast<__nv_bfloat16*>(p.out) + row * p.ldo + col0, v);
  } else if constexpr (MODE == EPI_TOKENS) {
    const int img = row / p.tokens, t = row - img * p.tokens;
    store_f32x32(static_cast<float*>(p.out) + (static_cast<size_t>(img) * (p.tokens + 1) + 1 + t) * p.ldo + col0, v);
  } else if constexpr (MODE == EPI_RESID) {
    float4* dst = reinterpret_cast<float4*>(p.resid + row * p.ldo + col0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float4 r = dst[j];
      r.x += v[4 * j];
      r.y += v[4 * j + 1];
      r.z += v[4 * j + 2];
      r.w += v[4 * j + 3];
      dst[j] = r;
    }
  } else if constexpr (MODE == EPI_QKV_BF16 || MODE == EPI_QKV_F32) {
    const QkvPos q = qkv_pos(p, row, col0);
    const size_t off = ((static_cast<size_t>(q.image) * p.heads + q.head) * p.tokens + q.t) * 64 + q.axis * 32;
    void* base = q.g == 0 ? p.q : (q.g == 1 ? p.k : p.v);
    if constexpr (MODE == EPI_QKV_BF16) {
      if (q.g == 2)
        store_f16x32(static_cast<__half*>(base) + off, v);
      else
        store_bf16x32(static_cast<__nv_bfloat16*>(base) + off, v);
    }
    else
      store_f32x32(static_cast<float*>(base) + off, v);
  } else if constexpr (MODE == EPI_Q8_GELU) {
    // this 32-column chunk is exactly one Q8_0 block of the row
    // (quantize_row_q8_0, src/q8_0_dot.rs:34-45).
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
    const float dd = amax / 127.0f;
    const float id = dd != 0.0f ? 1.0f / dd : 0.0f;
    p.q8d[static_cast<size_t>(row) * (N / 32) + col0 / 32] = __float2half_rn(dd);
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
    uint4* dst = reinterpret_cast<uint4*>(p.q8 + static_cast<size_t>(row) * N + col0);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
  (void)N;
}

template <int MODE>
__device__ __forceinline__ void epilogue_chunk(const GemmEpi& p, int row, int col0, int N, float (&v)[32]) {
  epi_math<MODE, true>(p, row, col0, v, p.bias ? p.bias + col0 : nullptr, p.scale ? p.scale + col0 : nullptr);
  epi_direct<MODE>(p, row, col0, N, v);
}

}  // namespace vk
