// vk_attention.cu -- non-causal online-softmax attention for [heads, tokens, 64].
//
// Replaces flash_attention_f32_da3_base / attention::attention
// (src/specialized.rs:730-765, 1400-1562, 1906-2258; src/attention.rs:66-201).
//
// attention_bf16: flash-style kernel on bf16 tensor-core MMAs (m16n8k16,
//   f32 accumulation).  One CTA = 4 warps = 64 queries of one (image, head);
//   64-key K/V panels are double-buffered through shared memory with cp.async;
//   scores, the running max / sum and the output accumulator stay in
//   registers.  The key tail (865 = 13 * 64 + 33) is masked with -inf.  The
//   output is written token-major [images * tokens, heads * 64] in bf16 (the
//   out-projection's A operand) or as Q8_0 blocks, so no transpose pass is
//   needed; the f32 API gets head-major f32.
//
// attention_f32: the f32 API path.  One thread per (head, query) row keeps
//   the reference's exact per-row order (src/attention.rs:111-201): 64-key
//   panels, dot products summed left to right, tile max, correction
//   exp(m_old - m_new), exp(s - m_new), sequential P.V accumulation.
#include "vk_common.cuh"
#include "vk_internal.h"

namespace vk {

namespace {
constexpr int FA_Q = 64;     // queries per CTA
constexpr int FA_KV = 64;    // keys per panel
constexpr int FA_D = 64;     // head dim
constexpr int FA_PITCH = 72; // bf16 elements per smem row (144 B: conflict-free ldmatrix)

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const uint32_t s = smem_u32(smem);
  const int bytes = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Loads a [64 rows x 64 dims] bf16 tile (rows >= valid are zero-filled).
__device__ __forceinline__ void load_tile(__nv_bfloat16* dst, const __nv_bfloat16* src, int valid_rows) {
  const int tid = threadIdx.x;
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int idx = tid + it * 128;  // 512 16-byte chunks
    const int r = idx >> 3, c = (idx & 7) * 8;
    const bool ok = r < valid_rows;
    cp_async16(dst + r * FA_PITCH + c, src + (ok ? r : 0) * FA_D + c, ok);
  }
}
}  // namespace

template <int OUT>
__global__ void __launch_bounds__(128) k_attention_bf16(const __nv_bfloat16* __restrict__ q,
                                                        const __nv_bfloat16* __restrict__ k,
                                                        const __nv_bfloat16* __restrict__ v, int heads, int tokens,
                                                        void* out, __half* out_q8d) {
  __shared__ __align__(16) __nv_bfloat16 sQ[FA_Q * FA_PITCH];
  __shared__ __align__(16) __nv_bfloat16 sK[2][FA_KV * FA_PITCH];
  __shared__ __align__(16) __nv_bfloat16 sV[2][FA_KV * FA_PITCH];

  const int bh = blockIdx.y;
  const int q0 = blockIdx.x * FA_Q;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t head_off = static_cast<size_t>(bh) * tokens * FA_D;
  const __nv_bfloat16* qh = q + head_off;
  const __nv_bfloat16* kh = k + head_off;
  const __nv_bfloat16* vh = v + head_off;

  load_tile(sQ, qh + static_cast<size_t>(q0) * FA_D, tokens - q0);
  load_tile(sK[0], kh, tokens);
  load_tile(sV[0], vh, tokens);
  cp_async_commit();

  const int n_panels = (tokens + FA_KV - 1) / FA_KV;
  const float scale_log2 = 0.125f * 1.4426950408889634f;  // (1/sqrt(64)) * log2(e)

  uint32_t qa[4][4];  // A fragments of this warp's 16 query rows, 4 k-steps
  float o[8][4];      // output accumulator: 8 dim-tiles of 8
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY};  // rows g and g + 8 (log2 domain)
  float l_run[2] = {0.0f, 0.0f};

  const int g = lane >> 2, t4 = lane & 3;

  for (int p = 0; p < n_panels; ++p) {
    const int buf = p & 1;
    if (p + 1 < n_panels) {
      const int k1 = (p + 1) * FA_KV;
      load_tile(sK[buf ^ 1], kh + static_cast<size_t>(k1) * FA_D, tokens - k1);
      load_tile(sV[buf ^ 1], vh + static_cast<size_t>(k1) * FA_D, tokens - k1);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (p == 0) {
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        ldsm_x4(qa[ks], sQ + (warp * 16 + (lane & 15)) * FA_PITCH + ks * 16 + (lane >> 4) * 8);
    }
    // S = Q K^T for 16 rows x 64 keys
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
    const __nv_bfloat16* kb = sK[buf];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int kp = 0; kp < 2; ++kp) {  // two pairs of k-steps (32 dims each)
        uint32_t b[4];
        ldsm_x4(b, kb + (j * 8 + (lane & 7)) * FA_PITCH + kp * 32 + (lane >> 3) * 8);
        mma_bf16(s[j], qa[2 * kp], b[0], b[1]);
        mma_bf16(s[j], qa[2 * kp + 1], b[2], b[3]);
      }
    }
    // mask the key tail, scale into the log2 domain, online softmax
    const int kbase = p * FA_KV;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kbase + j * 8 + 2 * t4 + (e & 1);
        const float val = key < tokens ? s[j][e] * scale_log2 : -INFINITY;
        s[j][e] = val;
        mx[e >> 1] = fmaxf(mx[e >> 1], val);
      }
    }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float m_new = fmaxf(m_run[r], mx[r]);
      corr[r] = (m_run[r] == -INFINITY) ? 0.0f : exp2f(m_run[r] - m_new);
      m_run[r] = m_new;
    }
    float rs[2] = {0.0f, 0.0f};
    uint32_t pa[4][4];  // P as A fragments (bf16), 4 k-steps of 16 keys
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p0 = exp2f(s[j][0] - m_run[0]);
      const float p1 = exp2f(s[j][1] - m_run[0]);
      const float p2 = exp2f(s[j][2] - m_run[1]);
      const float p3 = exp2f(s[j][3] - m_run[1]);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      const int ks = j >> 1;
      if ((j & 1) == 0) {
        pa[ks][0] = pack_bf16x2(p0, p1);
        pa[ks][1] = pack_bf16x2(p2, p3);
      } else {
        pa[ks][2] = pack_bf16x2(p0, p1);
        pa[ks][3] = pack_bf16x2(p2, p3);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l_run[r] = l_run[r] * corr[r] + rs[r];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      o[j][0] *= corr[0];
      o[j][1] *= corr[0];
      o[j][2] *= corr[1];
      o[j][3] *= corr[1];
    }
    // O += P V
    const __nv_bfloat16* vb = sV[buf];
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int dp = 0; dp < 4; ++dp) {  // pairs of 8-wide dim tiles
        uint32_t b[4];
        ldsm_x4_t(b, vb + (ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * FA_PITCH + dp * 16 + (lane >> 4) * 8);
        mma_bf16(o[2 * dp], pa[ks], b[0], b[1]);
        mma_bf16(o[2 * dp + 1], pa[ks], b[2], b[3]);
      }
    }
    __syncthreads();
  }

  // normalise and store
  const float inv[2] = {1.0f / l_run[0], 1.0f / l_run[1]};
  const int b_img = bh / heads, h = bh - b_img * heads;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int t = q0 + warp * 16 + g + r * 8;
    const bool valid = t < tokens;
    if constexpr (OUT == ATTN_OUT_HEAD_F32) {
      if (valid) {
        float* dst = static_cast<float*>(out) + head_off + static_cast<size_t>(t) * FA_D;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<float2*>(dst + j * 8 + 2 * t4) = make_float2(o[j][2 * r] * inv[r], o[j][2 * r + 1] * inv[r]);
      }
    } else if constexpr (OUT == ATTN_OUT_TOKEN_BF16) {
      if (valid) {
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(out) +
                             (static_cast<size_t>(b_img) * tokens + t) * (static_cast<size_t>(heads) * FA_D) + h * FA_D;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<uint32_t*>(dst + j * 8 + 2 * t4) = pack_bf16x2(o[j][2 * r] * inv[r], o[j][2 * r + 1] * inv[r]);
      }
    } else {  // Q8_0 blocks: dims [0,32) are tiles j = 0..3, [32,64) are j = 4..7
#pragma unroll
      for (int blk = 0; blk < 2; ++blk) {
        float vals[8];
        float amax = 0.0f;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          vals[2 * jj] = o[blk * 4 + jj][2 * r] * inv[r];
          vals[2 * jj + 1] = o[blk * 4 + jj][2 * r + 1] * inv[r];
          amax = fmaxf(amax, fmaxf(fabsf(vals[2 * jj]), fabsf(vals[2 * jj + 1])));
        }
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        const float dd = amax / 127.0f;
        const float id = dd != 0.0f ? 1.0f / dd : 0.0f;
        if (valid) {
          const size_t row = static_cast<size_t>(b_img) * tokens + t;
          const size_t col0 = static_cast<size_t>(h) * FA_D + blk * 32;
          int8_t* dst = static_cast<int8_t*>(out) + row * (static_cast<size_t>(heads) * FA_D) + col0;
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const int q_lo = static_cast<int>(fminf(fmaxf(roundf(vals[2 * jj] * id), -127.0f), 127.0f));
            const int q_hi = static_cast<int>(fminf(fmaxf(roundf(vals[2 * jj + 1] * id), -127.0f), 127.0f));
            const uint16_t pk = static_cast<uint16_t>((q_lo & 0xff) | ((q_hi & 0xff) << 8));
            *reinterpret_cast<uint16_t*>(dst + jj * 8 + 2 * t4) = pk;
          }
          if (t4 == 0) out_q8d[row * (static_cast<size_t>(heads) * FA_D / 32) + col0 / 32] = __float2half_rn(dd);
        }
      }
    }
  }
}

cudaError_t attention_bf16(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v, int images,
                           int heads, int tokens, int out_mode, void* out, __half* out_q8d, cudaStream_t s) {
  if (images <= 0 || heads <= 0 || tokens <= 0) return cudaErrorInvalidValue;
  dim3 grid((tokens + FA_Q - 1) / FA_Q, images * heads);
  switch (out_mode) {
    case ATTN_OUT_HEAD_F32: k_attention_bf16<ATTN_OUT_HEAD_F32><<<grid, 128, 0, s>>>(q, k, v, heads, tokens, out, out_q8d); break;
    case ATTN_OUT_TOKEN_BF16: k_attention_bf16<ATTN_OUT_TOKEN_BF16><<<grid, 128, 0, s>>>(q, k, v, heads, tokens, out, out_q8d); break;
    case ATTN_OUT_TOKEN_Q8: k_attention_bf16<ATTN_OUT_TOKEN_Q8><<<grid, 128, 0, s>>>(q, k, v, heads, tokens, out, out_q8d); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

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
