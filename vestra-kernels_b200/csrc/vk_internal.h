// vk_internal.h -- launchers shared between the kernel files and the C-ABI
// layer.  Nothing here crosses the public boundary (include/vestra_b200.h).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace vk {

// Epilogues of the projection GEMMs.  Every mode first adds bias[col] when a
// bias is given (the reference's `acc + bias`, src/specialized.rs:1150-1163).
enum EpiMode : int {
  EPI_F32 = 0,        // out_f32 = (acc + bias) [* scale]
  EPI_BF16 = 1,       // out_bf16 = acc + bias
  EPI_BF16_GELU = 2,  // out_bf16 = gelu(acc + bias)              (fc1)
  EPI_RESID = 3,      // resid_f32 += (acc + bias) * scale        (out-proj, fc2)
  EPI_QKV_BF16 = 4,   // head-major bf16 q/k/v, optional RoPE on q and k
  EPI_QKV_F32 = 5,    // head-major f32 q/k/v, optional RoPE on q and k
  EPI_Q8_GELU = 6,    // Q8_0 blocks of gelu(acc + bias)          (fc1, Q8_0 mode)
  EPI_F32_GELU = 7,   // out_f32 = gelu(acc + bias)               (fc1, f32 mode)
  EPI_TOKENS = 8,     // out_f32[img][1 + p] = (acc + bias) + pos[1 + p]   (patch embedding; rows are (img, p))
};

struct GemmEpi {
  const float* bias = nullptr;   // [N] or null
  const float* scale = nullptr;  // [N] or null
  void* out = nullptr;           // [M, ldo]
  int64_t ldo = 0;
  float* resid = nullptr;        // [M, ldo] (EPI_RESID)
  void* q = nullptr;             // [images, heads, tokens, 64]
  void* k = nullptr;
  void* v = nullptr;
  const float* rope = nullptr;   // [2 * 8, tokens] of (sin_i, cos_i, sin_i+1, cos_i+1): [axis * 8 + i / 2][t], or null
  int tokens = 0;                // rows per image (per group of views for a global layer)
  int rope_tokens = 0;           // rows of the rotation table (0: tokens); token t uses row t % rope_tokens
  int heads = 0;                 // embed = heads * 64
  const float* pos = nullptr;    // [tokens + 1, ldo] position table (EPI_TOKENS; `tokens` = patches per image)
  const float* qkn = nullptr;    // [4][64] q gamma, q beta, k gamma, k beta: LayerNorm of each q / k head before RoPE, or null
  float qkn_eps = 0.0f;
  int8_t* q8 = nullptr;          // [M, N] int8 quants (EPI_Q8_GELU)
  __half* q8d = nullptr;         // [M, N / 32] scales
};

// Tensor-map helpers (driver entry point fetched through the runtime).
bool make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
                  uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                  uint32_t box_outer, CUtensorMapSwizzle swz);

bool make_tmap_3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1,
                  uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0,
                  uint32_t box1, CUtensorMapSwizzle swz);

// Any rank up to 5: dims[0] innermost; strides_bytes[i] is the stride of
// dimension i + 1; out-of-range box elements read as zero.
bool make_tmap_nd(CUtensorMap* map, CUtensorMapDataType dt, const void* base, int rank, const uint64_t* dims,
                  const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz);

int num_sms();
// Launch attributes for programmatic dependent launch (off with VK_NO_PDL).
bool pdl_enabled();
// Raises `func`'s dynamic shared-memory limit to `bytes` on the current
// device (once per device and function; the attribute is per device).
cudaError_t ensure_smem_limit(const void* func, int bytes);
// Per-device cache slot for launch facts computed once (e.g. resident CTA
// pairs); returns a pointer to an int initialised to 0 for (key, device).
int* per_device_slot(const void* key);

// bf16 x bf16 -> f32 tcgen05 GEMM: C[M,N] = A[M,K] . W[N,K]^T (both K-major),
// K % 64 == 0, N % 128 == 0.  Returns a cudaError_t.
cudaError_t gemm_bf16_tc(const __nv_bfloat16* A, const __nv_bfloat16* W, int M, int N, int K,
                         int mode, const GemmEpi& epi, int* err, cudaStream_t s);

// f32 SIMT GEMM (CUDA cores, FFMA): C[M,N] = A[M,K] . B[K,N] (reference
// layout, B row-major [K, N]); every output is one ascending-K chain of
// FMAs, the accumulation of src/specialized.rs:1133-1148.  Epilogue modes
// EPI_F32, EPI_F32_GELU, EPI_RESID, EPI_QKV_F32 (RoPE is a separate pass).
cudaError_t gemm_f32_simt(const float* A, const float* B, int M, int N, int K, int mode,
                          const GemmEpi& epi, cudaStream_t s);

// Q8_0: A int8 [M,K] + f16 scales [M,K/32]; W int8 [N,K] + scales [N,K/32].
cudaError_t gemm_q8_tc(const int8_t* Aq, const __half* Ad, const int8_t* Wq, const __half* Wd,
                       int M, int N, int K, int mode, const GemmEpi& epi, int32_t* dots_out,
                       int* err, cudaStream_t s);

// Elementwise / normalisation kernels (vk_elementwise.cu).
cudaError_t layernorm_f32(const float* x, float* y, __nv_bfloat16* y_bf16, int8_t* y_q8,
                          __half* y_q8d, int rows, int cols, const float* g, const float* b,
                          float eps, cudaStream_t s);
cudaError_t gelu_f32(float* x, size_t n, cudaStream_t s);
cudaError_t add_f32(float* dst, const float* src, size_t n, cudaStream_t s);
cudaError_t add_bias_rows_f32(float* x, size_t rows, size_t cols, const float* bias,
                              cudaStream_t s);
cudaError_t layerscale_f32(float* x, size_t rows, size_t cols, const float* g, cudaStream_t s);
// Per-token rotation table rot[(t * 2q + axis * q + i) * 2 + {sin, cos}] from
// device positions pos[t, 2]: integer positions in [0, lut_positions) are
// looked up in lut[(p * q + i) * 2 + {sin, cos}] (bit-identical to the host
// table); others fall back to sin / cos in double precision rounded to f32.
constexpr int VK_ROPE_LUT_POSITIONS = 4096;
struct RopeInv {
  float v[32];
};
cudaError_t rope_rotations_device(const int64_t* pos, int n, int quarter, RopeInv inv, const float* lut,
                                  float* rot, cudaStream_t s);
cudaError_t rope2d_f32(float* x, int heads, int n, int head_dim, const float* rot,
                       cudaStream_t s,
                       int period = 0);  // rows of `rot` (0: n); token p uses row p % period
cudaError_t qk_norm_rope_f32(float* q, float* k, int heads, int tokens, const float* qg,
                             const float* qb, const float* kg, const float* kb, const float* rot,
                             float eps, cudaStream_t s);
cudaError_t quantize_q8_0(const float* x, size_t nblocks, int8_t* qs, __half* d,
                          cudaStream_t s);
cudaError_t pack_blocks_q8_0(const int8_t* qs, const __half* d, size_t nblocks, void* blocks,
                             cudaStream_t s);
cudaError_t unpack_blocks_q8_0(const void* blocks, size_t nblocks, int8_t* qs, __half* d,
                               cudaStream_t s);
cudaError_t cast_f32_bf16(const float* x, __nv_bfloat16* y, size_t n, cudaStream_t s);
cudaError_t cast_f32_f16(const float* x, __half* y, size_t n, cudaStream_t s);
// w [K, N] f32 (reference layout) -> wt [N, K] bf16 / f32.
cudaError_t transpose_cast_bf16(const float* w, __nv_bfloat16* wt, int K, int N, cudaStream_t s);
cudaError_t transpose_f32(const float* w, float* wt, int K, int N, cudaStream_t s);
cudaError_t hnd_to_token_f32(const float* x, float* y, int images, int heads, int tokens,
                             cudaStream_t s);

// Attention (vk_attention.cu).  q,k,v head-major [images*heads, tokens, 64].
// bf16 path: out either head-major bf16/f32 or token-major bf16 [images*tokens, heads*64].
enum AttnOut : int { ATTN_OUT_HEAD_F32 = 0, ATTN_OUT_TOKEN_BF16 = 1, ATTN_OUT_TOKEN_Q8 = 2 };
cudaError_t attention_bf16(const __nv_bfloat16* q, const __nv_bfloat16* k,
                           const __half* v, int images, int heads, int tokens,
                           int out_mode, void* out, __half* out_q8d, int* err, cudaStream_t s,
                           bool precise = false);
// f32 SIMT online attention for any head_dim <= 128 (head-major in and out).
cudaError_t attention_f32(const float* q, const float* k, const float* v, int bh, int tokens,
                          int head_dim, float* out, cudaStream_t s);

}  // namespace vk
