// vk_abi_internal.h -- definitions behind the opaque handles of the C ABI.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <climits>
#include <initializer_list>
#include <map>
#include <tuple>
#include <vector>

#include "vestra_b200.h"

struct vk_ctx {
  int device = 0;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  int math = VK_MATH_F32;
  int* d_err = nullptr;  // device error word written by bounded waits
  void* ws = nullptr;    // grow-only scratch for the f32-interface operators
  size_t ws_bytes = 0;
  // Rotation lookup tables of the RoPE operators, one per (head_dim, freq):
  // (sin, cos) of position * inv_freq[i] for integer positions [0, VK_ROPE_LUT_POSITIONS),
  // computed once on the host with the reference's f32 calls.
  struct RopeLut {
    size_t quarter;
    uint32_t freq_bits;
    float inv[32];
    float* lut;
  };
  std::vector<RopeLut> rope_luts;
};

// Sub-allocates a workspace in two passes: a sizing pass (base == nullptr)
// returns null pointers and totals the bytes, a second pass hands out slices.
struct Arena {
  void* base = nullptr;
  size_t off = 0;
  void* take(size_t bytes);
  template <class T>
  T* get(size_t count) {
    return static_cast<T*>(take(count * sizeof(T)));
  }
};

struct vk_linear {
  int device = 0;
  int math = VK_MATH_F32;
  size_t k = 0, n = 0;
  float* w_f32 = nullptr;          // [k, n] (f32 math)
  __nv_bfloat16* w_bf16 = nullptr; // [n, k] (bf16 math)
  int8_t* w_q = nullptr;           // [n, k] (Q8_0)
  __half* w_d = nullptr;           // [n, k / 32]
  float* bias = nullptr;           // [n] or null
  float* scale = nullptr;          // [n] or null
};

struct EncLayer {
  float *ln1_g, *ln1_b, *ln2_g, *ln2_b;
  float *qkv_b, *proj_b, *ls1, *fc1_b, *fc2_b, *ls2;
  // weights in the form of the encoder's math
  float *qkv_w32, *proj_w32, *fc1_w32, *fc2_w32;          // [K, N]
  __nv_bfloat16 *qkv_w16, *proj_w16, *fc1_w16, *fc2_w16;  // [N, K]
  int8_t *qkv_q, *proj_q, *fc1_q, *fc2_q;                 // [N, K]
  __half *qkv_d, *proj_d, *fc1_d, *fc2_d;                 // [N, K / 32]
  float* qkn;  // [4][64]: q gamma, q beta, k gamma, k beta (Q/K LayerNorm before RoPE), or null
};

struct vk_encoder {
  int device = 0;
  vk_encoder_config cfg{};
  int embed = 0;
  std::vector<void*> allocations;
  std::vector<EncLayer> layers;
  // activations, sized for `cap_rows` rows
  size_t cap_rows = 0;
  void* act = nullptr;
  // rotation table for the last (grid_h, grid_w)
  size_t rope_h = 0, rope_w = 0;
  float* rope = nullptr;
  // captured forwards: (images, grid_h, grid_w, in, out, stream) -> graph
  std::map<std::tuple<size_t, size_t, size_t, const void*, void*, cudaStream_t>, cudaGraphExec_t> graphs;
  std::map<std::tuple<size_t, size_t, size_t, const void*, void*, cudaStream_t>, int> seen;
  int last_launches = 0;
  // end-to-end pipeline resources
  // (three device slots of image chunks cycle H2D -> compute -> D2H; the
  // ring and its events persist across calls so consecutive calls overlap)
  cudaStream_t h2d = nullptr, d2h = nullptr, comp = nullptr;
  float* slots[3] = {nullptr, nullptr, nullptr};
  cudaEvent_t slot_free[3] = {nullptr, nullptr, nullptr};  // D2H out of the slot finished
  cudaEvent_t slot_in[3] = {nullptr, nullptr, nullptr};    // H2D into the slot finished
  cudaEvent_t slot_out[3] = {nullptr, nullptr, nullptr};   // compute on the slot finished
  cudaEvent_t dev_tail = nullptr;  // last use of the activations from the context stream
  size_t slot_rows = 0;
  size_t next_slot = 0;
};

int vk_fail(int status, const char* fmt, ...);

// The kernels take their dimensions as 32-bit ints: an entry point rejects
// any dimension beyond INT_MAX with VK_UNSUPPORTED_SHAPE instead of letting a
// narrowing cast truncate it.
inline int vk_dims_fit(const char* name, std::initializer_list<size_t> dims) {
  for (size_t d : dims)
    if (d > static_cast<size_t>(INT_MAX))
      return vk_fail(VK_UNSUPPORTED_SHAPE, "%s: dimension %zu exceeds the 32-bit range of the kernels", name, d);
  return VK_OK;
}
int vk_cuda_status(cudaError_t e, const char* what);
int ctx_reserve(vk_ctx* ctx, size_t bytes);

#define VK_TRY_CUDA(expr, what)                    \
  do {                                             \
    cudaError_t _e = (expr);                       \
    if (_e != cudaSuccess) return vk_cuda_status(_e, what); \
  } while (0)
#define VK_TRY(expr)           \
  do {                         \
    int _s = (expr);           \
    if (_s != VK_OK) return _s; \
  } while (0)
