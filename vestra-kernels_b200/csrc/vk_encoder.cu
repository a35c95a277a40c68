// vk_encoder.cu -- the DA3-BASE ViT encoder driver behind vk_encoder_*.
//
// The reference crate exposes only operators; Vestra Engine composes them
// per block (src/lib.rs:52-130 called in the order pre-LN, qkv, rope / qk-norm,
// attention, out-proj + LayerScale, residual add, LN, fc1 + bias + GELU,
// fc2 + LayerScale, residual add).  Here one block is seven kernels:
//
//   bf16 / Q8_0 math                         residual stream `x` is f32 [M, E]
//   1. LayerNorm(x)      -> bf16 (or Q8_0) [M, E]
//   2. QKV GEMM          -> +bias, RoPE on q/k, head-major bf16 q, k, v
//   3. attention         -> token-major bf16 (or Q8_0) [M, E]
//   4. out-proj GEMM     -> x += (acc + b) * ls1
//   5. LayerNorm(x)      -> bf16 (or Q8_0)
//   6. fc1 GEMM          -> gelu(acc + b) bf16 (or Q8_0) [M, F]
//   7. fc2 GEMM          -> x += (acc + b) * ls2
//
// Images are batched into the GEMMs' M dimension (M = images * tokens).  A
// forward for a given (images, grid, buffers, stream) is recorded into a CUDA
// graph on its second call and replayed afterwards.
#include <stdlib.h>

#include <algorithm>

#include <vector>

#include "vestra_b200.h"
#include "vk_abi_internal.h"
#include "vk_internal.h"

using namespace vk;

void host_rotations(const int64_t* pos, size_t n, size_t head_dim, float freq, std::vector<float>& rot);
int prepare_weight(size_t k, size_t n, const float* w_host, int math, float** w32, __nv_bfloat16** w16, int8_t** wq,
                   __half** wd, std::vector<void*>* track);

namespace {

struct Acts {
  __nv_bfloat16 *ln16, *q16, *k16, *att16, *h16;
  __half* v16;  // V is f16: attention's P V product runs in f16
  int8_t *lnq, *attq, *hq;
  __half *lnd, *attd, *hd;
  float *ln32, *q32, *k32, *v32, *att32, *tok32, *h32;
};

void layout_acts(Arena& ar, int math, size_t M, size_t E, size_t F, Acts& a) {
  a = Acts{};
  if (math == VK_MATH_F32) {
    a.ln32 = ar.get<float>(M * E);
    a.q32 = ar.get<float>(M * E);
    a.k32 = ar.get<float>(M * E);
    a.v32 = ar.get<float>(M * E);
    a.att32 = ar.get<float>(M * E);
    a.tok32 = ar.get<float>(M * E);
    a.h32 = ar.get<float>(M * F);
    return;
  }
  a.q16 = ar.get<__nv_bfloat16>(M * E);
  a.k16 = ar.get<__nv_bfloat16>(M * E);
  a.v16 = ar.get<__half>(M * E);
  if (math == VK_MATH_BF16) {
    a.ln16 = ar.get<__nv_bfloat16>(M * E);
    a.att16 = ar.get<__nv_bfloat16>(M * E);
    a.h16 = ar.get<__nv_bfloat16>(M * F);
  } else {
    a.lnq = ar.get<int8_t>(M * E);
    a.lnd = ar.get<__half>(M * E / 32);
    a.attq = ar.get<int8_t>(M * E);
    a.attd = ar.get<__half>(M * E / 32);
    a.hq = ar.get<int8_t>(M * F);
    a.hd = ar.get<__half>(M * F / 32);
  }
}

int ensure_acts(vk_encoder* enc, size_t M, Acts& a) {
  const size_t E = enc->embed, F = enc->cfg.ffn;
  if (M > enc->cap_rows) {
    if (enc->act) {
      cudaDeviceSynchronize();
      cudaFree(enc->act);
      enc->act = nullptr;
      enc->cap_rows = 0;
      for (auto& kv : enc->graphs) cudaGraphExecDestroy(kv.second);
      enc->graphs.clear();
      enc->seen.clear();
    }
    Arena sizing;
    layout_acts(sizing, enc->cfg.math, M, E, F, a);
    VK_TRY_CUDA(cudaMalloc(&enc->act, sizing.off + 256), "encoder activations");
    enc->cap_rows = M;
  }
  Arena ar{enc->act, 0};
  layout_acts(ar, enc->cfg.math, enc->cap_rows, E, F, a);
  return VK_OK;
}

int ensure_rope(vk_encoder* enc, size_t gh, size_t gw) {
  if (enc->rope && enc->rope_h == gh && enc->rope_w == gw) return VK_OK;
  const size_t T = gh * gw + 1;
  std::vector<int64_t> pos(2 * T, 0);
  for (size_t p = 0; p < gh * gw; ++p) {
    pos[2 * (p + 1)] = static_cast<int64_t>(p / gw + 1);
    pos[2 * (p + 1) + 1] = static_cast<int64_t>(p % gw + 1);
  }
  std::vector<float> rot;
  host_rotations(pos.data(), T, 64, enc->cfg.rope_freq, rot);
  if (enc->rope) {
    cudaDeviceSynchronize();
    cudaFree(enc->rope);
    enc->rope = nullptr;
    for (auto& kv : enc->graphs) cudaGraphExecDestroy(kv.second);
    enc->graphs.clear();
    enc->seen.clear();
  }
  // Two layouts of the same values: [t][axis][i](sin, cos) for the f32 RoPE
  // pass, and [axis * 8 + i / 2][t](sin_i, cos_i, sin_i+1, cos_i+1) for the
  // GEMM epilogue, where the 32 threads of a warp hold 32 consecutive tokens
  // (coalesced 16-byte reads, two frequencies each).
  std::vector<float> both(2 * rot.size());
  std::copy(rot.begin(), rot.end(), both.begin());
  for (size_t t = 0; t < T; ++t)
    for (size_t ai = 0; ai < 32; ++ai) {
      const size_t dst = rot.size() + ((ai / 2) * T + t) * 4 + (ai & 1) * 2;
      both[dst] = rot[(t * 32 + ai) * 2];
      both[dst + 1] = rot[(t * 32 + ai) * 2 + 1];
    }
  VK_TRY_CUDA(cudaMalloc(&enc->rope, both.size() * sizeof(float)), "rotation table");
  VK_TRY_CUDA(cudaMemcpy(enc->rope, both.data(), both.size() * sizeof(float), cudaMemcpyHostToDevice), "rotation table");
  enc->rope_h = gh;
  enc->rope_w = gw;
  return VK_OK;
}

size_t rope_tokens(const vk_encoder* enc) { return enc->rope_h * enc->rope_w + 1; }

// Images per attention sequence in layer li: cfg.views for a global
// cross-view layer, else 1.
size_t layer_views(const vk_encoder* enc, size_t li) {
  const int v = enc->cfg.views;
  if (v <= 1 || li >= 64 || ((enc->cfg.global_layers >> li) & 1u) == 0) return 1;
  return static_cast<size_t>(v);
}

// Whether `images` splits into whole groups for every global layer.
bool views_fit(const vk_encoder* enc, size_t images) {
  for (size_t li = 0; li < enc->layers.size(); ++li)
    if (images % layer_views(enc, li) != 0) return false;
  return true;
}

// Enqueues one forward on `s`; returns the number of kernels launched or a
// negative value on a launch error.
int encoder_enqueue(vk_encoder* enc, int* d_err, size_t images, size_t T, const Acts& a, float* x, cudaStream_t s,
                    cudaEvent_t* evs = nullptr) {
  const int E = enc->embed, F = enc->cfg.ffn, H = enc->cfg.heads;
  const int M = static_cast<int>(images * T);
  const float eps = enc->cfg.eps;
  const int math = enc->cfg.math;
  int launches = 0;
#define VK_L(expr)                                      \
  do {                                                  \
    if (evs != nullptr) cudaEventRecord(evs[launches], s); \
    if ((expr) != cudaSuccess) return -1;               \
    ++launches;                                         \
  } while (0)
  for (size_t li = 0; li < enc->layers.size(); ++li) {
    const EncLayer& L = enc->layers[li];
    // A global cross-view layer attends over each group of `views`
    // consecutive images as one sequence (src/specialized.rs:720-757);
    // rows stay image-major, so only the attention's (images, tokens) and
    // the head-major q / k / v layout change.  RoPE keeps per-view positions.
    const size_t V = layer_views(enc, li);
    const size_t ai = images / V, aT = T * V;
    GemmEpi qkv;
    qkv.bias = L.qkv_b;
    qkv.tokens = static_cast<int>(aT);
    qkv.rope_tokens = static_cast<int>(T);
    qkv.heads = H;
    qkv.qkn = L.qkn;
    qkv.qkn_eps = eps;
    GemmEpi proj;
    proj.bias = L.proj_b;
    proj.scale = L.ls1;
    proj.resid = x;
    proj.ldo = E;
    GemmEpi fc1;
    fc1.bias = L.fc1_b;
    fc1.ldo = F;
    GemmEpi fc2;
    fc2.bias = L.fc2_b;
    fc2.scale = L.ls2;
    fc2.resid = x;
    fc2.ldo = E;
    if (math == VK_MATH_BF16) {
      qkv.q = a.q16; qkv.k = a.k16; qkv.v = a.v16; qkv.rope = enc->rope + (rope_tokens(enc) * 64);
      fc1.out = a.h16;
      VK_L(layernorm_f32(x, nullptr, a.ln16, nullptr, nullptr, M, E, L.ln1_g, L.ln1_b, eps, s));
      VK_L(gemm_bf16_tc(a.ln16, L.qkv_w16, M, 3 * E, E, EPI_QKV_BF16, qkv, d_err, s));
      // Q/K-normalised heads (DA3's late blocks) give unit-variance q and k,
      // so sharper softmax rows whose f16 P rounding shows more in the
      // update: those layers take the split P V product
      VK_L(attention_bf16(a.q16, a.k16, a.v16, (int)ai, H, (int)aT, ATTN_OUT_TOKEN_BF16, a.att16, nullptr, d_err, s,
                          L.qkn != nullptr));
      VK_L(gemm_bf16_tc(a.att16, L.proj_w16, M, E, E, EPI_RESID, proj, d_err, s));
      VK_L(layernorm_f32(x, nullptr, a.ln16, nullptr, nullptr, M, E, L.ln2_g, L.ln2_b, eps, s));
      VK_L(gemm_bf16_tc(a.ln16, L.fc1_w16, M, F, E, EPI_BF16_GELU, fc1, d_err, s));
      VK_L(gemm_bf16_tc(a.h16, L.fc2_w16, M, E, F, EPI_RESID, fc2, d_err, s));
    } else if (math == VK_MATH_Q8_0) {
      qkv.q = a.q16; qkv.k = a.k16; qkv.v = a.v16; qkv.rope = enc->rope + (rope_tokens(enc) * 64);
      fc1.q8 = a.hq;
      fc1.q8d = a.hd;
      VK_L(layernorm_f32(x, nullptr, nullptr, a.lnq, a.lnd, M, E, L.ln1_g, L.ln1_b, eps, s));
      VK_L(gemm_q8_tc(a.lnq, a.lnd, L.qkv_q, L.qkv_d, M, 3 * E, E, EPI_QKV_BF16, qkv, nullptr, d_err, s));
      VK_L(attention_bf16(a.q16, a.k16, a.v16, (int)ai, H, (int)aT, ATTN_OUT_TOKEN_Q8, a.attq, a.attd, d_err, s));
      VK_L(gemm_q8_tc(a.attq, a.attd, L.proj_q, L.proj_d, M, E, E, EPI_RESID, proj, nullptr, d_err, s));
      VK_L(layernorm_f32(x, nullptr, nullptr, a.lnq, a.lnd, M, E, L.ln2_g, L.ln2_b, eps, s));
      VK_L(gemm_q8_tc(a.lnq, a.lnd, L.fc1_q, L.fc1_d, M, F, E, EPI_Q8_GELU, fc1, nullptr, d_err, s));
      VK_L(gemm_q8_tc(a.hq, a.hd, L.fc2_q, L.fc2_d, M, E, F, EPI_RESID, fc2, nullptr, d_err, s));
    } else {
      qkv.q = a.q32; qkv.k = a.k32; qkv.v = a.v32;
      fc1.out = a.h32;
      VK_L(layernorm_f32(x, a.ln32, nullptr, nullptr, nullptr, M, E, L.ln1_g, L.ln1_b, eps, s));
      VK_L(gemm_f32_simt(a.ln32, L.qkv_w32, M, 3 * E, E, EPI_QKV_F32, qkv, s));
      if (L.qkn != nullptr) {  // rows of [ai * H, aT, 64]; the table row is row % T
        VK_L(qk_norm_rope_f32(a.q32, a.k32, (int)(ai * H * (aT / T)), (int)T, L.qkn, L.qkn + 64, L.qkn + 128,
                              L.qkn + 192, enc->rope, eps, s));
      } else {
        VK_L(rope2d_f32(a.q32, (int)ai * H, (int)aT, 64, enc->rope, s, (int)T));
        VK_L(rope2d_f32(a.k32, (int)ai * H, (int)aT, 64, enc->rope, s, (int)T));
      }
      VK_L(attention_f32(a.q32, a.k32, a.v32, (int)ai * H, (int)aT, 64, a.att32, s));
      VK_L(hnd_to_token_f32(a.att32, a.tok32, (int)ai, H, (int)aT, s));
      VK_L(gemm_f32_simt(a.tok32, L.proj_w32, M, E, E, EPI_RESID, proj, s));
      VK_L(layernorm_f32(x, a.ln32, nullptr, nullptr, nullptr, M, E, L.ln2_g, L.ln2_b, eps, s));
      VK_L(gemm_f32_simt(a.ln32, L.fc1_w32, M, F, E, EPI_F32_GELU, fc1, s));
      VK_L(gemm_f32_simt(a.h32, L.fc2_w32, M, E, F, EPI_RESID, fc2, s));
    }
  }
#undef VK_L
  if (evs != nullptr) cudaEventRecord(evs[launches], s);
  return launches;
}

void free_encoder(vk_encoder* enc) {
  if (!enc) return;
  cudaSetDevice(enc->device);
  cudaDeviceSynchronize();
  for (auto& kv : enc->graphs) cudaGraphExecDestroy(kv.second);
  for (void* p : enc->allocations) cudaFree(p);
  if (enc->act) cudaFree(enc->act);
  if (enc->rope) cudaFree(enc->rope);
  for (float* p : enc->slots)
    if (p) cudaFree(p);
  for (cudaStream_t st : {enc->h2d, enc->d2h, enc->comp})
    if (st) cudaStreamDestroy(st);
  for (int i = 0; i < 3; ++i)
    for (cudaEvent_t ev : {enc->slot_free[i], enc->slot_in[i], enc->slot_out[i]})
      if (ev) cudaEventDestroy(ev);
  if (enc->dev_tail) cudaEventDestroy(enc->dev_tail);
  delete enc;
}

}  // namespace

extern "C" int vk_encoder_prepare(vk_ctx* ctx, const vk_encoder_config* cfg, const vk_layer_weights* layers_host,
                                  vk_encoder** out) {
  if (!ctx || !cfg || !layers_host || !out) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_encoder_prepare: NULL argument");
  *out = nullptr;
  cudaSetDevice(ctx->device);
  if (cfg->views < 0) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_encoder_prepare: negative views");
  if (cfg->layers <= 0 || cfg->heads <= 0 || cfg->ffn <= 0)
    return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_encoder_prepare: empty configuration");
  const int E = cfg->heads * 64, F = cfg->ffn;
  if (cfg->math != VK_MATH_F32 && cfg->math != VK_MATH_BF16 && cfg->math != VK_MATH_Q8_0)
    return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_encoder_prepare: unknown math %d", cfg->math);
  if (cfg->math != VK_MATH_F32 && (E % 128 != 0 || F % 128 != 0 || E > 1024))
    return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_encoder_prepare: tensor-core paths need embed, ffn %% 128 == 0, embed <= 1024");
  vk_encoder* enc = new vk_encoder();
  enc->device = ctx->device;
  enc->cfg = *cfg;
  enc->embed = E;
  enc->layers.resize(cfg->layers);
  auto vec = [&](const float* src, size_t n, float** dst) -> int {
    if (src == nullptr) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_encoder_prepare: NULL layer vector");
    VK_TRY_CUDA(cudaMalloc(reinterpret_cast<void**>(dst), n * sizeof(float)), "encoder vector");
    enc->allocations.push_back(*dst);
    VK_TRY_CUDA(cudaMemcpy(*dst, src, n * sizeof(float), cudaMemcpyHostToDevice), "encoder vector");
    return VK_OK;
  };
  int st = VK_OK;
  for (int l = 0; l < cfg->layers && st == VK_OK; ++l) {
    const vk_layer_weights& w = layers_host[l];
    EncLayer& L = enc->layers[l];
    L = EncLayer{};
    if (st == VK_OK) st = vec(w.ln1_gamma, E, &L.ln1_g);
    if (st == VK_OK) st = vec(w.ln1_beta, E, &L.ln1_b);
    if (st == VK_OK) st = vec(w.ln2_gamma, E, &L.ln2_g);
    if (st == VK_OK) st = vec(w.ln2_beta, E, &L.ln2_b);
    if (st == VK_OK) st = vec(w.qkv_bias, 3 * E, &L.qkv_b);
    if (st == VK_OK) st = vec(w.proj_bias, E, &L.proj_b);
    if (st == VK_OK) st = vec(w.ls1, E, &L.ls1);
    if (st == VK_OK) st = vec(w.fc1_bias, F, &L.fc1_b);
    if (st == VK_OK) st = vec(w.fc2_bias, E, &L.fc2_b);
    if (st == VK_OK) st = vec(w.ls2, E, &L.ls2);
    const int nq = (w.q_norm_gamma != nullptr) + (w.q_norm_beta != nullptr) + (w.k_norm_gamma != nullptr) +
                   (w.k_norm_beta != nullptr);
    if (st == VK_OK && nq != 0 && nq != 4)
      st = vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_encoder_prepare: layer %d sets only some Q/K norm vectors", l);
    if (st == VK_OK && nq == 4 && cfg->math == VK_MATH_Q8_0)
      st = vk_fail(VK_UNSUPPORTED_SHAPE, "vk_encoder_prepare: Q/K LayerNorm needs bf16 or f32 math");
    if (st == VK_OK && nq == 4) {
      float qkn[256];
      for (int i = 0; i < 64; ++i) {
        qkn[i] = w.q_norm_gamma[i];
        qkn[64 + i] = w.q_norm_beta[i];
        qkn[128 + i] = w.k_norm_gamma[i];
        qkn[192 + i] = w.k_norm_beta[i];
      }
      st = vec(qkn, 256, &L.qkn);
    }
    if (st == VK_OK && (!w.qkv_weight || !w.proj_weight || !w.fc1_weight || !w.fc2_weight))
      st = vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_encoder_prepare: NULL layer weight");
    if (st == VK_OK)
      st = prepare_weight(E, 3 * E, w.qkv_weight, cfg->math, &L.qkv_w32, &L.qkv_w16, &L.qkv_q, &L.qkv_d, &enc->allocations);
    if (st == VK_OK)
      st = prepare_weight(E, E, w.proj_weight, cfg->math, &L.proj_w32, &L.proj_w16, &L.proj_q, &L.proj_d, &enc->allocations);
    if (st == VK_OK)
      st = prepare_weight(E, F, w.fc1_weight, cfg->math, &L.fc1_w32, &L.fc1_w16, &L.fc1_q, &L.fc1_d, &enc->allocations);
    if (st == VK_OK)
      st = prepare_weight(F, E, w.fc2_weight, cfg->math, &L.fc2_w32, &L.fc2_w16, &L.fc2_q, &L.fc2_d, &enc->allocations);
  }
  if (st != VK_OK) {
    free_encoder(enc);
    return st;
  }
  *out = enc;
  return VK_OK;
}

static int forward_on_stream(vk_ctx* ctx, vk_encoder* enc, size_t images, size_t gh, size_t gw, const float* in,
                             float* out, cudaStream_t s) {
  const size_t T = gh * gw + 1, E = enc->embed;
  const size_t M = images * T;
  Acts a;
  VK_TRY(ensure_acts(enc, M, a));
  VK_TRY(ensure_rope(enc, gh, gw));
  const auto key = std::make_tuple(images, gh, gw, static_cast<const void*>(in), static_cast<void*>(out), s);
  const bool use_graph = s != nullptr && getenv("VK_NO_GRAPH") == nullptr;
  auto it = enc->graphs.find(key);
  if (use_graph && it != enc->graphs.end()) {
    VK_TRY_CUDA(cudaGraphLaunch(it->second, s), "encoder graph launch");
    return VK_OK;
  }
  const bool capture = use_graph && enc->seen[key] >= 1;
  if (capture) VK_TRY_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "encoder capture");
  if (in != out) {
    cudaError_t e = cudaMemcpyAsync(out, in, M * E * sizeof(float), cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) {
      if (capture) {
        cudaGraph_t g;
        cudaStreamEndCapture(s, &g);
      }
      return vk_cuda_status(e, "encoder input copy");
    }
  }
  const int n = encoder_enqueue(enc, ctx->d_err, images, T, a, out, s);
  if (capture) {
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(s, &g);
    if (n < 0 || e != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      return vk_fail(VK_ERR_CUDA, "encoder capture failed: %s", cudaGetErrorString(e != cudaSuccess ? e : cudaGetLastError()));
    }
    cudaGraphExec_t ex = nullptr;
    e = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return vk_cuda_status(e, "encoder graph instantiate");
    enc->graphs[key] = ex;
    VK_TRY_CUDA(cudaGraphLaunch(ex, s), "encoder graph launch");
  } else {
    if (n < 0) return vk_cuda_status(cudaGetLastError(), "encoder launch");
    enc->seen[key] += 1;
  }
  enc->last_launches = n;
  return VK_OK;
}

extern "C" int vk_encoder_forward(vk_ctx* ctx, vk_encoder* enc, size_t images, size_t grid_h, size_t grid_w,
                                  const float* tokens_dev, float* out_dev) {
  if (!ctx || !enc || !tokens_dev || !out_dev) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_encoder_forward: NULL argument");
  cudaSetDevice(ctx->device);
  if (images == 0) return VK_OK;
  if (grid_h == 0 || grid_w == 0) return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_encoder_forward: empty patch grid");
  // after any host-pipeline compute still using the shared activations
  if (enc->comp) {
    for (cudaEvent_t ev : enc->slot_out)
      if (ev) VK_TRY_CUDA(cudaStreamWaitEvent(ctx->stream, ev, 0), "vk_encoder_forward ordering");
  }
  if (!views_fit(enc, images))
    return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_encoder_forward: %zu images are not whole groups of %d views", images,
                   enc->cfg.views);
  VK_TRY(forward_on_stream(ctx, enc, images, grid_h, grid_w, tokens_dev, out_dev, ctx->stream));
  if (enc->dev_tail) VK_TRY_CUDA(cudaEventRecord(enc->dev_tail, ctx->stream), "vk_encoder_forward ordering");
  return VK_OK;
}

// Host tokens in, host result out, in chunks of `chunk` images through the
// three-slot ring: H2D on one stream, the encoder on another, D2H on a
// third, so the copies of one chunk overlap the compute of its neighbours.
// The ring continues across calls, so back-to-back calls overlap too.
static int host_pipeline(vk_ctx* ctx, vk_encoder* enc, size_t images, size_t grid_h, size_t grid_w,
                         const float* tokens_host, float* out_host, bool wait, const char* name) {
  if (!ctx || !enc || !tokens_host || !out_host) return vk_fail(VK_ERR_INVALID_ARGUMENT, "%s: NULL argument", name);
  cudaSetDevice(ctx->device);
  if (images == 0) return VK_OK;
  if (grid_h == 0 || grid_w == 0) return vk_fail(VK_UNSUPPORTED_SHAPE, "%s: empty patch grid", name);
  if (!views_fit(enc, images))
    return vk_fail(VK_UNSUPPORTED_SHAPE, "%s: %zu images are not whole groups of %d views", name, images,
                   enc->cfg.views);
  const size_t T = grid_h * grid_w + 1, E = enc->embed;
  // A waiting call overlaps copies with compute only inside itself, so it
  // cuts the batch into 16-image chunks; back-to-back asynchronous calls
  // overlap with each other, so each takes its batch whole (up to 64 images,
  // where the GEMMs already fill the GPU), which keeps every GEMM large.
  size_t chunk = wait ? 16 : 64;
  if (const char* c = getenv("VK_E2E_CHUNK")) chunk = static_cast<size_t>(atoi(c));
  if (chunk == 0 || chunk > images) chunk = images;
  if (enc->cfg.views > 1) chunk = (chunk + enc->cfg.views - 1) / enc->cfg.views * enc->cfg.views;  // whole groups
  if (chunk > images) chunk = images;
  const size_t rows = chunk * T;
  if (!enc->comp) {
    for (cudaStream_t* st : {&enc->comp, &enc->h2d, &enc->d2h})
      VK_TRY_CUDA(cudaStreamCreateWithFlags(st, cudaStreamNonBlocking), "pipeline stream");
    for (int i = 0; i < 3; ++i)
      for (cudaEvent_t* ev : {&enc->slot_free[i], &enc->slot_in[i], &enc->slot_out[i]})
        VK_TRY_CUDA(cudaEventCreateWithFlags(ev, cudaEventDisableTiming), "pipeline event");
    VK_TRY_CUDA(cudaEventCreateWithFlags(&enc->dev_tail, cudaEventDisableTiming), "pipeline event");
  }
  if (rows > enc->slot_rows) {
    cudaDeviceSynchronize();
    for (float*& p : enc->slots) {
      if (p) cudaFree(p);
      p = nullptr;
    }
    for (float*& p : enc->slots) VK_TRY_CUDA(cudaMalloc(&p, rows * E * sizeof(float)), "pipeline slot");
    enc->slot_rows = rows;
  }
  // the compute follows earlier device-path forwards on the context stream
  VK_TRY_CUDA(cudaStreamWaitEvent(enc->comp, enc->dev_tail, 0), name);
  const size_t nchunks = (images + chunk - 1) / chunk;
  size_t last = 0;
  for (size_t c = 0; c < nchunks; ++c) {
    const size_t im0 = c * chunk, nim = (images - im0 < chunk) ? images - im0 : chunk;
    const size_t k = enc->next_slot++ % 3;
    float* slot = enc->slots[k];
    const size_t bytes = nim * T * E * sizeof(float);
    VK_TRY_CUDA(cudaStreamWaitEvent(enc->h2d, enc->slot_free[k], 0), name);  // the slot's last D2H is done
    VK_TRY_CUDA(cudaMemcpyAsync(slot, tokens_host + im0 * T * E, bytes, cudaMemcpyHostToDevice, enc->h2d), name);
    VK_TRY_CUDA(cudaEventRecord(enc->slot_in[k], enc->h2d), name);
    VK_TRY_CUDA(cudaStreamWaitEvent(enc->comp, enc->slot_in[k], 0), name);
    VK_TRY(forward_on_stream(ctx, enc, nim, grid_h, grid_w, slot, slot, enc->comp));
    VK_TRY_CUDA(cudaEventRecord(enc->slot_out[k], enc->comp), name);
    VK_TRY_CUDA(cudaStreamWaitEvent(enc->d2h, enc->slot_out[k], 0), name);
    VK_TRY_CUDA(cudaMemcpyAsync(out_host + im0 * T * E, slot, bytes, cudaMemcpyDeviceToHost, enc->d2h), name);
    VK_TRY_CUDA(cudaEventRecord(enc->slot_free[k], enc->d2h), name);
    last = k;
  }
  // later work on the context stream (and vk_synchronize) sees the result
  VK_TRY_CUDA(cudaStreamWaitEvent(ctx->stream, enc->slot_free[last], 0), name);
  if (wait) VK_TRY_CUDA(cudaStreamSynchronize(enc->d2h), name);
  return VK_OK;
}

extern "C" int vk_encoder_forward_host(vk_ctx* ctx, vk_encoder* enc, size_t images, size_t grid_h, size_t grid_w,
                                       const float* tokens_host, float* out_host) {
  return host_pipeline(ctx, enc, images, grid_h, grid_w, tokens_host, out_host, true, "vk_encoder_forward_host");
}

extern "C" int vk_encoder_forward_host_async(vk_ctx* ctx, vk_encoder* enc, size_t images, size_t grid_h,
                                             size_t grid_w, const float* tokens_host, float* out_host) {
  return host_pipeline(ctx, enc, images, grid_h, grid_w, tokens_host, out_host, false,
                       "vk_encoder_forward_host_async");
}

extern "C" int vk_encoder_profile(vk_ctx* ctx, vk_encoder* enc, size_t images, size_t grid_h, size_t grid_w,
                                  const float* tokens_dev, float* out_dev, float* ms_per_slot, int slots) {
  if (!ctx || !enc || !tokens_dev || !out_dev || !ms_per_slot)
    return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_encoder_profile: NULL argument");
  cudaSetDevice(ctx->device);
  if (images == 0 || grid_h == 0 || grid_w == 0) return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_encoder_profile: empty shape");
  if (!views_fit(enc, images)) return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_encoder_profile: images not whole view groups");
  const size_t T = grid_h * grid_w + 1, M = images * T;
  Acts a;
  VK_TRY(ensure_acts(enc, M, a));
  VK_TRY(ensure_rope(enc, grid_h, grid_w));
  const int per_layer = enc->cfg.math == VK_MATH_F32 ? 10 : 7;
  if (slots < per_layer) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_encoder_profile: need %d slots", per_layer);
  // launch i of the forward -> (slot); an f32 layer with Q/K LayerNorm runs
  // one fused norm + RoPE kernel in the two RoPE slots (it is booked to the first)
  std::vector<int> slot_of;
  for (const EncLayer& L : enc->layers)
    for (int j = 0; j < per_layer; ++j)
      if (!(enc->cfg.math == VK_MATH_F32 && L.qkn != nullptr && j == 3)) slot_of.push_back(j);
  const int total = static_cast<int>(slot_of.size());
  std::vector<cudaEvent_t> evs(total + 1);
  for (auto& e : evs) VK_TRY_CUDA(cudaEventCreate(&e), "profile event");
  if (tokens_dev != out_dev)
    VK_TRY_CUDA(cudaMemcpyAsync(out_dev, tokens_dev, M * enc->embed * sizeof(float), cudaMemcpyDeviceToDevice, ctx->stream),
                "profile input copy");
  const int n = encoder_enqueue(enc, ctx->d_err, images, T, a, out_dev, ctx->stream, evs.data());
  cudaError_t e = cudaStreamSynchronize(ctx->stream);
  for (int i = 0; i < slots; ++i) ms_per_slot[i] = 0.0f;
  if (n == total && e == cudaSuccess)
    for (int i = 0; i < n; ++i) {
      float ms = 0.0f;
      cudaEventElapsedTime(&ms, evs[i], evs[i + 1]);
      ms_per_slot[slot_of[i]] += ms;
    }
  for (auto& ev : evs) cudaEventDestroy(ev);
  if (e != cudaSuccess) return vk_cuda_status(e, "vk_encoder_profile");
  if (n != total) return vk_fail(VK_ERR_CUDA, "vk_encoder_profile: launch failed");
  return VK_OK;
}

extern "C" int vk_encoder_last_launches(const vk_encoder* enc) { return enc ? enc->last_launches : 0; }

extern "C" int vk_encoder_release(vk_encoder* enc) {
  free_encoder(enc);
  return VK_OK;
}
