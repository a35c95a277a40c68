// vk_noalloc.cu -- vk_gemm_q8_0_noalloc: the Q8_0 GEMM entry point for
// callers that must not allocate device memory.
//
// Some callers cannot call cudaMalloc at the point where they run the GEMM:
// real-time or embedded hosts whose device memory is fully budgeted up
// front, and plugins that live inside an engine that owns every allocation.
// vk_gemm_q8_0 needs scratch to unpack the 34-byte BlockQ8_0 records into the
// split int8 / f16 arrays its tensor-core kernel reads, and takes it from a
// context workspace that grows with cudaMalloc.  This variant takes no
// context and unpacks into a fixed array in the library's own device memory,
// declared below.
//
// Limits and behaviour:
//  - the scratch holds at most VK_NOALLOC_SCRATCH_BYTES (8 MiB):
//      (m + n) * k  bytes of int8 quants  +  (m + n) * (k / 32) * 2 bytes of scales
//    (each section rounded up to 256 bytes); larger problems are rejected
//    with VK_UNSUPPORTED_SHAPE and a message;
//  - every GPU that loads the library holds the 8 MiB until the process exits;
//  - the first call on a device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current); make that first call
//    before any stream capture;
//  - all calls share the one array: calls whose work overlaps on the GPU (on
//    different streams without ordering) race on it;
//  - the array keeps the last call's contents; each call overwrites every byte
//    it reads before reading it, so nothing needs clearing;
//  - device-side wait timeouts are not reported by this entry point (it has
//    no context to carry an error word).
#include <mutex>

#include "vestra_b200.h"
#include "vk_abi_internal.h"
#include "vk_internal.h"

#define VK_NOALLOC_SCRATCH_BYTES (8u << 20)
#define VK_NOALLOC_MAX_DEVICES 64

static __device__ __align__(256) uint8_t g_noalloc_scratch[VK_NOALLOC_SCRATCH_BYTES];

// Device address of the scratch array on `device` (the current device).
static uint8_t* scratch_address(int device, int* status) {
  static std::mutex mu;
  static uint8_t* addr[VK_NOALLOC_MAX_DEVICES] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (device < 0 || device >= VK_NOALLOC_MAX_DEVICES) {
    *status = vk_fail(VK_ERR_NO_DEVICE, "vk_gemm_q8_0_noalloc: device %d out of range", device);
    return nullptr;
  }
  if (addr[device] == nullptr) {
    // In host code the array's name is only a stand-in; kernels need the
    // device address, looked up once per device with that device current.
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *status = vk_cuda_status(e != cudaSuccess ? e : cudaErrorInvalidSymbol, "vk_gemm_q8_0_noalloc: scratch lookup");
      return nullptr;
    }
    addr[device] = static_cast<uint8_t*>(p);
  }
  *status = VK_OK;
  return addr[device];
}

extern "C" int vk_gemm_q8_0_noalloc(void* stream, size_t m, size_t n, size_t k, const vk_block_q8_0* a_q,
                                    const vk_block_q8_0* b_q, float* c) {
  if (m == 0 || n == 0) return VK_OK;
  if (!a_q || !b_q || !c) return vk_fail(VK_ERR_INVALID_ARGUMENT, "vk_gemm_q8_0_noalloc: NULL buffer");
  if (k == 0 || k % 128 != 0 || n % 128 != 0)
    return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_gemm_q8_0_noalloc: needs k %% 128 == 0 and n %% 128 == 0 (k=%zu, n=%zu)",
                   k, n);
  // bound each factor first so that the byte counts below cannot wrap
  if (m > VK_NOALLOC_SCRATCH_BYTES || n > VK_NOALLOC_SCRATCH_BYTES || k > VK_NOALLOC_SCRATCH_BYTES)
    return vk_fail(VK_UNSUPPORTED_SHAPE, "vk_gemm_q8_0_noalloc: m=%zu n=%zu k=%zu exceeds the fixed %u-byte scratch", m,
                   n, k, VK_NOALLOC_SCRATCH_BYTES);
  const size_t nb = k / 32;
  auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
  const size_t a_q_bytes = up(m * k), b_q_bytes = up(n * k), a_d_bytes = up(m * nb * 2), b_d_bytes = up(n * nb * 2);
  const size_t need = a_q_bytes + b_q_bytes + a_d_bytes + b_d_bytes;
  if (need > VK_NOALLOC_SCRATCH_BYTES)
    return vk_fail(VK_UNSUPPORTED_SHAPE,
                   "vk_gemm_q8_0_noalloc: m=%zu n=%zu k=%zu needs %zu bytes of scratch, more than the fixed %u",
                   m, n, k, need, VK_NOALLOC_SCRATCH_BYTES);
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return vk_cuda_status(e, "vk_gemm_q8_0_noalloc");
  int st = VK_OK;
  uint8_t* base = scratch_address(device, &st);
  if (base == nullptr) return st;
  int8_t* aq = reinterpret_cast<int8_t*>(base);
  int8_t* bq = reinterpret_cast<int8_t*>(base + a_q_bytes);
  __half* ad = reinterpret_cast<__half*>(base + a_q_bytes + b_q_bytes);
  __half* bd = reinterpret_cast<__half*>(base + a_q_bytes + b_q_bytes + a_d_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  e = vk::unpack_blocks_q8_0(a_q, m * nb, aq, ad, s);
  if (e == cudaSuccess) e = vk::unpack_blocks_q8_0(b_q, n * nb, bq, bd, s);
  if (e != cudaSuccess) return vk_cuda_status(e, "vk_gemm_q8_0_noalloc: unpack");
  vk::GemmEpi epi;
  epi.out = c;
  epi.ldo = static_cast<int64_t>(n);
  return vk_cuda_status(vk::gemm_q8_tc(aq, ad, bq, bd, (int)m, (int)n, (int)k, vk::EPI_F32, epi, nullptr, nullptr, s),
                        "vk_gemm_q8_0_noalloc");
}
