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
//  - every call looks up the array's device address on the current device
//    with cudaGetSymbolAddress; make the first call on a device before any
//    stream capture (it loads the module);
//  - the stream must belong to the current device (VK_ERR_INVALID_ARGUMENT
//    otherwise);
//  - all calls share the one array: calls whose work overlaps on the GPU (on
//    different streams without ordering) race on it;
//  - the array keeps the last call's contents; each call overwrites every byte
//    it reads before reading it, so nothing needs clearing;
//  - device-side wait timeouts are not reported by this entry point (it has
//    no context to carry an error word): a kernel that gave up a bounded wait
//    leaves c partly written and the call has already returned VK_OK.
#include "vestra_b200.h"
#include "vk_abi_internal.h"
#include "vk_internal.h"

#define VK_NOALLOC_SCRATCH_BYTES (8u << 20)

static __device__ __align__(256) uint8_t g_noalloc_scratch[VK_NOALLOC_SCRATCH_BYTES];

// Device address of the scratch array on the current device.  Looked up on
// every call (cheap once the module is loaded), so a context that was reset
// and re-created never hands out a stale address.
static uint8_t* scratch_address(int* status) {
  // In host code the array's name is only a stand-in; kernels need the
  // device address, looked up with the device current.
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr) {
    *status = vk_cuda_status(e != cudaSuccess ? e : cudaErrorInvalidSymbol, "vk_gemm_q8_0_noalloc: scratch lookup");
    return nullptr;
  }
  *status = VK_OK;
  return static_cast<uint8_t*>(p);
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
  if (stream != nullptr) {  // the stream must belong to the current device
    int sdev = -1;
    e = cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev);
    if (e != cudaSuccess) return vk_cuda_status(e, "vk_gemm_q8_0_noalloc: stream device");
    if (sdev != device)
      return vk_fail(VK_ERR_INVALID_ARGUMENT,
                     "vk_gemm_q8_0_noalloc: stream belongs to device %d, current device is %d", sdev, device);
  }
  int st = VK_OK;
  uint8_t* base = scratch_address(&st);
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
