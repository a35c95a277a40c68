// vk_common.cuh -- sm_100a building blocks shared by the vestra B200 kernels:
// mbarriers with bounded waits, TMA tile loads, tcgen05 (UMMA/TMEM) wrappers,
// and the device error word that replaces traps.
//
// Every spin-wait here gives up after VK_WAIT_NS nanoseconds of %globaltimer,
// records a code in the caller's error word and returns false; the kernels
// then leave their loops, release TMEM and exit so the context stays usable.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef VK_WAIT_NS
#define VK_WAIT_NS 1000000000ull  // one second
#endif

// Error codes written to the device error word (first writer wins).
enum : int {
  VK_DEV_OK = 0,
  VK_DEV_TIMEOUT_PRODUCER = 0x101,
  VK_DEV_TIMEOUT_MMA = 0x102,
  VK_DEV_TIMEOUT_EPILOGUE = 0x103,
  VK_DEV_TIMEOUT_OTHER = 0x104,
};

namespace vk {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
// Programmatic dependent launch: a kernel launched with the programmatic
// stream-serialization attribute is scheduled as the previous kernel's CTAs
// exit, not after the whole grid.  It sets up (barriers, TMEM, descriptor
// prefetch), then waits here until the previous grid has completed and its
// writes are visible, before touching global memory.  (No kernel triggers
// its dependents early: measured, that made the chain slower.)  Without the
// attribute the wait returns at once.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel in the stream be scheduled once every CTA of this grid
// has executed it (or exited).  The persistent kernels issue it when a CTA
// starts its last unit of work, and only for small grids (a few rounds of
// work per CTA, as with 8 images per GPU), so that the next kernel's CTAs
// take the SMs of CTAs that finish early.  Measured on the 12-layer
// forward: +2.2% at 8 images with a 4-round limit, a further +0.5% with 8
// rounds (fc1's 5 rounds at 8 images), -1.8% at 64 if issued there (where
// the grids have 9 or more rounds and it is not).  Every
// CTA of this grid is resident by the time the dependents launch, so they
// cannot starve it; their griddepcontrol.wait still waits for this grid to
// complete.
constexpr int VK_EARLY_LAUNCH_ROUNDS = 8;
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for the phase with the given parity.  Returns false (and records
// `code`) after VK_WAIT_NS; also returns false at once when another thread of
// the grid already recorded an error, so a failed kernel drains quickly.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(a, parity)) return true;
    if ((it & 255u) == 0) {
      if (err && *((volatile int*)err) != 0) return false;
      if (globaltimer() - t0 > VK_WAIT_NS) {
        record_error(err, code);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const void* desc) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(desc)) : "memory");
}
// 2D tiled bulk-tensor load (no multicast) into shared memory, completing
// `bytes` on the mbarrier.  x is the innermost coordinate (elements).
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* desc, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* desc, uint64_t* bar,
                                            int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// TMA stores from shared memory (bulk-group completion).  The staging writes
// are made visible to the async proxy with fence_proxy_async first.
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tma_store_2d(const void* desc, const void* smem_src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(desc)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const void* desc, const void* smem_src, int32_t x, int32_t y,
                                             int32_t z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(desc)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}
// global[tile] += smem tile (f32 add performed at L2, one rounding per element).
__device__ __forceinline__ void tma_reduce_add_2d(const void* desc, const void* smem_src, int32_t x, int32_t y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(desc)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------- clusters
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// All threads of all CTAs of the cluster (also orders mbarrier inits).
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the same variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// 2D tiled load for a CTA pair (no multicast): data lands in this CTA's
// shared memory, completion is signalled on the mbarrier at cluster address
// `bar` (the leader CTA's barrier).
__device__ __forceinline__ void tma_load_2d_cg2(void* smem_dst, const void* desc, uint32_t bar, int32_t x,
                                                int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, bf16/f16 inputs, f32 accumulate.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Pair-wide variants: TMEM is allocated on both SMs of the CTA pair, the
// MMA (issued by the leader CTA) spans both, commits arrive on both CTAs'
// barriers at the same offset (cta_mask 0b11).
__device__ __forceinline__ void tmem_alloc_cg2(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_cg2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_cg2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma_f16_cg2(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit_cg2_mc(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T (A operand read from tensor memory).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, signed int8 inputs, s32 accumulate.
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier once every previously issued tcgen05.mma of this
// thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// K-major operand tile whose rows are 128 bytes, written by TMA with the
// 128-byte swizzle: 8-row groups are 1024 bytes apart (SBO), the layout code
// 2 is SWIZZLE_128B and bit 46 is the sm_100 descriptor version.
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;              // LBO (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;      // SBO
  d |= static_cast<uint64_t>(1u) << 46;              // version
  d |= static_cast<uint64_t>(2u) << 61;              // SWIZZLE_128B
  return d;
}

// MN-major operand tile (rows along K, 128-byte rows along M/N) written by
// TMA with the 128-byte swizzle: 8-row groups along K are 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_mn_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;              // LBO (one 64-element atom along N)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;      // SBO: next 8 rows along K
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor: kind::f16 with bf16 A/B, f32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}
// As idesc_bf16 with B MN-major (B rows run along K).
__host__ __device__ constexpr uint32_t idesc_bf16_bmn(int M, int N) {
  return idesc_bf16(M, N) | (1u << 16);
}
// kind::f16 with f16 A/B (A and B of one MMA must share the type), f32 D,
// A K-major and B MN-major.
__host__ __device__ constexpr uint32_t idesc_f16_bmn(int M, int N) {
  return (1u << 4) | (1u << 16) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}
// Instruction descriptor: kind::i8 with signed A/B, s32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_s8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// 32 lanes x 32 columns of 32-bit TMEM words: thread i of the warp receives
// lane (base_lane + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 32 lanes x 32 columns store from registers into TMEM.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// 32 lanes x 16 columns store from registers into TMEM.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// A&S 7.1.26 erf and the exact-erf GELU of the reference (0.5 x (1 + erf(x/sqrt 2))).
__device__ __forceinline__ float erf_as(float x) {
  const float s = (__float_as_uint(x) >> 31) ? -1.0f : 1.0f;
  x = fabsf(x);
  const float t = 1.0f / (1.0f + 0.3275911f * x);
  const float poly =
      ((((1.0614054f * t - 1.453152f) * t) + 1.4214137f) * t - 0.28449674f) * t + 0.2548296f;
  const float y = 1.0f - poly * t * expf(-x * x);
  return s * y;
}
__device__ __forceinline__ float gelu_erf(float v) {
  return 0.5f * v * (1.0f + erf_as(v * 0.70710678118654752440f));
}

// The same GELU with the fast exponential and division, for results that are
// rounded to bf16 right after (error far below half a bf16 ulp).
// 2^x on the FMA pipe (offloads the MUFU unit): x = n + f with n the nearest
// integer (rounded through the 1.5 * 2^23 shift) and f in [-0.5, 0.5]; 2^f
// from a degree-4 polynomial fitted here for relative error (max 2.7e-6 on
// [-0.5, 0.5]); 2^n is added to the exponent field.  Valid for x in
// [-126, 127]; inputs below -126 are clamped (result ~1e-38).
__device__ __forceinline__ float exp2_poly(float x) {
  x = fmaxf(x, -126.0f);
  const float t = x + 12582912.0f;
  const float f = x - (t - 12582912.0f);
  float p = fmaf(0.009571120f, f, 0.055920936f);
  p = fmaf(p, f, 0.24024746f);
  p = fmaf(p, f, 0.69312137f);
  p = fmaf(p, f, 0.99999923f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// 2^x for two lanes on the FMA pipe (packed f32x2), to take part of a
// softmax's exponentials off the MUFU unit.  Cody-Waite split x = n + f with
// n = rint(x), f in [-0.5, 0.5]; 2^f from a degree-4 minimax-style
// polynomial fitted here for relative error (max 2.7e-6 on [-0.5, 0.5]); 2^n
// added to the exponent field.  Inputs below -126 are clamped (result
// ~1e-38, far below what a bf16 probability can carry next to the row max).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c);
__device__ __forceinline__ float2 fadd2(float2 a, float2 b);
__device__ __forceinline__ float2 fsub2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "sub.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  x.x = fmaxf(x.x, -126.0f);
  x.y = fmaxf(x.y, -126.0f);
  const float2 magic = make_float2(12582912.0f, 12582912.0f);  // 1.5 * 2^23
  const float2 t = fadd2(x, magic);                            // rint(x) in the low mantissa bits
  const float2 f = fsub2(x, fsub2(t, magic));
  float2 q = ffma2(make_float2(0.009571120f, 0.009571120f), f, make_float2(0.055920936f, 0.055920936f));
  q = ffma2(q, f, make_float2(0.24024746f, 0.24024746f));
  q = ffma2(q, f, make_float2(0.69312137f, 0.69312137f));
  q = ffma2(q, f, make_float2(0.99999923f, 0.99999923f));
  return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}

// Three-input max and two-lane packed f32 arithmetic (sm_100): fewer issued
// instructions per element in the softmax.
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}


// exact-erf GELU, 0.5 v (1 + erf(v / sqrt 2)), for two lanes with one MUFU
// ex2 each (the fused fc1 epilogues).  With x = |v| / sqrt 2 clamped to 4,
// erfc(x) = 2^(g(y) - x^2 log2 e), y = x / 2 - 1, where g approximates
// log2(exp(x^2) erfc(x)) on [0, 4]: a degree-7 least-squares polynomial
// fitted here (Chebyshev basis, converted to powers of y).  Then
// gelu = h + |h| - |h| erfc(x), h = v / 2.  Max error against the exact
// GELU: 4.9e-7 absolute in f32 (A&S 7.1.26, the reference's erf: 2.1e-7;
// relative, where |gelu| > 1e-3, this fit is the tighter of the two).
__device__ __forceinline__ float2 gelu_erf_ex2(float2 v) {
  const float2 av = make_float2(fminf(fabsf(v.x), 5.656854f), fminf(fabsf(v.y), 5.656854f));
  const float2 y = ffma2(av, make_float2(0.35355339f, 0.35355339f), make_float2(-1.0f, -1.0f));  // |v|/(2 sqrt 2) - 1
  float2 g = ffma2(make_float2(-0.00288643665f, -0.00288643665f), y, make_float2(0.0129643874f, 0.0129643874f));
  g = ffma2(g, y, make_float2(-0.0346219689f, -0.0346219689f));
  g = ffma2(g, y, make_float2(0.082343936f, 0.082343936f));
  g = ffma2(g, y, make_float2(-0.18980518f, -0.18980518f));
  g = ffma2(g, y, make_float2(0.440013081f, 0.440013081f));
  g = ffma2(g, y, make_float2(-1.20657349f, -1.20657349f));
  g = ffma2(g, y, make_float2(-1.96919358f, -1.96919358f));
  const float2 t = ffma2(fmul2(av, av), make_float2(-0.72134752f, -0.72134752f), g);  // - x^2 log2 e
  const float2 e = make_float2(ex2_approx(t.x), ex2_approx(t.y));                    // erfc(x)
  const float2 h = fmul2(v, make_float2(0.5f, 0.5f));
  const float2 nah = make_float2(fminf(h.x, -h.x), fminf(h.y, -h.y));  // -|h|
  return ffma2(nah, e, fsub2(h, nah));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace vk
