// vk_gemm_q8.cu -- Q8_0 x Q8_0 -> f32 projection GEMM on the int8 tensor cores.
//
// Replaces Kernels::gemm_q8_0 (src/dispatch.rs:91-105; scalar oracle
// src/scalar.rs:25-56, AVX-512 VNNI path src/simd_avx512.rs:262-351):
//
//   c[i, j] = sum over blocks b (ascending) of  (d_a[i,b] * d_b[j,b]) * isum_b[i,j]
//   isum_b[i,j] = sum_{l<32} qa[i, 32b + l] * qb[j, 32b + l]      (int32, exact)
//
// One tcgen05.mma.kind::i8 with K = 32 is exactly one Q8_0 block, so every
// block's int32 dot products land in their own TMEM accumulator (4 rotating
// buffers of 128 columns).  Sixteen epilogue warps drain each buffer with
// tcgen05.ld and fold it into f32 registers in the reference's order:
// acc = acc + (d_a * d_b) * float(isum).  The f32-output operator
// (vk_gemm_q8_0) rounds at every step (no FMA), so its result equals the
// reference scalar oracle bit for bit; the encoder's fused epilogues fold
// with one FMA per step (the int32 block dots are exact either way).
//
//   warp 0       TMA producer: A / W int8 tiles [128 x 128 bytes], 128B swizzle
//   warp 1       TMEM owner; one lane issues one MMA per Q8_0 block
//   warps 2..17  epilogue: four warps per TMEM lane quadrant, 32 columns each
#include "vk_common.cuh"
#include "vk_epilogue.cuh"
#include "vk_internal.h"

namespace vk {

namespace {
constexpr int QBM = 128;
constexpr int QBN = 128;
constexpr int QBK = 128;  // bytes = int8 elements = 4 Q8_0 blocks per stage
constexpr int QSTAGES = 4;
constexpr int QNACC = 4;  // TMEM accumulators of QBN columns
constexpr int Q_THREADS = 576;  // producer, MMA, 16 epilogue warps
constexpr int Q_EPI_THREADS = 512;
constexpr int Q_A_BYTES = QBM * QBK;
constexpr int Q_B_BYTES = QBN * QBK;
constexpr int Q_STAGE_BYTES = Q_A_BYTES + Q_B_BYTES;

__device__ __forceinline__ void epi_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(Q_EPI_THREADS) : "memory");
}

size_t q8_smem_bytes(int K) {
  return 1024 + static_cast<size_t>(QSTAGES) * Q_STAGE_BYTES + static_cast<size_t>(K / 32) * QBN * 4 + 256;
}
}  // namespace

template <int MODE, bool DUMP>
__global__ void __launch_bounds__(Q_THREADS, 1)
    k_gemm_q8(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const __half* __restrict__ Ad, const __half* __restrict__ Wd, const GemmEpi epi, int M, int N, int K,
              int32_t* dots, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nb = K / 32;
  uint8_t* sA = smem;
  uint8_t* sB = smem + QSTAGES * Q_A_BYTES;
  float* sWd = reinterpret_cast<float*>(smem + QSTAGES * Q_STAGE_BYTES);  // [nb][QBN]
  uint64_t* full = reinterpret_cast<uint64_t*>(sWd + static_cast<size_t>(nb) * QBN);
  uint64_t* empty = full + QSTAGES;
  uint64_t* tfull = empty + QSTAGES;
  uint64_t* tempty = tfull + QNACC;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + QNACC);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tiles = (M + QBM - 1) / QBM;
  const int n_tiles = N / QBN;
  const int num_tiles = m_tiles * n_tiles;
  const int kb_n = K / QBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < QSTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < QNACC; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], Q_EPI_THREADS / 32);  // one arrival per epilogue warp
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, QNACC * QBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  grid_dependency_wait();  // the previous kernel's outputs are visible from here

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile / n_tiles) * QBM, n0 = (tile % n_tiles) * QBN;
        for (int kb = 0; kb < kb_n; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, err, VK_DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], Q_STAGE_BYTES);
          tma_load_2d(sA + stage * Q_A_BYTES, &tmA, &full[stage], kb * QBK, m0);
          tma_load_2d(sB + stage * Q_B_BYTES, &tmB, &full[stage], kb * QBK, n0);
          if (++stage == QSTAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_s8(QBM, QBN);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t blk = 0;  // running Q8_0 block counter (selects the accumulator)
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        for (int kb = 0; kb < kb_n && ok; ++kb) {
          if (!mbar_wait(&full[stage], phase, err, VK_DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = smem_desc_k_sw128(smem_u32(sA + stage * Q_A_BYTES));
          const uint64_t bdesc = smem_desc_k_sw128(smem_u32(sB + stage * Q_B_BYTES));
#pragma unroll 1
          for (int j = 0; j < QBK / 32; ++j, ++blk) {
            const uint32_t buf = blk % QNACC;
            const uint32_t bph = (blk / QNACC) & 1u;
            if (!mbar_wait(&tempty[buf], bph ^ 1u, err, VK_DEV_TIMEOUT_MMA)) {
              ok = false;
              break;
            }
            tc_fence_after();
            umma_i8(tmem_base + buf * QBN, adesc + static_cast<uint64_t>(j * 2),
                    bdesc + static_cast<uint64_t>(j * 2), idesc, 0u);
            umma_commit(&tfull[buf]);
          }
          umma_commit(&empty[stage]);
          if (++stage == QSTAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else {
    const int et = threadIdx.x - 64;  // 0..511
    const int quad = warp & 3;
    const int cq = (warp - 2) >> 2;  // columns [32 * cq, 32 * cq + 32) of the tile
    uint32_t blk = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      const int m0 = (tile / n_tiles) * QBM, n0 = (tile % n_tiles) * QBN;
      if (tile + static_cast<int>(gridDim.x) >= num_tiles &&
          num_tiles <= VK_EARLY_LAUNCH_ROUNDS * static_cast<int>(gridDim.x))
        grid_launch_dependents();
      const int row = m0 + quad * 32 + lane;
      // weight scales of this column tile, f32, [nb][QBN]
      epi_bar();
      for (int i = et; i < nb * QBN; i += Q_EPI_THREADS) {
        const int c = i % QBN, b = i / QBN;
        sWd[i] = __half2float(Wd[static_cast<size_t>(n0 + c) * nb + b]);
      }
      epi_bar();
      float acc[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) acc[j] = 0.0f;
      const __half* arow = Ad + static_cast<size_t>(row < M ? row : 0) * nb;
      float da_next = __half2float(__ldg(arow));  // activation scales run one block ahead
#pragma unroll 1
      for (int b = 0; b < nb; ++b, ++blk) {
        const float da = da_next;
        if (b + 1 < nb) da_next = __half2float(__ldg(arow + b + 1));
        const uint32_t buf = blk % QNACC;
        const uint32_t bph = (blk / QNACC) & 1u;
        // warp-uniform outcome: the TMEM read after the wait is warp-collective
        if (!__all_sync(0xffffffffu, mbar_wait(&tfull[buf], bph, err, VK_DEV_TIMEOUT_EPILOGUE))) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t r0[32];
        const uint32_t ta = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + buf * QBN + cq * 32;
        tmem_ld32(ta, r0);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[buf]);
        const float4* wd4 = reinterpret_cast<const float4*>(sWd + b * QBN + cq * 32);
        // acc + (d_a * d_b) * isum, each step rounded (src/scalar.rs:47-52),
        // the multiplies two columns per packed f32x2 operation (IEEE
        // round-to-nearest per lane, as the scalar steps).  |isum| <= 32 * 127^2 < 2^22, so
        // float(isum) is exact and comes from the bits of 1.5 * 2^23 + isum
        // minus 1.5 * 2^23 on the integer and FMA pipes.
        const float2 da2 = make_float2(da, da);
        const float2 magic2 = make_float2(12582912.0f, 12582912.0f);
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4) {
          const float4 db = wd4[j4];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int j = j4 * 4 + 2 * h;
            const float2 s2 = fmul2(da2, h == 0 ? make_float2(db.x, db.y) : make_float2(db.z, db.w));
            const float2 f2 = fsub2(make_float2(__int_as_float(static_cast<int32_t>(r0[j]) + 0x4B400000),
                                                __int_as_float(static_cast<int32_t>(r0[j + 1]) + 0x4B400000)),
                                    magic2);
            if constexpr (MODE == EPI_F32) {
              // the adds stay scalar: a packed multiply feeding a packed add
              // was contracted into a fused multiply-add, which rounds once
              const float2 p2 = fmul2(s2, f2);
              acc[j] = __fadd_rn(acc[j], p2.x);
              acc[j + 1] = __fadd_rn(acc[j + 1], p2.y);
            } else {
              // encoder epilogues: one fused multiply-add per column (the
              // block dots stay exact; the sum is within tolerance)
              const float2 a2 = ffma2(s2, f2, make_float2(acc[j], acc[j + 1]));
              acc[j] = a2.x;
              acc[j + 1] = a2.y;
            }
          }
          if constexpr (DUMP) {
            if (row < M)
              for (int t = 0; t < 4; ++t)
                dots[(static_cast<size_t>(row) * N + n0 + cq * 32 + j4 * 4 + t) * nb + b] =
                    static_cast<int32_t>(r0[j4 * 4 + t]);
          }
        }
      }
      if (!ok) break;
      if (row < M) epilogue_chunk<MODE>(epi, row, n0 + cq * 32, N, acc);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, QNACC * QBN);
  }
}

template <int MODE, bool DUMP>
static cudaError_t launch_q8(const CUtensorMap& ta, const CUtensorMap& tb, const __half* Ad, const __half* Wd,
                             const GemmEpi& epi, int M, int N, int K, int32_t* dots, int* err, cudaStream_t s) {
  const size_t smem = q8_smem_bytes(K);
  cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(k_gemm_q8<MODE, DUMP>), static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int tiles = ((M + QBM - 1) / QBM) * (N / QBN);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(Q_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k_gemm_q8<MODE, DUMP>, ta, tb, Ad, Wd, epi, M, N, K, dots, err);
}

cudaError_t gemm_q8_tc(const int8_t* Aq, const __half* Ad, const int8_t* Wq, const __half* Wd, int M, int N, int K,
                       int mode, const GemmEpi& epi, int32_t* dots_out, int* err, cudaStream_t s) {
  if (M <= 0 || N <= 0 || K <= 0 || K % QBK != 0 || N % QBN != 0) return cudaErrorInvalidValue;
  if (q8_smem_bytes(K) > 232448) return cudaErrorInvalidValue;
  if (mode == EPI_RESID && epi.scale == nullptr) return cudaErrorInvalidValue;
  CUtensorMap ta, tb;
  if (!make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, Aq, K, M, static_cast<uint64_t>(K), QBK, QBM,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (!make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, Wq, K, N, static_cast<uint64_t>(K), QBK, QBN,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (dots_out != nullptr) return launch_q8<EPI_F32, true>(ta, tb, Ad, Wd, epi, M, N, K, dots_out, err, s);
  switch (mode) {
    case EPI_F32: return launch_q8<EPI_F32, false>(ta, tb, Ad, Wd, epi, M, N, K, nullptr, err, s);
    case EPI_RESID: return launch_q8<EPI_RESID, false>(ta, tb, Ad, Wd, epi, M, N, K, nullptr, err, s);
    case EPI_QKV_F32: return launch_q8<EPI_QKV_F32, false>(ta, tb, Ad, Wd, epi, M, N, K, nullptr, err, s);
    case EPI_QKV_BF16: return launch_q8<EPI_QKV_BF16, false>(ta, tb, Ad, Wd, epi, M, N, K, nullptr, err, s);
    case EPI_Q8_GELU: return launch_q8<EPI_Q8_GELU, false>(ta, tb, Ad, Wd, epi, M, N, K, nullptr, err, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace vk
