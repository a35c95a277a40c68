// vk_gemm_tc.cu -- bf16 projection GEMM on the 5th-generation tensor cores.
//
// Replaces the reference's shape-specialised AVX-512 projections
// (src/specialized.rs:770-1300: linear_f32_da3_base, linear_bias_scale_f32_da3_base,
// qkv_f32_da3_base) and the separate bias / GELU / LayerScale / residual passes
// (src/scalar.rs:65-155, src/dispatch.rs:56-77) with one persistent kernel:
//
//   warp 0      TMA producer: A [128 x 64] and W [BN x 64] bf16 tiles, 128B swizzle,
//               into a STAGES-deep shared-memory ring (mbarrier full/empty pairs)
//   warp 1      allocates TMEM, one elected lane issues tcgen05.mma (M=128, N=BN,
//               K=16) into one of two f32 accumulators in TMEM (2 x BN columns)
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time (one row per thread),
//               fused bias / GELU / LayerScale+residual / head-major QKV+RoPE, store
//
// The accumulator double buffer lets the epilogue of tile i overlap the MMAs
// of tile i+1.  Tiles are visited m-major across the persistent grid so the
// CTAs resident at one time share A row-blocks in L2.
#include <cudaTypedefs.h>

#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "vk_common.cuh"
#include "vk_internal.h"
#include "vk_epilogue.cuh"

namespace vk {

namespace {
constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = one 128-byte swizzle row
constexpr int GEMM_THREADS = 192;

template <int BN>
struct GemmCfg {
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  // epilogue staging: 4 warps x 2 buffers x (32 rows x 128 B)
  static constexpr int STAGE_OUT_BYTES = 4 * 2 * 4096;
  static constexpr size_t SMEM = 1024 + static_cast<size_t>(STAGES) * STAGE_BYTES + STAGE_OUT_BYTES + 256;
};

// Output element size and the TMA swizzle of the 32 x 32 staging tile.
template <int MODE>
struct OutTraits {
  static constexpr bool F32 = (MODE == EPI_F32 || MODE == EPI_RESID || MODE == EPI_QKV_F32);
  static constexpr int ROW_BYTES = F32 ? 128 : 64;
};

// Writes this thread's 32 values as row `lane` of a 32-row staging tile in
// the TMA 128-byte (f32) or 64-byte (bf16) swizzle, so that the 16-byte
// chunks of one store instruction spread over all banks.
template <int MODE>
__device__ __forceinline__ void stage_row(uint8_t* buf, int lane, const float (&v)[32]) {
  if constexpr (OutTraits<MODE>::F32) {
    uint8_t* row = buf + lane * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<float4*>(row + ((j ^ (lane & 7)) << 4)) =
          make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  } else {
    uint8_t* row = buf + lane * 64;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<uint4*>(row + ((j ^ ((lane >> 1) & 3)) << 4)) =
          make_uint4(pack_bf16x2(v[8 * j], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                     pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
  }
}
}  // namespace

// Epilogue of one accumulator tile for one epilogue warp: rows
// [row0, row0 + 32) of the output, columns [n0, n0 + BN_).  Reads TMEM 32
// columns at a time, applies the fused epilogue and writes through a
// swizzled staging buffer with TMA stores.  `release` runs once the
// accumulator has been read completely (it hands it back to the MMA warp).
template <int MODE, int BN_, class Release>
__device__ __forceinline__ void epilogue_tile(const GemmEpi& epi, const CUtensorMap* tmO0, const CUtensorMap* tmO1,
                                              const CUtensorMap* tmO2, int M, int N, int row0, int n0,
                                              uint32_t tbase, uint8_t* stage, int& sb, int lane, Release release) {
  const int row = row0 + lane;
  // A 32-row chunk of the head-major QKV output that crosses an image
  // boundary (or the end of M) is written row by row instead of by TMA.
  bool direct = false;
  int img = 0, t0 = 0;
  if constexpr (MODE == EPI_QKV_BF16 || MODE == EPI_QKV_F32) {
    img = row0 / epi.tokens;
    t0 = row0 - img * epi.tokens;
    direct = (t0 + 32 > epi.tokens) || (row0 + 32 > M);
  }
#pragma unroll 1
  for (int c = 0; c < BN_ / 32; ++c) {
    uint32_t r[32];
    tmem_ld32(tbase + static_cast<uint32_t>(c * 32), r);
    tmem_wait_ld();
    if (c == BN_ / 32 - 1) release();
    if (row0 >= M) continue;
    const int col0 = n0 + c * 32;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    epi_math<MODE, true>(epi, row, col0, v);
    if (direct) {
      if (row < M) epi_direct<MODE>(epi, row, col0, N, v);
      continue;
    }
    uint8_t* buf = stage + sb * 4096;
    if (lane == 0) bulk_wait_read<1>();  // the store that last read `buf` is done with it
    __syncwarp();
    stage_row<MODE>(buf, lane, v);
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
      if constexpr (MODE == EPI_RESID) {
        tma_reduce_add_2d(tmO0, buf, col0, row0);
      } else if constexpr (MODE == EPI_QKV_BF16 || MODE == EPI_QKV_F32) {
        const QkvPos q = qkv_pos(epi, row0, col0);
        const CUtensorMap* map = q.g == 0 ? tmO0 : (q.g == 1 ? tmO1 : tmO2);
        tma_store_3d(map, buf, q.axis * 32, t0, img * epi.heads + q.head);
      } else {
        tma_store_2d(tmO0, buf, col0, row0);
      }
      bulk_commit();
    }
    sb ^= 1;
  }
}

// ------------------------------------------------------------------ kernel
template <int BN, int MODE>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    k_gemm_bf16(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmO0, const __grid_constant__ CUtensorMap tmO1,
                const __grid_constant__ CUtensorMap tmO2, const GemmEpi epi, int M, int N, int K, int* err) {
  using C = GemmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint8_t* sOut = smem + C::STAGES * C::STAGE_BYTES;  // 1024-aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + C::STAGE_OUT_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tiles = (M + BM - 1) / BM;
  const int n_tiles = N / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int kb_n = K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile / n_tiles) * BM;
        const int n0 = (tile % n_tiles) * BN;
        for (int kb = 0; kb < kb_n; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, err, VK_DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          tma_load_2d(sA + stage * C::A_BYTES, &tmA, &full[stage], kb * BK, m0);
          tma_load_2d(sB + stage * C::B_BYTES, &tmB, &full[stage], kb * BK, n0);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++it) {
        const int acc = it & 1;
        const uint32_t aphase = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], aphase ^ 1u, err, VK_DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < kb_n; ++kb) {
          if (!mbar_wait(&full[stage], phase, err, VK_DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = smem_desc_k_sw128(smem_u32(sA + stage * C::A_BYTES));
          const uint64_t bdesc = smem_desc_k_sw128(smem_u32(sB + stage * C::B_BYTES));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(d_tmem, adesc + static_cast<uint64_t>(k * 2), bdesc + static_cast<uint64_t>(k * 2),
                     idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit(&tfull[acc]);
      }
    }
  } else {
    const int quad = warp & 3;  // TMEM lanes [32*quad, 32*quad + 32) are this warp's
    uint8_t* stage = sOut + (warp - 2) * 2 * 4096;
    int sb = 0;
    int it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t aphase = (it >> 1) & 1;
      if (!mbar_wait(&tfull[acc], aphase, err, VK_DEV_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const int m0 = (tile / n_tiles) * BM;
      const int n0 = (tile % n_tiles) * BN;
      const int row0 = m0 + quad * 32;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
      epilogue_tile<MODE, BN>(epi, &tmO0, &tmO1, &tmO2, M, N, row0, n0, tbase, stage, sb, lane, [&] {
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
      });
    }
    if (lane == 0) bulk_wait<0>();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ CTA-pair kernel
// Same pipeline on a cluster of two CTAs (one per SM): the pair computes a
// 256 x 256 tile with tcgen05.mma.cta_group::2 (M = 256 split across the two
// SMs' TMEM, N = 256 with each SM staging half of the W tile).  Per SM this
// halves the W bytes staged per FLOP, the bound of the single-CTA kernel.
//   both CTAs   warp 0 loads its A rows [m0 + 128 r, +128) and W rows
//               [n0 + 128 r, +128); both loads complete on the leader's
//               barrier; warps 2..5 run the epilogue on their own TMEM rows
//   leader      warp 1 issues the MMAs and commits to both CTAs' barriers
namespace {
constexpr int P_STAGES = 6;
constexpr int P_A_BYTES = 128 * BK * 2;
constexpr int P_B_BYTES = 128 * BK * 2;
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;
constexpr int P_STAGE_OUT_BYTES = 4 * 2 * 4096;
constexpr size_t P_SMEM = 1024 + static_cast<size_t>(P_STAGES) * P_STAGE_BYTES + P_STAGE_OUT_BYTES + 256;
}  // namespace

template <int MODE>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    k_gemm_bf16_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmO0, const __grid_constant__ CUtensorMap tmO1,
                     const __grid_constant__ CUtensorMap tmO2, const GemmEpi epi, int M, int N, int K, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + P_STAGES * P_A_BYTES;
  uint8_t* sOut = smem + P_STAGES * P_STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + P_STAGE_OUT_BYTES);
  uint64_t* empty = full + P_STAGES;
  uint64_t* tfull = empty + P_STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int m_tiles = (M + 255) / 256;
  const int n_tiles = N / 256;
  const int num_tiles = m_tiles * n_tiles;
  const int kb_n = K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);  // one arrival per epilogue warp of both CTAs
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_cg2(tmem_slot, 512);
    tmem_relinquish_cg2();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
        const int m0 = (tile / n_tiles) * 256;
        const int n0 = (tile % n_tiles) * 256;
        for (int kb = 0; kb < kb_n; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, err, VK_DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * P_STAGE_BYTES);
          const uint32_t bar = mapa_shared(&full[stage], 0);
          tma_load_2d_cg2(sA + stage * P_A_BYTES, &tmA, bar, kb * BK, m0 + 128 * static_cast<int>(rank));
          tma_load_2d_cg2(sB + stage * P_B_BYTES, &tmB, bar, kb * BK, n0 + 128 * static_cast<int>(rank));
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_bf16(256, 256);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs, ++it) {
        const int acc = it & 1;
        const uint32_t aphase = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], aphase ^ 1u, err, VK_DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * 256);
        for (int kb = 0; kb < kb_n; ++kb) {
          if (!mbar_wait(&full[stage], phase, err, VK_DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = smem_desc_k_sw128(smem_u32(sA + stage * P_A_BYTES));
          const uint64_t bdesc = smem_desc_k_sw128(smem_u32(sB + stage * P_B_BYTES));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16_cg2(d_tmem, adesc + static_cast<uint64_t>(k * 2), bdesc + static_cast<uint64_t>(k * 2), idesc,
                         (kb | k) != 0 ? 1u : 0u);
          umma_commit_cg2_mc(&empty[stage], 0x3);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit_cg2_mc(&tfull[acc], 0x3);
      }
    }
  } else {
    const int quad = warp & 3;
    uint8_t* stage = sOut + (warp - 2) * 2 * 4096;
    int sb = 0;
    int it = 0;
    for (int tile = pair; tile < num_tiles; tile += npairs, ++it) {
      const int acc = it & 1;
      const uint32_t aphase = (it >> 1) & 1;
      if (!mbar_wait(&tfull[acc], aphase, err, VK_DEV_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const int m0 = (tile / n_tiles) * 256;
      const int n0 = (tile % n_tiles) * 256;
      const int row0 = m0 + 128 * static_cast<int>(rank) + quad * 32;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * 256);
      epilogue_tile<MODE, 256>(epi, &tmO0, &tmO1, &tmO2, M, N, row0, n0, tbase, stage, sb, lane, [&] {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(&tempty[acc], 0));
      });
    }
    if (lane == 0) bulk_wait<0>();
  }
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_cg2(tmem_base, 512);
  }
}

// ------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
                  uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                  uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0, uint32_t box1,
                  CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {box0, box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

struct OutMaps {
  CUtensorMap m[3];
};

template <int BN, int MODE>
static cudaError_t launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const OutMaps& om, const GemmEpi& epi,
                               int M, int N, int K, int* err, cudaStream_t s) {
  using C = GemmCfg<BN>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm_bf16<BN, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(C::SMEM));
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  const int tiles = ((M + BM - 1) / BM) * (N / BN);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  k_gemm_bf16<BN, MODE><<<grid, GEMM_THREADS, C::SMEM, s>>>(ta, tb, om.m[0], om.m[1], om.m[2], epi, M, N, K, err);
  return cudaGetLastError();
}

template <int MODE>
static cudaError_t launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const OutMaps& om, const GemmEpi& epi,
                               int M, int N, int K, int* err, cudaStream_t s) {
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm_bf16_pair<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(P_SMEM));
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  const int tiles = ((M + 255) / 256) * (N / 256);
  cudaLaunchConfig_t cfg = {};
  static int max_pairs = 0;  // clusters of 2 that can be resident at once
  if (max_pairs == 0) {
    cudaLaunchConfig_t q = {};
    q.gridDim = dim3(2 * (num_sms() / 2));
    q.blockDim = dim3(GEMM_THREADS);
    q.dynamicSmemBytes = P_SMEM;
    cudaLaunchAttribute qa[1];
    qa[0].id = cudaLaunchAttributeClusterDimension;
    qa[0].val.clusterDim.x = 2;
    qa[0].val.clusterDim.y = 1;
    qa[0].val.clusterDim.z = 1;
    q.attrs = qa;
    q.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, k_gemm_bf16_pair<MODE>, &q) != cudaSuccess || n <= 0) n = num_sms() / 2;
    max_pairs = n;
  }
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = P_SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_gemm_bf16_pair<MODE>, ta, tb, om.m[0], om.m[1], om.m[2], epi, M, N, K, err);
}

static cudaError_t dispatch_pair(int mode, const CUtensorMap& ta, const CUtensorMap& tb, const OutMaps& om,
                                 const GemmEpi& epi, int M, int N, int K, int* err, cudaStream_t s) {
  switch (mode) {
    case EPI_F32: return launch_pair<EPI_F32>(ta, tb, om, epi, M, N, K, err, s);
    case EPI_BF16: return launch_pair<EPI_BF16>(ta, tb, om, epi, M, N, K, err, s);
    case EPI_BF16_GELU: return launch_pair<EPI_BF16_GELU>(ta, tb, om, epi, M, N, K, err, s);
    case EPI_RESID: return launch_pair<EPI_RESID>(ta, tb, om, epi, M, N, K, err, s);
    case EPI_QKV_BF16: return launch_pair<EPI_QKV_BF16>(ta, tb, om, epi, M, N, K, err, s);
    case EPI_QKV_F32: return launch_pair<EPI_QKV_F32>(ta, tb, om, epi, M, N, K, err, s);
    default: return cudaErrorInvalidValue;
  }
}

template <int BN>
static cudaError_t dispatch_mode(int mode, const CUtensorMap& ta, const CUtensorMap& tb, const OutMaps& om,
                                 const GemmEpi& epi, int M, int N, int K, int* err, cudaStream_t s) {
  switch (mode) {
    case EPI_F32: return launch_gemm<BN, EPI_F32>(ta, tb, om, epi, M, N, K, err, s);
    case EPI_BF16: return launch_gemm<BN, EPI_BF16>(ta, tb, om, epi, M, N, K, err, s);
    case EPI_BF16_GELU: return launch_gemm<BN, EPI_BF16_GELU>(ta, tb, om, epi, M, N, K, err, s);
    case EPI_RESID: return launch_gemm<BN, EPI_RESID>(ta, tb, om, epi, M, N, K, err, s);
    case EPI_QKV_BF16: return launch_gemm<BN, EPI_QKV_BF16>(ta, tb, om, epi, M, N, K, err, s);
    case EPI_QKV_F32: return launch_gemm<BN, EPI_QKV_F32>(ta, tb, om, epi, M, N, K, err, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t gemm_bf16_tc(const __nv_bfloat16* A, const __nv_bfloat16* W, int M, int N, int K, int mode,
                         const GemmEpi& epi, int* err, cudaStream_t s) {
  if (M <= 0 || N <= 0 || K <= 0 || K % BK != 0 || N % 128 != 0) return cudaErrorInvalidValue;
  if (mode == EPI_RESID && epi.scale == nullptr) return cudaErrorInvalidValue;
  // Wide tiles when they still give at least one full wave of CTAs.
  const int m_tiles = (M + BM - 1) / BM;
  const bool wide = (N % 256 == 0) && m_tiles * (N / 256) >= num_sms();
  // CTA pairs (256 x 256 tiles) when they fill every SM at least once.
  static const bool pair_enabled = getenv("VK_GEMM_NO_PAIR") == nullptr;
  const bool pair = pair_enabled && (N % 256 == 0) && ((M + 255) / 256) * (N / 256) >= num_sms() / 2;
  const int bn = pair ? 128 : (wide ? 256 : 128);
  CUtensorMap ta, tb;
  if (!make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, A, K, M, static_cast<uint64_t>(K) * 2, BK, BM,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (!make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, W, K, N, static_cast<uint64_t>(K) * 2, BK, bn,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  OutMaps om;
  memset(&om, 0, sizeof(om));
  bool ok = true;
  const bool f32 = (mode == EPI_F32 || mode == EPI_RESID || mode == EPI_QKV_F32);
  const CUtensorMapDataType odt = f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint64_t esz = f32 ? 4 : 2;
  const CUtensorMapSwizzle oswz = f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  if (mode == EPI_QKV_BF16 || mode == EPI_QKV_F32) {
    if (epi.tokens <= 0 || M % epi.tokens != 0 || N != 3 * epi.heads * 64) return cudaErrorInvalidValue;
    const uint64_t images = M / epi.tokens;
    void* bases[3] = {epi.q, epi.k, epi.v};
    for (int g = 0; g < 3 && ok; ++g)
      ok = make_tmap_3d(&om.m[g], odt, bases[g], 64, epi.tokens, images * epi.heads, 64 * esz,
                        static_cast<uint64_t>(epi.tokens) * 64 * esz, 32, 32, oswz);
  } else if (mode == EPI_RESID) {
    ok = make_tmap_2d(&om.m[0], odt, epi.resid, N, M, static_cast<uint64_t>(epi.ldo) * esz, 32, 32, oswz);
  } else {
    ok = make_tmap_2d(&om.m[0], odt, epi.out, N, M, static_cast<uint64_t>(epi.ldo) * esz, 32, 32, oswz);
  }
  if (!ok) return cudaErrorInvalidValue;
  if (pair) return dispatch_pair(mode, ta, tb, om, epi, M, N, K, err, s);
  return wide ? dispatch_mode<256>(mode, ta, tb, om, epi, M, N, K, err, s)
              : dispatch_mode<128>(mode, ta, tb, om, epi, M, N, K, err, s);
}

}  // namespace vk
