// vk_gemm_tc.cu -- bf16 projection GEMM on the 5th-generation tensor cores.
//
// Replaces the reference's shape-specialised AVX-512 projections
// (src/specialized.rs:770-1300: linear_f32_da3_base, linear_bias_scale_f32_da3_base,
// qkv_f32_da3_base) and the separate bias / GELU / LayerScale / residual passes
// (src/scalar.rs:65-155, src/dispatch.rs:56-77) with one persistent kernel,
// C[M, N] = A[M, K] . W[N, K]^T (both K-major bf16, f32 accumulation):
//
//   warp 0       TMA producer: A [128 x 64] and W [128 x 64] bf16 slabs, 128-byte
//                swizzle, into a STAGES-deep shared-memory ring (full/empty mbarriers)
//   warp 1       allocates TMEM; one elected lane issues tcgen05.mma into one of two
//                f32 accumulators in TMEM (double buffer: the epilogue of tile i
//                overlaps the MMAs of tile i+1)
//   warps 2..9   epilogue, two warps per TMEM lane quadrant (each takes half of the
//                tile's columns): tcgen05.ld 32 columns at a time, software-pipelined,
//                bias / scale from shared memory, fused GELU / LayerScale / RoPE,
//                swizzled staging + TMA store (TMA reduce-add for the residual)
//
// PAIR = false: one CTA per 128 x 128 tile (MMA M=128, N=128).
// PAIR = true:  a cluster of two CTAs (one per SM) per 256 x 256 tile with
//               tcgen05.mma.cta_group::2 (M=256 split over the two SMs' TMEM, each
//               SM staging its 128 rows of A and half of the W tile); used when the
//               problem fills every SM pair at least once.
// Tiles are visited m-major over the persistent grid so the CTAs resident at one
// time share A row-blocks in L2.
#include <stdlib.h>
#include <string.h>

#include "vk_common.cuh"
#include "vk_epilogue.cuh"
#include "vk_internal.h"

namespace vk {

namespace {
constexpr int BK = 64;  // 64 bf16 = one 128-byte swizzle row
constexpr int GEMM_THREADS = 320;
constexpr int SLAB_BYTES = 128 * BK * 2;  // one 128-row operand slab per stage

// WIDE (CTA pairs, residual epilogue only): 256 x 384 tiles, each CTA
// staging 192 rows of W (two 96-row boxes) and issuing two N = 192 MMAs per
// K step into one
// 384-column accumulator (no second buffer: TMEM holds 512 columns).  For
// the N = 768 GEMMs when their 256 x 256 tiles would need a second, mostly
// idle round while 256 x 384 ones fit in one (a few images per GPU).
template <int MODE, bool PAIR, bool WIDE = false>
struct Cfg {
  static constexpr bool F32OUT = (MODE == EPI_F32 || MODE == EPI_RESID || MODE == EPI_QKV_F32 || MODE == EPI_TOKENS);
  static constexpr int TILE_M = PAIR ? 256 : 128;  // rows of C per tile
  static constexpr int TILE_N = PAIR ? (WIDE ? 384 : 256) : 128;  // columns of C per tile
  static constexpr int MMA_N = WIDE ? 192 : TILE_N;                // columns per MMA
  static constexpr int B_ROWS = PAIR ? TILE_N / 2 : TILE_N;        // rows of W this CTA stages
  static constexpr int B_SLAB = B_ROWS * BK * 2;
  static constexpr int ACCS = WIDE ? 1 : 2;                        // TMEM accumulators
  static constexpr int TMEM_COLS = WIDE ? 512 : 2 * TILE_N;
  static constexpr int WARP_COLS = TILE_N / 2;     // columns one epilogue warp handles
  static constexpr int STAGE_BYTES = SLAB_BYTES + B_SLAB;
  static constexpr int OUT_BUF = F32OUT ? 4096 : 2048;  // 32 x 32 staging tile
  // f32 outputs: two 32 x 32 tiles per warp, double buffered chunk by chunk;
  // bf16 outputs: the warp's whole 32 x WARP_COLS slice, one fence per tile
  static constexpr int WARP_BUFS = F32OUT ? 2 : (WARP_COLS / 32 > 2 ? WARP_COLS / 32 : 2);
  static constexpr int OUT_BYTES = 8 * WARP_BUFS * OUT_BUF;
  // as many K stages as shared memory holds (at most 6)
  static constexpr int STAGES_FIT = static_cast<int>((232448 - 1024 - 256 - OUT_BYTES) / STAGE_BYTES);
  static constexpr int STAGES = STAGES_FIT < 6 ? STAGES_FIT : 6;
  static constexpr size_t SMEM = 1024 + static_cast<size_t>(STAGES) * STAGE_BYTES + OUT_BYTES + 256;
  static_assert(SMEM <= 232448, "shared memory budget");
};


// Writes this thread's 32 values as row `lane` of a 32-row staging tile in
// the TMA 128-byte (f32) or 64-byte (bf16) swizzle, so that the 16-byte
// chunks of one store instruction spread over all banks.
// f16 packs IEEE half instead of bf16 (the V third of the QKV output).
template <bool F32>
__device__ __forceinline__ void stage_row(uint8_t* buf, int lane, const float (&v)[32], bool f16 = false) {
  if constexpr (F32) {
    uint8_t* row = buf + lane * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<float4*>(row + ((j ^ (lane & 7)) << 4)) =
          make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  } else {
    uint8_t* row = buf + lane * 64;
    if (f16) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(row + ((j ^ ((lane >> 1) & 3)) << 4)) =
            make_uint4(pack_f16x2(v[8 * j], v[8 * j + 1]), pack_f16x2(v[8 * j + 2], v[8 * j + 3]),
                       pack_f16x2(v[8 * j + 4], v[8 * j + 5]), pack_f16x2(v[8 * j + 6], v[8 * j + 7]));
      return;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<uint4*>(row + ((j ^ ((lane >> 1) & 3)) << 4)) =
          make_uint4(pack_bf16x2(v[8 * j], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                     pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
  }
}
}  // namespace

// TMA store (or reduce-add) of one staged 32 x 32 chunk at rows
// [row0, row0 + 32), columns [col0, col0 + 32).
template <int MODE>
__device__ __forceinline__ void store_chunk(const GemmEpi& epi, const CUtensorMap* tmO0, const CUtensorMap* tmO1,
                                            const CUtensorMap* tmO2, uint8_t* buf, int row0, int col0, int img,
                                            int t0) {
  if constexpr (MODE == EPI_RESID) {
    tma_reduce_add_2d(tmO0, buf, col0, row0);
  } else if constexpr (MODE == EPI_TOKENS) {
    tma_store_3d(tmO0, buf, col0, t0, img);  // the map starts at token row 1 of image 0
  } else if constexpr (MODE == EPI_QKV_BF16 || MODE == EPI_QKV_F32) {
    const QkvPos q = qkv_pos(epi, row0, col0);
    const CUtensorMap* map = q.g == 0 ? tmO0 : (q.g == 1 ? tmO1 : tmO2);
    tma_store_3d(map, buf, q.axis * 32, t0, img * epi.heads + q.head);
  } else {
    tma_store_2d(tmO0, buf, col0, row0);
  }
}

// Epilogue of one warp's share of an accumulator tile: rows [row0, row0+32),
// columns [c0, c0 + NCOL).  `release` runs once the TMEM columns have all
// been read (it hands the accumulator back to the MMA warp).
template <int MODE, int NCOL, class Release>
__device__ __forceinline__ void epilogue_part(const GemmEpi& epi, const CUtensorMap* tmO0, const CUtensorMap* tmO1,
                                              const CUtensorMap* tmO2, int M, int N, int row0, int c0,
                                              uint32_t tbase, const float* sbias, const float* sscale,
                                              uint8_t* stage, int& sb, int lane, Release release) {
  constexpr bool F32 = (MODE == EPI_F32 || MODE == EPI_RESID || MODE == EPI_QKV_F32 || MODE == EPI_TOKENS);
  constexpr int OUT_BUF = F32 ? 4096 : 2048;
  const int row = row0 + lane;
  // A 32-row chunk of the head-major QKV output that crosses an image
  // boundary (or the end of M) is written row by row instead of by TMA.
  bool direct = false;
  int img = 0, t0 = 0;
  if constexpr (MODE == EPI_QKV_BF16 || MODE == EPI_QKV_F32 || MODE == EPI_TOKENS) {
    img = row0 / epi.tokens;
    t0 = row0 - img * epi.tokens;
    direct = (t0 + 32 > epi.tokens) || (row0 + 32 > M);
  }
  // bf16 outputs stage every chunk of the slice (buffer c) and publish them
  // with one proxy fence; f32 outputs alternate two buffers chunk by chunk.
  constexpr bool GROUPED = !F32;
  bool staged = false;
  if constexpr (GROUPED) {
    if (lane == 0) bulk_wait_read<0>();  // the previous tile's stores are done with the slice
    __syncwarp();
  }
  if constexpr (MODE == EPI_QKV_BF16) {
    if (epi.qkn != nullptr) {
      // Q/K LayerNorm before RoPE (src/specialized.rs:278-454): the two
      // 32-column chunks of a head (both RoPE axis halves) belong to this
      // thread, so the 64-wide row is normalised in registers.
#pragma unroll 1
      for (int cp = 0; cp < NCOL / 64; ++cp) {
        float v[64];
        tmem_ld32(tbase + static_cast<uint32_t>(cp * 64), *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        tmem_ld32(tbase + static_cast<uint32_t>(cp * 64 + 32), *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        tmem_wait_ld();
        if (cp + 1 == NCOL / 64) release();
        if (row0 >= M) continue;
        const int col0 = c0 + cp * 64;
        if (sbias != nullptr)
#pragma unroll
          for (int d = 0; d < 64; ++d) v[d] += sbias[cp * 64 + d];
        const QkvPos q = qkv_pos(epi, row, col0);
        if (q.g < 2) {
          // layernorm_row's arithmetic (src/scalar.rs:99-113): ascending folds
          // from -0.0, every product and sum separately rounded
          const float* gm = epi.qkn + q.g * 128;  // gamma, then beta
          float sum = -0.0f;
#pragma unroll
          for (int d = 0; d < 64; ++d) sum = __fadd_rn(sum, v[d]);
          const float mean = __fdiv_rn(sum, 64.0f);
          float sq = -0.0f;
#pragma unroll
          for (int d = 0; d < 64; ++d) {
            const float dv = __fsub_rn(v[d], mean);
            sq = __fadd_rn(sq, __fmul_rn(dv, dv));
          }
          const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sq, 64.0f), epi.qkn_eps)));
#pragma unroll
          for (int d = 0; d < 64; ++d)
            v[d] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[d], mean), inv), __ldg(gm + d)), __ldg(gm + 64 + d));
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float(&half)[32] = *reinterpret_cast<float(*)[32]>(&v[32 * h]);
          epi_math<MODE, true>(epi, row, col0 + 32 * h, half, nullptr, nullptr);  // RoPE on q / k
          if (direct) {
            if (row < M) epi_direct<MODE>(epi, row, col0 + 32 * h, N, half);
          } else {
            stage_row<false>(stage + (2 * cp + h) * OUT_BUF, lane, half, qkv_is_v(epi, col0));
            staged = true;
          }
        }
      }
      if (staged) {
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
#pragma unroll
          for (int c = 0; c < NCOL / 32; ++c)
            store_chunk<MODE>(epi, tmO0, tmO1, tmO2, stage + c * OUT_BUF, row0, c0 + c * 32, img, t0);
          bulk_commit();
        }
      }
      return;
    }
  }
  uint32_t r[2][32];
  tmem_ld32(tbase, r[0]);
#pragma unroll
  for (int c = 0; c < NCOL / 32; ++c) {
    tmem_wait_ld();
    if (c + 1 < NCOL / 32)
      tmem_ld32(tbase + static_cast<uint32_t>((c + 1) * 32), r[(c + 1) & 1]);  // overlaps this chunk's math
    else
      release();
    if (row0 >= M) continue;
    const int col0 = c0 + c * 32;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[c & 1][j]);
    epi_math<MODE, true>(epi, row, col0, v, sbias ? sbias + c * 32 : nullptr, sscale ? sscale + c * 32 : nullptr);
    if (direct) {
      if (row < M) epi_direct<MODE>(epi, row, col0, N, v);
      continue;
    }
    if constexpr (GROUPED) {
      stage_row<F32>(stage + c * OUT_BUF, lane, v, MODE == EPI_QKV_BF16 && qkv_is_v(epi, col0));
      staged = true;
      continue;
    }
    uint8_t* buf = stage + sb * OUT_BUF;
    if (lane == 0) bulk_wait_read<1>();  // the store that last read `buf` is done with it
    __syncwarp();
    stage_row<F32>(buf, lane, v);
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
      store_chunk<MODE>(epi, tmO0, tmO1, tmO2, buf, row0, col0, img, t0);
      bulk_commit();
    }
    sb ^= 1;
  }
  if constexpr (GROUPED) {
    if (staged) {
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
#pragma unroll
        for (int c = 0; c < NCOL / 32; ++c) store_chunk<MODE>(epi, tmO0, tmO1, tmO2, stage + c * OUT_BUF, row0, c0 + c * 32, img, t0);
        bulk_commit();
      }
    }
  }
}

template <int MODE, bool PAIR, bool WIDE>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    k_gemm_bf16(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmO0, const __grid_constant__ CUtensorMap tmO1,
                const __grid_constant__ CUtensorMap tmO2, const GemmEpi epi, int M, int N, int K, int* err) {
  using C = Cfg<MODE, PAIR, WIDE>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * SLAB_BYTES;
  uint8_t* sOut = smem + C::STAGES * C::STAGE_BYTES;  // 1024-aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + C::OUT_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int unit = PAIR ? (blockIdx.x >> 1) : blockIdx.x;  // CTA pair or CTA
  const int units = PAIR ? (gridDim.x >> 1) : gridDim.x;
  const int m_tiles = (M + C::TILE_M - 1) / C::TILE_M;
  const int n_tiles = N / C::TILE_N;
  const int num_tiles = m_tiles * n_tiles;
  const int kb_n = K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], PAIR ? 16 : 8);  // one arrival per epilogue warp (of both CTAs)
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_cg2(tmem_slot, C::TMEM_COLS);
      tmem_relinquish_cg2();
    } else {
      tmem_alloc(tmem_slot, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  tc_fence_before();
  if constexpr (PAIR) cluster_sync(); else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  grid_dependency_wait();  // the previous kernel's outputs (our A, the residual) are visible from here

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = unit; tile < num_tiles && ok; tile += units) {
        const int m0 = (tile / n_tiles) * C::TILE_M + 128 * static_cast<int>(rank);
        // A CTA pair's MMA takes half of its N columns from each CTA's W
        // rows: 128 + 128 for 256-wide tiles; for WIDE tiles each of the two
        // N = 192 MMAs takes 96 + 96, so a CTA stages rows [96 rank, +96) and
        // [192 + 96 rank, +96) of the tile's 384.
        const int n0 = (tile % n_tiles) * C::TILE_N + (WIDE ? 96 : C::B_ROWS) * static_cast<int>(rank);
        for (int kb = 0; kb < kb_n; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, err, VK_DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          if constexpr (PAIR) {
            // both CTAs' slabs complete on the leader's barrier
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
            const uint32_t bar = mapa_shared(&full[stage], 0);
            tma_load_2d_cg2(sA + stage * SLAB_BYTES, &tmA, bar, kb * BK, m0);
            tma_load_2d_cg2(sB + stage * C::B_SLAB, &tmB, bar, kb * BK, n0);
            if constexpr (WIDE) tma_load_2d_cg2(sB + stage * C::B_SLAB + 96 * 128, &tmB, bar, kb * BK, n0 + 192);
          } else {
            mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
            tma_load_2d(sA + stage * SLAB_BYTES, &tmA, &full[stage], kb * BK, m0);
            tma_load_2d(sB + stage * C::B_SLAB, &tmB, &full[stage], kb * BK, n0);
          }
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_bf16(C::TILE_M, C::MMA_N);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int tile = unit; tile < num_tiles && ok; tile += units, ++it) {
        const int acc = it % C::ACCS;
        const uint32_t aphase = (it / C::ACCS) & 1;
        if (!mbar_wait(&tempty[acc], aphase ^ 1u, err, VK_DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * C::TILE_N);
        for (int kb = 0; kb < kb_n; ++kb) {
          if (!mbar_wait(&full[stage], phase, err, VK_DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = smem_desc_k_sw128(smem_u32(sA + stage * SLAB_BYTES));
          const uint64_t bdesc = smem_desc_k_sw128(smem_u32(sB + stage * C::B_SLAB));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint32_t accum = (kb | k) != 0 ? 1u : 0u;
            if constexpr (PAIR) {
              umma_f16_cg2(d_tmem, adesc + static_cast<uint64_t>(k * 2), bdesc + static_cast<uint64_t>(k * 2), idesc,
                           accum);
              if constexpr (WIDE)  // columns [192, 384): W rows [96, 192) of each CTA's slab (12 KB on)
                umma_f16_cg2(d_tmem + 192, adesc + static_cast<uint64_t>(k * 2),
                             bdesc + static_cast<uint64_t>((96 * 128) >> 4) + static_cast<uint64_t>(k * 2), idesc,
                             accum);
            } else {
              umma_f16(d_tmem, adesc + static_cast<uint64_t>(k * 2), bdesc + static_cast<uint64_t>(k * 2), idesc,
                       accum);
            }
          }
          if constexpr (PAIR) umma_commit_cg2_mc(&empty[stage], 0x3); else umma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) {
          if constexpr (PAIR) umma_commit_cg2_mc(&tfull[acc], 0x3); else umma_commit(&tfull[acc]);
        }
      }
    }
  } else {
    const int ew = warp - 2;        // 0..7
    const int quad = warp & 3;      // TMEM lanes [32*quad, 32*quad + 32) are this warp's
    const int chalf = ew >> 2;      // which half of the tile's columns
    uint8_t* stage = sOut + ew * C::WARP_BUFS * C::OUT_BUF;
    int sb = 0;
    int it = 0;
    bool ok = true;
    for (int tile = unit; tile < num_tiles && ok; tile += units, ++it) {
      const int acc = it % C::ACCS;
      const uint32_t aphase = (it / C::ACCS) & 1;
      if (tile + units >= num_tiles && num_tiles <= VK_EARLY_LAUNCH_ROUNDS * units) grid_launch_dependents();
      const int m0 = (tile / n_tiles) * C::TILE_M;
      const int n0 = (tile % n_tiles) * C::TILE_N;
      // warp-uniform outcome: the TMEM reads after the wait are warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], aphase, err, VK_DEV_TIMEOUT_EPILOGUE))) {
        ok = false;  // every epilogue warp gives up at the same tile
        break;
      }
      tc_fence_after();
      const int row0 = m0 + 128 * static_cast<int>(rank) + quad * 32;
      const int c_off = chalf * C::WARP_COLS;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * C::TILE_N + c_off);
      epilogue_part<MODE, C::WARP_COLS>(epi, &tmO0, &tmO1, &tmO2, M, N, row0, n0 + c_off, tbase,
                                        // bias / scale straight from global memory (L1): no
                                        // per-tile barrier across the epilogue warps
                                        epi.bias ? epi.bias + n0 + c_off : nullptr,
                                        epi.scale ? epi.scale + n0 + c_off : nullptr,
                                        stage, sb, lane, [&] {
                                          tc_fence_before();
                                          __syncwarp();
                                          if (lane == 0) {
                                            if constexpr (PAIR)
                                              mbar_arrive_cluster(mapa_shared(&tempty[acc], 0));
                                            else
                                              mbar_arrive(&tempty[acc]);
                                          }
                                        });
    }
    if (lane == 0) bulk_wait<0>();
  }
  tc_fence_before();
  if constexpr (PAIR) cluster_sync(); else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_cg2(tmem_base, C::TMEM_COLS); else tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side
namespace {
struct OutMaps {
  CUtensorMap m[3];
};

template <int MODE, bool PAIR, bool WIDE = false>
cudaError_t launch(const CUtensorMap& ta, const CUtensorMap& tb, const OutMaps& om, const GemmEpi& epi, int M, int N,
                   int K, int* err, cudaStream_t s) {
  using C = Cfg<MODE, PAIR, WIDE>;
  // CTAs (or CTA pairs) that can be resident at once, per device
  int& max_units = *per_device_slot(reinterpret_cast<const void*>(k_gemm_bf16<MODE, PAIR, WIDE>));
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (PAIR) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 2;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  if (max_units == 0) {
    cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(k_gemm_bf16<MODE, PAIR, WIDE>), static_cast<int>(C::SMEM));
    if (e != cudaSuccess) return e;
    int n = 0;
    if (PAIR) {
      cfg.gridDim = dim3(2 * (num_sms() / 2));
      if (cudaOccupancyMaxActiveClusters(&n, k_gemm_bf16<MODE, PAIR, WIDE>, &cfg) != cudaSuccess || n <= 0) n = num_sms() / 2;
    } else {
      n = num_sms();
    }
    max_units = n;
  }
  const int tiles = ((M + C::TILE_M - 1) / C::TILE_M) * (N / C::TILE_N);
  const int units = tiles < max_units ? tiles : max_units;
  cfg.gridDim = dim3(PAIR ? 2 * units : units);
  return cudaLaunchKernelEx(&cfg, k_gemm_bf16<MODE, PAIR, WIDE>, ta, tb, om.m[0], om.m[1], om.m[2], epi, M, N, K, err);
}

template <bool PAIR>
cudaError_t dispatch(int mode, const CUtensorMap& ta, const CUtensorMap& tb, const OutMaps& om, const GemmEpi& epi,
                     int M, int N, int K, int* err, cudaStream_t s) {
  switch (mode) {
    case EPI_F32: return launch<EPI_F32, PAIR>(ta, tb, om, epi, M, N, K, err, s);
    case EPI_BF16: return launch<EPI_BF16, PAIR>(ta, tb, om, epi, M, N, K, err, s);
    case EPI_BF16_GELU: return launch<EPI_BF16_GELU, PAIR>(ta, tb, om, epi, M, N, K, err, s);
    case EPI_RESID: return launch<EPI_RESID, PAIR>(ta, tb, om, epi, M, N, K, err, s);
    case EPI_QKV_BF16: return launch<EPI_QKV_BF16, PAIR>(ta, tb, om, epi, M, N, K, err, s);
    case EPI_QKV_F32: return launch<EPI_QKV_F32, PAIR>(ta, tb, om, epi, M, N, K, err, s);
    case EPI_TOKENS: return launch<EPI_TOKENS, PAIR>(ta, tb, om, epi, M, N, K, err, s);
    default: return cudaErrorInvalidValue;
  }
}
}  // namespace

cudaError_t gemm_bf16_tc(const __nv_bfloat16* A, const __nv_bfloat16* W, int M, int N, int K, int mode,
                         const GemmEpi& epi, int* err, cudaStream_t s) {
  if (M <= 0 || N <= 0 || K <= 0 || K % BK != 0 || N % 128 != 0) return cudaErrorInvalidValue;
  if (mode == EPI_RESID && epi.scale == nullptr) return cudaErrorInvalidValue;
  // CTA pairs (256 x 256 tiles) when they fill every SM pair at least once.
  static const bool pair_enabled = getenv("VK_GEMM_NO_PAIR") == nullptr;
  const bool pair = pair_enabled && (N % 256 == 0) && ((M + 255) / 256) * (N / 256) >= num_sms() / 2;
  // residual GEMMs whose 256 x 256 tiles need a second, mostly idle round
  // while 256 x 384 tiles fit in one
  const int mt256 = (M + 255) / 256, pairs = num_sms() / 2;
  static const bool wide_enabled = getenv("VK_GEMM_NO_WIDE") == nullptr;
  const bool wide = pair_enabled && wide_enabled && mode == EPI_RESID && N % 384 == 0 && mt256 * (N / 384) <= pairs &&
                    mt256 * (N / 256) > pairs;
  CUtensorMap ta, tb;
  if (!make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, A, K, M, static_cast<uint64_t>(K) * 2, BK, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (!make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, W, K, N, static_cast<uint64_t>(K) * 2, BK, wide ? 96 : 128,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  OutMaps om;
  memset(&om, 0, sizeof(om));
  bool ok = true;
  const bool f32 = (mode == EPI_F32 || mode == EPI_RESID || mode == EPI_QKV_F32 || mode == EPI_TOKENS);
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
  } else if (mode == EPI_TOKENS) {
    // [images][tokens + 1][N] f32 from token row 1: patch p of image b is row 1 + p
    if (epi.tokens <= 0 || M % epi.tokens != 0 || epi.pos == nullptr || epi.ldo != N) return cudaErrorInvalidValue;
    const uint64_t images = M / epi.tokens;
    ok = make_tmap_3d(&om.m[0], odt, static_cast<float*>(epi.out) + N, N, epi.tokens, images,
                      static_cast<uint64_t>(N) * esz, static_cast<uint64_t>(epi.tokens + 1) * N * esz, 32, 32, oswz);
  } else if (mode == EPI_RESID) {
    ok = make_tmap_2d(&om.m[0], odt, epi.resid, N, M, static_cast<uint64_t>(epi.ldo) * esz, 32, 32, oswz);
  } else {
    ok = make_tmap_2d(&om.m[0], odt, epi.out, N, M, static_cast<uint64_t>(epi.ldo) * esz, 32, 32, oswz);
  }
  if (!ok) return cudaErrorInvalidValue;
  if (wide) return launch<EPI_RESID, true, true>(ta, tb, om, epi, M, N, K, err, s);
  return pair ? dispatch<true>(mode, ta, tb, om, epi, M, N, K, err, s)
              : dispatch<false>(mode, ta, tb, om, epi, M, N, K, err, s);
}

}  // namespace vk
