// vk_attention_tc.cu -- bf16 flash attention on the 5th-generation tensor
// cores for [images * heads, tokens, 64] head-major Q, K, V.
//
// Replaces flash_attention_f32_da3_base / attention::attention on the bf16
// path (src/specialized.rs:730-765, 1400-1562; src/attention.rs:111-201):
// non-causal softmax(Q K^T / 8) V with an online softmax over key blocks.
//
// A persistent CTA per SM works through (image*head, pair of 128-query
// tiles) items.  Every K/V block is loaded once for the item's two tiles,
// and the tiles ping-pong on the tensor core: while the softmax warps of one
// work on S_t(j), the tensor core runs the other tile's O += P V and next S.
// When a head has an odd number of query tiles (865 tokens: 7), the heads'
// last tiles are paired across heads instead of running alone: such an item
// streams two K/V sequences, one per tile.
// The Q tiles and the O accumulators are double-buffered across items, so
// the next item's loads and first MMAs overlap this item's output.
//
//   warp 0      TMA: per item the Q tiles, then K and V blocks of 128 keys
//               (AST-stage ring running across items)
//   warp 1      TMEM owner; one lane issues, per key block j and tile t,
//                 O_t     += P_t(j) V_j      (M=128, N=64, K=128; A = P_t from TMEM;
//                                             P and V in f16: an 11-bit P keeps the
//                                             P V rounding near 2e-4 relative)
//                 S_t(j+1) = Q_t K_j+1^T     (M=128, N=128, K=64; A, B from smem)
//               in that order: the tensor core runs MMAs in issue order, so
//               S_t(j+1) overwrites P_t(j) only after O_t read it
//   warps 2..5  softmax of tile 0, warps 6..9 of tile 1, one query row per
//               thread: p = 2^(s*log2e/8 - m_ref) in one pass over S against
//               the running reference (block 0's max), row sum, P -> TMEM as
//               f16 over S.  O accumulates in TMEM; a block whose row sum
//               would leave the f16 range of P (2^15) is redone against its
//               own max with O rescaled.  Finally O / l is stored token-major bf16 / Q8_0 or
//               head-major f32.
// TMEM per tile (256 columns): S / P [0, 128), O for even / odd items
// [128, 192) / [192, 256).
#include "vk_common.cuh"
#include "vk_internal.h"

namespace vk {

namespace {
constexpr int AQ = 128;        // queries per tile
constexpr int AKV = 128;       // keys per block
constexpr int AST = 4;         // K/V pipeline stages
constexpr int A_THREADS = 320; // producer, MMA, 2 x 4 softmax warps
constexpr int TILE_BYTES = 128 * 128;  // 128 rows x 64 bf16
// Pairs i (of the 16 per 32-column chunk) whose exponentials use the
// FMA-pipe polynomial instead of MUFU ex2 (16 lanes per clock per SM).
// Measured on the current kernel: 0 (all MUFU) is fastest; 4, 6 and 8 of
// 16 on the polynomial cost 1-4 %.
#ifndef VK_ATT_POLY_MASK
#define VK_ATT_POLY_MASK 0x0u
#endif
constexpr uint32_t POLY_MASK = VK_ATT_POLY_MASK;
constexpr uint32_t COL_S = 0, COL_O = 128, TILE_COLS = 256;  // S / P [0, 128), O buffers [128, 192), [192, 256)
constexpr size_t ATT_SMEM = 1024 + TILE_BYTES * (4 + 2 * AST) + 512;
}  // namespace

// SPLIT: P is stored as two f16 halves, P = P_hi + P_lo (P_hi over S columns
// [0, 64), P_lo over [64, 128)), and O += P_hi V + P_lo V, so the P V
// product carries about 22 bits of P instead of 11.
template <int OUT, bool SPLIT>
__global__ void __launch_bounds__(A_THREADS, 1)
    k_attention_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, int heads, int tokens, int items, int tpi, int rph,
                   int mixed_from, int bh_count, int split_from, void* out, __half* out_q8d, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;  // [item parity][tile]
  uint8_t* sK = smem + 4 * TILE_BYTES;
  uint8_t* sV = sK + AST * TILE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + AST * TILE_BYTES);
  uint64_t* q_full = bars;             // [2] per Q buffer
  uint64_t* q_empty = q_full + 2;      // [2]
  uint64_t* kv_full = q_empty + 2;     // [AST]
  uint64_t* kv_empty = kv_full + AST;  // [AST]
  uint64_t* s_full = kv_empty + AST;   // [2] per tile: S_t(j) ready (and O_t(j-1) done)
  uint64_t* p_full = s_full + 2;       // [2] per tile
  uint64_t* o_done = p_full + 2;       // [2] per tile: the item's last O_t finished
  uint64_t* o_free = o_done + 2;       // [2 tiles][2 buffers]: the item's O has been read
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_free + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Items [0, mixed_from) are `tpi` (2, or 1 when pairs would leave SMs
  // idle) consecutive query tiles of one (image, head), `rph` of them per
  // head.  With pairs and an odd number of query tiles per head, each
  // head's last tile is paired instead with the next head's last tile
  // (items from mixed_from on): the two tiles then read different K / V,
  // but still ping-pong on the tensor core, where a lone tile would run its
  // chain without a partner.
  const int nt = (tokens + AQ - 1) / AQ;  // query tiles per head
  const int nb = (tokens + AKV - 1) / AKV;
  struct Item {
    int bh[2], q0[2];
    int ntiles;  // 1 or 2
    int kvs;     // K / V streams: 2 when the tiles belong to different heads
  };
  // Items from split_from on are the tiles of the last round's two-tile
  // items taken one by one (2 per such item), so that a last round that
  // would leave most CTAs idle is spread over twice as many CTAs.
  auto pair_of = [&](int it) {
    Item r;
    if (it < mixed_from) {
      const int b = it / rph, p = it - b * rph;
      r.bh[0] = r.bh[1] = b;
      r.q0[0] = p * tpi * AQ;
      r.q0[1] = r.q0[0] + AQ;
      r.ntiles = (tpi == 2 && tokens - r.q0[0] > AQ) ? 2 : 1;  // tile 1 may not exist
      r.kvs = 1;
    } else {
      const int m = it - mixed_from;
      r.bh[0] = 2 * m;
      r.bh[1] = 2 * m + 1;
      r.q0[0] = r.q0[1] = (nt - 1) * AQ;
      r.ntiles = r.bh[1] < bh_count ? 2 : 1;
      r.kvs = r.ntiles;
    }
    return r;
  };
  auto item_of = [&](int it) {
    if (it < split_from) return pair_of(it);
    const int u = it - split_from;
    Item r = pair_of(split_from + (u >> 1));  // a two-tile item (the host checks)
    if (u & 1) {
      r.bh[0] = r.bh[1];
      r.q0[0] = r.q0[1];
    }
    r.ntiles = 1;
    r.kvs = 1;
    return r;
  };

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&q_full[b], 1);
      mbar_init(&q_empty[b], 1);
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 4);  // one arrival per softmax warp
      mbar_init(&o_done[b], 1);
    }
    for (int b = 0; b < 4; ++b) mbar_init(&o_free[b], 4);
    for (int s = 0; s < AST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dependency_wait();  // q, k, v from the QKV GEMM are visible from here

  if (warp == 0) {
    if (lane == 0) {
      uint32_t g = 0;  // K/V stages loaded so far
      bool ok = true;
      for (int it = blockIdx.x, c = 0; it < items && ok; it += gridDim.x, ++c) {
        const Item I = item_of(it);
        const int qb = c & 1;
        if (c >= 2 && !mbar_wait(&q_empty[qb], ((c >> 1) - 1) & 1, err, VK_DEV_TIMEOUT_PRODUCER)) break;
        mbar_arrive_expect_tx(&q_full[qb], I.ntiles * TILE_BYTES);
        for (int t = 0; t < I.ntiles; ++t)
          tma_load_3d(sQ + (qb * 2 + t) * TILE_BYTES, &tmQ, &q_full[qb], 0, t ? I.q0[1] : I.q0[0], t ? I.bh[1] : I.bh[0]);
        // per key block, one stage per K / V stream (in tile order)
        for (int j = 0; j < nb && ok; ++j) {
          for (int u = 0; u < I.kvs; ++u, ++g) {
            const uint32_t st = g % AST;
            if (!mbar_wait(&kv_empty[st], ((g / AST) & 1) ^ 1, err, VK_DEV_TIMEOUT_PRODUCER)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&kv_full[st], 2 * TILE_BYTES);
            tma_load_3d(sK + st * TILE_BYTES, &tmK, &kv_full[st], 0, j * AKV, u ? I.bh[1] : I.bh[0]);
            tma_load_3d(sV + st * TILE_BYTES, &tmV, &kv_full[st], 0, j * AKV, u ? I.bh[1] : I.bh[0]);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(128, 128);
      constexpr uint32_t idO = idesc_f16_bmn(128, 64);
      auto issue_s = [&](int t, int qb, uint32_t st) {
        const uint64_t qdesc = smem_desc_k_sw128(smem_u32(sQ + (qb * 2 + t) * TILE_BYTES));
        const uint64_t kdesc = smem_desc_k_sw128(smem_u32(sK + st * TILE_BYTES));
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16(tmem + t * TILE_COLS + COL_S, qdesc + static_cast<uint64_t>(k * 2),
                   kdesc + static_cast<uint64_t>(k * 2), idS, k > 0 ? 1u : 0u);
      };
      uint32_t g = 0;                 // K/V stages consumed so far
      uint32_t sp[2] = {0u, 0u};      // per tile: S / P hand-offs so far
      uint32_t ct[2] = {0u, 0u};      // per tile: items so far
      bool ok = true;
      auto kv_wait = [&](uint32_t gg) {
        return mbar_wait(&kv_full[gg % AST], (gg / AST) & 1, err, VK_DEV_TIMEOUT_MMA);
      };
      for (int it = blockIdx.x, c = 0; it < items && ok; it += gridDim.x, ++c) {
        const Item I = item_of(it);
        const int ntiles = I.ntiles;
        const uint32_t kvs = static_cast<uint32_t>(I.kvs);
        const int qb = c & 1;
        if (!(ok = mbar_wait(&q_full[qb], (c >> 1) & 1, err, VK_DEV_TIMEOUT_MMA))) break;
        for (uint32_t u = 0; u < kvs && ok; ++u) ok = kv_wait(g + u);
        if (!ok) break;
        tc_fence_after();
        // stage of tile t's K / V for the block at stage base gb
        auto st_of = [&](uint32_t gb, int t) { return (gb + (kvs == 2 ? static_cast<uint32_t>(t) : 0u)) % AST; };
        for (int t = 0; t < ntiles; ++t) {  // the previous item's last O_t was issued before
          issue_s(t, qb, st_of(g, t));
          umma_commit(&s_full[t]);
        }
        for (int j = 0; j < nb && ok; ++j, g += kvs) {
          const bool more = j + 1 < nb;
          if (more && kvs == 1 && !(ok = kv_wait(g + 1))) break;
          for (int t = 0; t < ntiles && ok; ++t) {
            if (more && kvs == 2 && !(ok = kv_wait(g + 2 + t))) break;
            const uint64_t vdesc = smem_desc_mn_sw128(smem_u32(sV + st_of(g, t) * TILE_BYTES));
            if (!(ok = mbar_wait(&p_full[t], sp[t] & 1, err, VK_DEV_TIMEOUT_MMA))) break;
            ++sp[t];
            const uint32_t ob = ct[t] & 1;
            // the first O of an item overwrites buffer ob: item ct-2's output must have been read
            if (j == 0 && ct[t] >= 2 &&
                !(ok = mbar_wait(&o_free[t * 2 + ob], ((ct[t] >> 1) - 1) & 1, err, VK_DEV_TIMEOUT_MMA)))
              break;
            tc_fence_after();
            const uint32_t base = tmem + t * TILE_COLS;
#pragma unroll
            for (int k = 0; k < AKV / 16; ++k)
              umma_f16_ts(base + COL_O + ob * 64, base + COL_S + static_cast<uint32_t>(k * 8),
                          vdesc + static_cast<uint64_t>(k * (2048 >> 4)), idO, (j | k) > 0 ? 1u : 0u);
            if constexpr (SPLIT) {
#pragma unroll
              for (int k = 0; k < AKV / 16; ++k)
                umma_f16_ts(base + COL_O + ob * 64, base + COL_S + 64 + static_cast<uint32_t>(k * 8),
                            vdesc + static_cast<uint64_t>(k * (2048 >> 4)), idO, 1u);
            }
            if (more) {
              issue_s(t, qb, st_of(g + kvs, t));
              umma_commit(&s_full[t]);  // also covers O_t(j)
            } else {
              umma_commit(&o_done[t]);
            }
            if (kvs == 2) umma_commit(&kv_empty[st_of(g, t)]);  // this tile's stage: S_t(j), O_t(j) issued
          }
          if (ok && kvs == 1) umma_commit(&kv_empty[g % AST]);  // after every MMA that read this stage
        }
        if (!ok) break;
        umma_commit(&q_empty[qb]);  // every S of this item has been issued
        for (int t = 0; t < ntiles; ++t) ++ct[t];
      }
    }
  } else {
    const int t = (warp - 2) >> 2;  // tile of this softmax warp
    const int quad = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tb = tmem + t * TILE_COLS + lane_base;
    const float sl2 = 0.125f * 1.4426950408889634f;  // (1/sqrt(64)) * log2(e)
    uint32_t sp = 0, ct = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
      const Item I = item_of(it);
      if (t >= I.ntiles) continue;
      const int bh = t ? I.bh[1] : I.bh[0], q0 = t ? I.q0[1] : I.q0[0];
      if (it + static_cast<int>(gridDim.x) >= items && items <= VK_EARLY_LAUNCH_ROUNDS * static_cast<int>(gridDim.x))
        grid_launch_dependents();
      const int qrow = q0 + quad * 32 + lane;
      const uint32_t col_o = COL_O + (ct & 1) * 64;
      float m_ref = -INFINITY;
      float l_run = 0.0f;
      for (int j = 0; j < nb; ++j, ++sp) {
        // warp-uniform outcome: the TMEM reads after the wait are warp-collective
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[t], sp & 1, err, VK_DEV_TIMEOUT_EPILOGUE))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int valid = tokens - j * AKV;
        const bool full_block = valid >= AKV;
        // block max over S(j), 32 TMEM columns at a time
        auto block_max = [&]() -> float {
          float pm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t r[32];
            tmem_ld32(tb + COL_S + c * 32, r);
            tmem_wait_ld();
            if (full_block) {
#pragma unroll
              for (int i = 0; i < 32; i += 2)
                pm[(i >> 1) & 3] = max3f(pm[(i >> 1) & 3], __uint_as_float(r[i]), __uint_as_float(r[i + 1]));
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (c * 32 + i < valid) pm[i & 3] = fmaxf(pm[i & 3], __uint_as_float(r[i]));
            }
          }
          return fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])) * sl2;
        };
        // p = 2^(s * log2e / 8 - m) packed as f16 pairs into pk; returns the row sum
        uint32_t pk[64];
        // set_ref (block 0): the reference m_ref is taken from the first 64
        // keys, already in registers, instead of a separate max pass over S;
        // keys past them may then give p above 1 (the 2^15 check below covers
        // them).
        auto exp_pass = [&](float m, bool set_ref) -> float {
          float2 ps[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
          float2 shift2 = make_float2(-m, -m);
          const float2 scale2 = make_float2(sl2, sl2);
#pragma unroll
          for (int c = 0; c < 4; c += 2) {
            uint32_t rr[64];
            tmem_ld32(tb + COL_S + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&rr[0]));
            tmem_ld32(tb + COL_S + c * 32 + 32, *reinterpret_cast<uint32_t(*)[32]>(&rr[32]));
            tmem_wait_ld();
            if (c == 0 && set_ref) {
              float pm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
              if (full_block) {
#pragma unroll
                for (int i = 0; i < 64; i += 2)
                  pm[(i >> 1) & 3] = max3f(pm[(i >> 1) & 3], __uint_as_float(rr[i]), __uint_as_float(rr[i + 1]));
              } else {
#pragma unroll
                for (int i = 0; i < 64; ++i)
                  if (i < valid) pm[i & 3] = fmaxf(pm[i & 3], __uint_as_float(rr[i]));
              }
              m_ref = fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])) * sl2;
              shift2 = make_float2(-m_ref, -m_ref);
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int k0 = c * 32 + 2 * i;
              const float2 x = ffma2(make_float2(__uint_as_float(rr[2 * i]), __uint_as_float(rr[2 * i + 1])), scale2, shift2);
              float2 pp = ((POLY_MASK >> (i & 15)) & 1) ? exp2_poly2(x)                                  // FMA pipe
                                                 : make_float2(ex2_approx(x.x), ex2_approx(x.y));  // MUFU
              if (!full_block) {
                pp.x = k0 < valid ? pp.x : 0.0f;
                pp.y = k0 + 1 < valid ? pp.y : 0.0f;
              }
              ps[i & 1] = fadd2(ps[i & 1], pp);
              pk[c * 16 + i] = pack_f16x2(pp.x, pp.y);
            }
          }
          return (ps[0].x + ps[0].y) + (ps[1].x + ps[1].y);
        };
        if constexpr (SPLIT) {
          // p = 2^(s log2e / 8 - m) as P_hi = f16(p) over columns [0, 64) and
          // P_lo = f16(p - P_hi) over [64, 128).  The block max is taken first,
          // so P can be written while S is still being read: keys [0, 64) are
          // read first, their P_hi lands on columns already read, their P_lo
          // waits in registers until columns [64, 128) have been read too.
          auto exp_split = [&](float m) -> float {
            float2 ps[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
            const float2 scale2 = make_float2(sl2, sl2), shift2 = make_float2(-m, -m);
            uint32_t lo_hold[32];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              uint32_t rr[64];
              tmem_ld32(tb + COL_S + h * 64, *reinterpret_cast<uint32_t(*)[32]>(&rr[0]));
              tmem_ld32(tb + COL_S + h * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&rr[32]));
              tmem_wait_ld();
              if (h == 1) {
                tmem_st16(tb + COL_S + 64, *reinterpret_cast<uint32_t(*)[16]>(&lo_hold[0]));
                tmem_st16(tb + COL_S + 80, *reinterpret_cast<uint32_t(*)[16]>(&lo_hold[16]));
              }
#pragma unroll
              for (int sub = 0; sub < 2; ++sub) {
                uint32_t hi16[16], lo16[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  const int pi = sub * 16 + i;  // pair within this half
                  const int k0 = h * 64 + 2 * pi;
                  const float2 x = ffma2(make_float2(__uint_as_float(rr[2 * pi]), __uint_as_float(rr[2 * pi + 1])),
                                         scale2, shift2);
                  float2 pp = make_float2(ex2_approx(x.x), ex2_approx(x.y));
                  if (!full_block) {
                    pp.x = k0 < valid ? pp.x : 0.0f;
                    pp.y = k0 + 1 < valid ? pp.y : 0.0f;
                  }
                  ps[i & 1] = fadd2(ps[i & 1], pp);
                  const __half2 hh = __floats2half2_rn(pp.x, pp.y);
                  const float2 hf = __half22float2(hh);
                  hi16[i] = *reinterpret_cast<const uint32_t*>(&hh);
                  lo16[i] = pack_f16x2(pp.x - hf.x, pp.y - hf.y);
                }
                tmem_st16(tb + COL_S + h * 32 + sub * 16, hi16);
                if (h == 1) {
                  tmem_st16(tb + COL_S + 96 + sub * 16, lo16);
                } else {
#pragma unroll
                  for (int i = 0; i < 16; ++i) lo_hold[sub * 16 + i] = lo16[i];
                }
              }
            }
            return (ps[0].x + ps[0].y) + (ps[1].x + ps[1].y);
          };
          const float bm = block_max();
          if (j == 0) {
            m_ref = bm;
          } else if (__any_sync(0xffffffffu, bm > m_ref + 15.0f)) {  // some p would reach 2^15
            const float m_new = fmaxf(m_ref, bm);
            const float f = ex2_approx(m_ref - m_new);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              uint32_t o[32];
              tmem_ld32(tb + col_o + h * 32, o);
              tmem_wait_ld();
#pragma unroll
              for (int d = 0; d < 32; ++d) o[d] = __float_as_uint(__uint_as_float(o[d]) * f);
              tmem_st32(tb + col_o + h * 32, o);
            }
            l_run *= f;
            m_ref = m_new;
          }
          const float l_blk = exp_split(m_ref);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_full[t]);
          l_run += l_blk;
          continue;
        }
        // One pass against the running reference m_ref (the max of block 0, or
        // of a later block that outgrew it).  Probabilities above 1 are fine:
        // the final O / l is invariant to the reference.  P is stored as f16
        // (largest finite 65504), so when a row's block sum reaches 2^15 (every
        // p of the row is then below it) the block is redone against its own
        // max, with O and l rescaled to match (O_t(j-1) is complete: S_t(j)
        // was issued after it).  Probabilities below the f16 range round to
        // zero: at most 2^-24 each, against a row sum of at least 1.
        float l_blk = exp_pass(m_ref, j == 0);
        // (in block 0 O holds nothing of this item yet: rescaling it is harmless,
        // the item's first P V overwrites it)
        if (__any_sync(0xffffffffu, !(l_blk < 32768.0f))) {  // TMEM access is warp-collective
          const float m_new = fmaxf(m_ref, block_max());
          const float f = ex2_approx(m_ref - m_new);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t o[32];
            tmem_ld32(tb + col_o + h * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int d = 0; d < 32; ++d) o[d] = __float_as_uint(__uint_as_float(o[d]) * f);
            tmem_st32(tb + col_o + h * 32, o);
          }
          l_run *= f;
          m_ref = m_new;
          l_blk = exp_pass(m_ref, false);
        }
        // P over the first 64 columns of S (S is no longer needed)
        tmem_st32(tb + COL_S, *reinterpret_cast<uint32_t(*)[32]>(&pk[0]));
        tmem_st32(tb + COL_S + 32, *reinterpret_cast<uint32_t(*)[32]>(&pk[32]));
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
        l_run += l_blk;
      }
      if (!ok || !__all_sync(0xffffffffu, mbar_wait(&o_done[t], ct & 1, err, VK_DEV_TIMEOUT_EPILOGUE))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float o[64];
      const float inv = 1.0f / l_run;
      tmem_ld32(tb + col_o, *reinterpret_cast<uint32_t(*)[32]>(&o[0]));
      tmem_ld32(tb + col_o + 32, *reinterpret_cast<uint32_t(*)[32]>(&o[32]));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[t * 2 + (ct & 1)]);  // O is in registers: item ct+2 may overwrite it
      ++ct;
#pragma unroll
      for (int d = 0; d < 64; ++d) o[d] *= inv;
      if (qrow < tokens) {
        const int b_img = bh / heads, h = bh - b_img * heads;
        if constexpr (OUT == ATTN_OUT_HEAD_F32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(out) + (static_cast<size_t>(bh) * tokens + qrow) * 64);
#pragma unroll
          for (int d = 0; d < 16; ++d) dst[d] = make_float4(o[4 * d], o[4 * d + 1], o[4 * d + 2], o[4 * d + 3]);
        } else if constexpr (OUT == ATTN_OUT_TOKEN_BF16) {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) +
                                                (static_cast<size_t>(b_img) * tokens + qrow) * (heads * 64) + h * 64);
#pragma unroll
          for (int d = 0; d < 8; ++d)
            dst[d] = make_uint4(pack_bf16x2(o[8 * d], o[8 * d + 1]), pack_bf16x2(o[8 * d + 2], o[8 * d + 3]),
                                pack_bf16x2(o[8 * d + 4], o[8 * d + 5]), pack_bf16x2(o[8 * d + 6], o[8 * d + 7]));
        } else {
          // two Q8_0 blocks of 32 dims (quantize_row_q8_0, src/q8_0_dot.rs:34-45)
          const size_t row = static_cast<size_t>(b_img) * tokens + qrow;
          int8_t* dst = static_cast<int8_t*>(out) + row * (heads * 64) + h * 64;
#pragma unroll
          for (int blk = 0; blk < 2; ++blk) {
            float amax = 0.0f;
#pragma unroll
            for (int d = 0; d < 32; ++d) amax = fmaxf(amax, fabsf(o[blk * 32 + d]));
            const float dd = amax / 127.0f;
            const float id = dd != 0.0f ? 1.0f / dd : 0.0f;
            uint32_t w[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              uint32_t packed = 0;
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const float qf = fminf(fmaxf(roundf(o[blk * 32 + 4 * q + u] * id), -127.0f), 127.0f);
                packed |= (static_cast<uint32_t>(static_cast<int32_t>(qf)) & 0xffu) << (8 * u);
              }
              w[q] = packed;
            }
            uint4* d4 = reinterpret_cast<uint4*>(dst + blk * 32);
            d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
            d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
            out_q8d[row * (heads * 2) + h * 2 + blk] = __float2half_rn(dd);
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int OUT, bool SPLIT>
static cudaError_t launch_attn(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, int images,
                               int heads, int tokens, void* out, __half* q8d, int* err, cudaStream_t s) {
  cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(k_attention_tc<OUT, SPLIT>), static_cast<int>(ATT_SMEM));
  if (e != cudaSuccess) return e;
  // tile pairs share each K/V block; single tiles when pairs would not fill
  // the SMs.  With pairs and an odd tile count per head, the heads' last
  // tiles pair up across heads (items from mixed_from on).
  const int bh_count = images * heads;
  const int nt = (tokens + AQ - 1) / AQ;
  int tpi = 2;
  if (((tokens + 2 * AQ - 1) / (2 * AQ)) * bh_count < num_sms()) tpi = 1;
  static const bool no_mix = getenv("VK_ATT_NO_MIX") != nullptr;
  int rph, mixed_from, items;
  if (tpi == 1) {
    rph = nt;
    items = mixed_from = nt * bh_count;
  } else if (no_mix || nt % 2 == 0) {
    // (VK_ATT_NO_MIX: a head's odd last tile runs alone, as its own item)
    rph = (nt + 1) / 2;
    items = mixed_from = rph * bh_count;
  } else {
    rph = nt / 2;
    mixed_from = rph * bh_count;
    items = mixed_from + (bh_count + 1) / 2;
  }
  // A last round of r two-tile items on the persistent grid leaves the other
  // CTAs idle while it runs; when 2 r single tiles fit in one round, run the
  // r items as single tiles instead (a lone tile takes about 0.87 of a pair's
  // time).  Every item in that range must hold two tiles.
  int split_from = items;
  static const bool no_split = getenv("VK_ATT_NO_SPLIT_TAIL") != nullptr;
  const int g0 = num_sms();
  const int r = items % g0;
  // every item holds two tiles: cross-head items pair all heads (an even
  // count), and otherwise each head's last pair has its second tile
  const bool last_pairs = tpi == 2 && (items == mixed_from ? (tokens - (rph - 1) * 2 * AQ > AQ) : (bh_count % 2 == 0));
  if (!no_split && items > g0 && r > 0 && 2 * r <= g0 && last_pairs) {
    split_from = items - r;
    items += r;
  }
  const int grid = items < num_sms() ? items : num_sms();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(A_THREADS);
  cfg.dynamicSmemBytes = ATT_SMEM;
  cfg.stream = s;
  cudaLaunchAttribute la[1];
  la[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  la[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = la;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k_attention_tc<OUT, SPLIT>, mq, mk, mv, heads, tokens, items, tpi, rph, mixed_from,
                            bh_count, split_from, out, q8d, err);
}

cudaError_t attention_bf16(const __nv_bfloat16* q, const __nv_bfloat16* k, const __half* v, int images,
                           int heads, int tokens, int out_mode, void* out, __half* out_q8d, int* err,
                           cudaStream_t s, bool precise) {
  if (images <= 0 || heads <= 0 || tokens <= 0) return cudaErrorInvalidValue;
  CUtensorMap mq, mk, mv;
  const uint64_t bh = static_cast<uint64_t>(images) * heads;
  const void* bases[3] = {q, k, v};
  CUtensorMap* maps[3] = {&mq, &mk, &mv};
  for (int i = 0; i < 3; ++i)
    if (!make_tmap_3d(maps[i], i == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, bases[i], 64, tokens, bh, 128,
                      static_cast<uint64_t>(tokens) * 128, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  // The split-P product for the Q8_0 output (its quantisation steps of
  // about 1/127 amplify any error of O), for the head-major f32 output of the
  // operator API, and for the encoder's bf16 output when the caller asks
  // (`precise`: layers with Q/K LayerNorm) or with VK_ATT_SPLIT=1.
  static const bool split_bf16 = [] {
    const char* e = getenv("VK_ATT_SPLIT");
    return e != nullptr && e[0] == '1';
  }();
  switch (out_mode) {
    case ATTN_OUT_HEAD_F32: {
      // VK_ATT_API_SPLIT=0 runs the operator on the single-f16-P kernel the
      // bf16 encoder uses (read per call: the parity tests switch it)
      const char* e = getenv("VK_ATT_API_SPLIT");
      if (e != nullptr && e[0] == '0')
        return launch_attn<ATTN_OUT_HEAD_F32, false>(mq, mk, mv, images, heads, tokens, out, out_q8d, err, s);
      return launch_attn<ATTN_OUT_HEAD_F32, true>(mq, mk, mv, images, heads, tokens, out, out_q8d, err, s);
    }
    case ATTN_OUT_TOKEN_BF16:
      return split_bf16 || precise ? launch_attn<ATTN_OUT_TOKEN_BF16, true>(mq, mk, mv, images, heads, tokens, out, out_q8d, err, s)
                        : launch_attn<ATTN_OUT_TOKEN_BF16, false>(mq, mk, mv, images, heads, tokens, out, out_q8d, err, s);
    case ATTN_OUT_TOKEN_Q8:
      return launch_attn<ATTN_OUT_TOKEN_Q8, true>(mq, mk, mv, images, heads, tokens, out, out_q8d, err, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace vk
