// Dense "TN" GEMM on the 5th-generation tensor cores (tcgen05), for sm_100a:
//
//   C[M, N] (+)= A[M, K] . B[N, K]^T (+ bias[N])
//
// A and B are fp16 or bf16 (the same type, row-major with K contiguous); the accumulator is fp32
// in tensor memory; C is fp16, bf16 or fp32 with a row stride. This replaces the cuBLAS
// `torch.addmm` / `torch.mm` calls of the reference step (solution/engine.py:1081-1093,
// 1111-1112, 1132-1139, 1163-1165, 1178-1179, 1238-1316, 1386-1390).
//
// Structure: a persistent, warp-specialised kernel with one CTA per SM.
//   warp 0      TMA producer: 128 x 64 tiles of A and BN x 64 tiles of B (BN = 96 .. 256, picked
//               per shape so that the output tiles fill whole waves of SMs) into a ring of STAGES
//               shared-memory slots (128-byte swizzle), completion counted on an mbarrier;
//   warp 1      allocates 2 x BN TMEM columns (two accumulators) and issues tcgen05.mma from one
//               thread, 4 x (K = 16) per 64-wide K step; tcgen05.commit frees each slot and, at
//               the end of a tile, signals the epilogue;
//   warps 2-5   epilogue: tcgen05.ld of their 32 TMEM lanes, bias add, conversion, stores.
// The accumulator of tile t+1 is written while the epilogue drains tile t.
#include <atomic>
#include <cstring>
#include <unordered_map>

#include "common.cuh"
#include "gemm_common.cuh"
#include "profile.h"

namespace ql {

template <int BN, bool IS_BF16, typename OutT, bool B_MN, int KC>
__global__ void __launch_bounds__(192, 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                   const __grid_constant__ CUtensorMap tma_c, GemmArgs p) {
  pdl_trigger();  // setup below reads no global memory; pdl_wait() follows it
  constexpr bool kTmaC = sizeof(OutT) == 2;
  using Cfg = GemmCfg<BN, kTmaC, KC>;
  using InT = typename std::conditional<IS_BF16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_stage = smem + Cfg::STAGES * Cfg::STAGE_BYTES;  // EPI bytes (16-bit C only)
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + Cfg::EPI);
  uint64_t* empty = full + Cfg::STAGES;
  uint64_t* tfull = empty + Cfg::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (int)cdiv(p.M, Cfg::BM), n_tiles = (int)cdiv(p.N, BN);
  const int num_tiles = m_tiles * n_tiles;
  const int k_blocks = (int)cdiv(p.K, Cfg::BK);
  const int S = p.splits;
  const int num_units = num_tiles * S;  // unit u: tile u / S, split u % S

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    fence_barrier_init();
    prefetch_tmap(&tma_a);
    prefetch_tmap(&tma_b);
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the previous kernel's results (A, counters, C) are visible from here on

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        const int tile = u / S, sp = u % S;
        const int mb = tile % m_tiles, nb = tile / m_tiles;
        const int kb0 = sp * p.kb_per_split, kb1 = min(k_blocks, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) { ok = false; break; }
          uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          if constexpr (KC == 2) {  // one 3-D copy per operand: two 64-wide K chunks
            tma_load_3d(sa, &tma_a, &full[stage], 0, mb * Cfg::BM, kb * 2);
            if constexpr (B_MN)  // [BN / 64 N chunks][128 K rows][64]
              tma_load_3d(sb, &tma_b, &full[stage], 0, kb * Cfg::BK, nb * (BN / 64));
            else
              tma_load_3d(sb, &tma_b, &full[stage], 0, nb * BN, kb * 2);
          } else {
            tma_load_2d(sa, &tma_a, &full[stage], kb * Cfg::BK, mb * Cfg::BM);
            if constexpr (B_MN) {  // B stored [K, N]: boxes of 64 N-columns x 64 K-rows, 8 KB each
              if (p.b3d) {  // all of them in one 3-D copy ([BN / 64 chunks][64 K rows][64])
                tma_load_3d(sb, &tma_b, &full[stage], 0, kb * Cfg::BK, nb * (BN / 64));
              } else {
#pragma unroll
                for (int j = 0; j < BN / 64; ++j)
                  tma_load_2d(sb + j * 8192, &tma_b, &full[stage], nb * BN + j * 64, kb * Cfg::BK);
              }
            } else {
              tma_load_2d(sb, &tma_b, &full[stage], kb * Cfg::BK, nb * BN);
            }
          }
          if (++stage == Cfg::STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(IS_BF16, 128, BN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++local) {
        const int sp = u % S;
        const int kb0 = sp * p.kb_per_split, kb1 = min(k_blocks, kb0 + p.kb_per_split);
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, p.err)) break;
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < Cfg::BK / 16; ++k) {  // K chunk k / 4, 16-wide step k % 4 of it
            const uint32_t ka = (k >> 2) * (Cfg::BM * 128) + (k & 3) * 32;
            const uint64_t db = B_MN ? umma_desc_mn_sw128(sb + k * 2048, Cfg::BK * 128, 1024)
                                     : umma_desc_k_sw128(sb + (k >> 2) * (BN * 128) + (k & 3) * 32);
            umma_f16(tmem_d, umma_desc_k_sw128(sa + ka), db, idesc,
                     (kb != kb0 || k != 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == Cfg::STAGES) { stage = 0; phase ^= 1; }
        }
        if (ok) umma_commit(&tfull[acc]);
      }
    }
  } else {
    // epilogue warps 2..5: TMEM lane quadrant = warp % 4
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    int local = 0;
    OutT* C = reinterpret_cast<OutT*>(p.C);
    const InT* bias = reinterpret_cast<const InT*>(p.bias);
    __shared__ int last_flag;
    int ebuf = 0;  // TMA-store staging buffer of this warp
    for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++local) {
      const int tile = u / S, sp = u % S;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase, p.err)) break;
      tc_fence_after();
      const int mb = tile % m_tiles, nb = tile / m_tiles;
      const int row = mb * Cfg::BM + row_in_tile;
      const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN;
      bool finish = true;  // this unit writes the output tile
      float* part = nullptr;
      if (S > 1) {
        // this split's fp32 partial, stored column-major within the tile ([BN][128 rows]) so
        // that the 32 lanes of a warp (32 consecutive rows) write and read whole 128-byte lines
        part = p.ws + ((int64_t)tile * S) * Cfg::BM * BN;
        float* mine = part + (int64_t)sp * Cfg::BM * BN + row_in_tile;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          tmem_ld32(taddr + c, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) __stcg(mine + (c + i) * Cfg::BM, v[i]);
        }
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");  // the 4 epilogue warps
        if (threadIdx.x == 64) {
          const int old = atomicAdd(p.counters + tile, 1);
          last_flag = (old == S - 1);
          if (old == S - 1) p.counters[tile] = 0;  // ready for the next launch
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        finish = last_flag != 0;
        if (finish) __threadfence();
      }
      if (finish) {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          if (S > 1) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0.f;
            const float* src = part + row_in_tile + (int64_t)c * Cfg::BM;
            for (int j = 0; j < S; j += 2) {  // fixed order p0 + p1 + ...: reproducible sums
              float x0[32], x1[32];
              const float* s0 = src + (int64_t)j * Cfg::BM * BN;
              const bool two = j + 1 < S;
#pragma unroll
              for (int i = 0; i < 32; ++i) x0[i] = __ldcg(s0 + i * Cfg::BM);
#pragma unroll
              for (int i = 0; i < 32; ++i) x1[i] = two ? __ldcg(s0 + Cfg::BM * BN + i * Cfg::BM) : 0.f;
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] += x0[i];
              if (two) {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] += x1[i];
              }
            }
          } else {
            tmem_ld32(taddr + c, v);
          }
          const int col0 = nb * BN + c;
          if constexpr (kTmaC) {
            if (p.tma_c) {
              const int wrow0 = mb * Cfg::BM + quad * 32;  // this warp's 32 rows
              if (col0 < p.N && wrow0 < p.M) {
                if (bias != nullptr) {
#pragma unroll
                  for (int i = 0; i < 32; ++i)
                    if (col0 + i < p.N) v[i] += to_f<InT>(bias[col0 + i]);
                }
                epi_tma_chunk<OutT>(&tma_c, epi_stage + quad * 4096, ebuf, v, col0, wrow0);
              }
              continue;
            }
          }
          if (row < p.M && col0 < p.N) {
            const int ncols = min(32, p.N - col0);
            if (bias != nullptr) {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (i < ncols) v[i] += to_f<InT>(bias[col0 + i]);
            }
            OutT* dst = C + (int64_t)row * p.ldc + col0;
            if constexpr (sizeof(OutT) == 4) {
              if (p.residual != nullptr) {
                const float* res = p.residual + (int64_t)row * p.ldc + col0;
#pragma unroll
                for (int i = 0; i < 32; ++i)
                  if (i < ncols) v[i] = to_f<InT>(from_f<InT>(v[i])) + res[i];
              } else if (p.accumulate) {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                  if (i < ncols) v[i] += to_f<OutT>(dst[i]);
              }
            }
            store_row32<OutT>(dst, v, ncols);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
    if (kTmaC && p.tma_c && lane == 0) bulk_wait<0>();  // this warp's stores are complete
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------------
// 2-SM variant: clusters of two CTAs compute 256 x BN pair tiles with tcgen05.mma.cta_group::2.
// CTA r of the pair loads rows [128 r, 128 r + 128) of the A tile and half r of the B tile (BN/2
// rows, or BN/2 columns of an MN-major B); the even CTA issues the MMAs, which read both halves
// and leave rows 0-127 of the accumulator in its TMEM and rows 128-255 in the odd CTA's. Per CTA
// and K step the operands are 16 KB + BN x 64 B for 128 x BN outputs: a third fewer bytes per
// FLOP than the single-CTA tile at BN = 256, the limit of that kernel.
//   full[s]   even CTA's: its producer expects both CTAs' bytes; the odd CTA's loads count there
//   empty[s]  each CTA's: the even CTA's MMA commit arrives in both (CTA mask 0b11)
//   tfull[a]  each CTA's: the accumulator is complete (commit to both)
//   tempty[a] even CTA's: 8 arrivals, the 4 epilogue warps of each CTA
// ---------------------------------------------------------------------------------------------
template <int BN, bool kEpi = false, int KC = 1>
struct PairCfg {
  static constexpr int BM = 128, BK = 64 * KC, HB = BN / 2;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = HB * BK * 2;  // this CTA's half of B
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI = kEpi ? EPI_BYTES : 0;
  static constexpr int STAGES_FIT = (225 * 1024 - 1280 - EPI) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int TMEM_COLS = 2 * BN <= 256 ? 256 : 512;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI + 1024 + 256;
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "UMMA N (M = 256) and 32-column epilogue");
  static_assert(B_BYTES % 1024 == 0, "128-byte swizzle atoms of 8 rows");
};

template <int BN, bool IS_BF16, typename OutT, bool B_MN, int KC>
__global__ void __launch_bounds__(192, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tma_a,
                     const __grid_constant__ CUtensorMap tma_b,
                     const __grid_constant__ CUtensorMap tma_c, GemmArgs p) {
  pdl_trigger();  // setup below reads no global memory; pdl_wait() follows it
  constexpr bool kTmaC = sizeof(OutT) == 2;
  using Cfg = PairCfg<BN, kTmaC, KC>;
  using InT = typename std::conditional<IS_BF16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_stage = smem + Cfg::STAGES * Cfg::STAGE_BYTES;  // EPI bytes (16-bit C only)
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + Cfg::EPI);
  uint64_t* empty = full + Cfg::STAGES;
  uint64_t* tfull = empty + Cfg::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int m_pairs = (int)cdiv(p.M, 2 * Cfg::BM), n_tiles = (int)cdiv(p.N, BN);
  const int S = p.splits;  // unit u: pair tile u / S, K split u % S
  const int num_units = m_pairs * n_tiles * S;
  const int k_blocks = (int)cdiv(p.K, Cfg::BK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);
    }
    fence_barrier_init();
    prefetch_tmap(&tma_a);
    prefetch_tmap(&tma_b);
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the previous kernel's results are visible from here on

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = pair; u < num_units && ok; u += npairs) {
        const int tile = u / S, sp = u % S;
        const int mp = tile % m_pairs, nb = tile / m_pairs;
        const int arow = mp * 2 * Cfg::BM + (int)rank * Cfg::BM;
        const int brow = nb * BN + (int)rank * Cfg::HB;
        const int kb0 = sp * p.kb_per_split, kb1 = min(k_blocks, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) { ok = false; break; }
          uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
          if constexpr (KC == 2) {  // one 3-D copy per operand: two 64-wide K chunks
            tma_load_3d_pair(sa, &tma_a, &full[stage], 0, arow, kb * 2);
            if constexpr (B_MN)
              tma_load_3d_pair(sb, &tma_b, &full[stage], 0, kb * Cfg::BK, brow / 64);
            else
              tma_load_3d_pair(sb, &tma_b, &full[stage], 0, brow, kb * 2);
          } else {
            tma_load_2d_pair(sa, &tma_a, &full[stage], kb * Cfg::BK, arow);
            if constexpr (B_MN) {
              if (p.b3d) {
                tma_load_3d_pair(sb, &tma_b, &full[stage], 0, kb * Cfg::BK, brow / 64);
              } else {
#pragma unroll
                for (int j = 0; j < Cfg::HB / 64; ++j)
                  tma_load_2d_pair(sb + j * 8192, &tma_b, &full[stage], brow + j * 64, kb * Cfg::BK);
              }
            } else {
              tma_load_2d_pair(sb, &tma_b, &full[stage], kb * Cfg::BK, brow);
            }
          }
          if (++stage == Cfg::STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = umma_idesc_f16(IS_BF16, 2 * Cfg::BM, BN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int u = pair; u < num_units && ok; u += npairs, ++local) {
        const int sp = u % S;
        const int kb0 = sp * p.kb_per_split, kb1 = min(k_blocks, kb0 + p.kb_per_split);
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, p.err)) break;
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < Cfg::BK / 16; ++k) {  // K chunk k / 4, 16-wide step k % 4 of it
            const uint32_t ka = (k >> 2) * (Cfg::BM * 128) + (k & 3) * 32;
            const uint64_t db = B_MN ? umma_desc_mn_sw128(sb + k * 2048, Cfg::BK * 128, 1024)
                                     : umma_desc_k_sw128(sb + (k >> 2) * (Cfg::HB * 128) + (k & 3) * 32);
            umma_f16_pair(tmem_d, umma_desc_k_sw128(sa + ka), db, idesc,
                          (kb != kb0 || k != 0) ? 1u : 0u);
          }
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == Cfg::STAGES) { stage = 0; phase ^= 1; }
        }
        if (ok) umma_commit_pair(&tfull[acc], 0x3);
      }
    }
  } else {
    // epilogue warps 2..5 of each CTA: TMEM lane quadrant = warp % 4, this CTA's 128 rows
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    int local = 0;
    OutT* C = reinterpret_cast<OutT*>(p.C);
    const InT* bias = reinterpret_cast<const InT*>(p.bias);
    int ebuf = 0;
    __shared__ int last_flag;
    for (int u = pair; u < num_units; u += npairs, ++local) {
      const int tile = u / S, sp = u % S;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase, p.err)) break;
      tc_fence_after();
      const int mp = tile % m_pairs, nb = tile / m_pairs;
      const int row = mp * 2 * Cfg::BM + (int)rank * Cfg::BM + row_in_tile;
      const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN;
      bool finish = true;  // this CTA writes its 128 rows of the output tile
      float* part = nullptr;
      if (S > 1) {
        // this CTA's 128 x BN sub-tile of the split: its fp32 partial, column-major within the
        // sub-tile so that a warp's 32 lanes (32 consecutive rows) write whole 128-byte lines;
        // the last of the S units of a sub-tile (its counter) adds them in split order
        const int64_t st = (int64_t)tile * 2 + rank;
        part = p.ws + st * S * Cfg::BM * BN;
        float* mine = part + (int64_t)sp * Cfg::BM * BN + row_in_tile;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          tmem_ld32(taddr + c, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) __stcg(mine + (c + i) * Cfg::BM, v[i]);
        }
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");  // the 4 epilogue warps
        if (threadIdx.x == 64) {
          const int old = atomicAdd(p.counters + st, 1);
          last_flag = (old == S - 1);
          if (old == S - 1) p.counters[st] = 0;  // ready for the next launch
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        finish = last_flag != 0;
        if (finish) __threadfence();
      }
#pragma unroll 1
      for (int c = 0; c < BN && finish; c += 32) {
        float v[32];
        if (S > 1) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.f;
          const float* src = part + row_in_tile + (int64_t)c * Cfg::BM;
          for (int j = 0; j < S; ++j) {  // fixed order p0 + p1 + ...: reproducible sums
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] += __ldcg(src + (int64_t)j * Cfg::BM * BN + i * Cfg::BM);
          }
        } else {
          tmem_ld32(taddr + c, v);
        }
        const int col0 = nb * BN + c;
        if constexpr (kTmaC) {
          if (p.tma_c) {
            const int wrow0 = mp * 2 * Cfg::BM + (int)rank * Cfg::BM + quad * 32;
            if (col0 < p.N && wrow0 < p.M) {
              if (bias != nullptr) {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                  if (col0 + i < p.N) v[i] += to_f<InT>(bias[col0 + i]);
              }
              epi_tma_chunk<OutT>(&tma_c, epi_stage + quad * 4096, ebuf, v, col0, wrow0);
            }
            continue;
          }
        }
        if (row < p.M && col0 < p.N) {
          const int ncols = min(32, p.N - col0);
          if (bias != nullptr) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < ncols) v[i] += to_f<InT>(bias[col0 + i]);
          }
          OutT* dst = C + (int64_t)row * p.ldc + col0;
          if constexpr (sizeof(OutT) == 4) {
            if (p.residual != nullptr) {
              const float* res = p.residual + (int64_t)row * p.ldc + col0;
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (i < ncols) v[i] = to_f<InT>(from_f<InT>(v[i])) + res[i];
            } else if (p.accumulate) {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (i < ncols) v[i] += to_f<OutT>(dst[i]);
            }
          }
          store_row32<OutT>(dst, v, ncols);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(&tempty[acc]);
        else mbar_arrive_cluster(&tempty[acc], 0);
      }
    }
    if (kTmaC && p.tma_c && lane == 0) bulk_wait<0>();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the pair's MMAs and both epilogues are done before the collective dealloc
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
template <int BN, bool IS_BF16, typename OutT, bool B_MN, int KC>
static int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const GemmArgs& a,
                       cudaStream_t stream) {
  using Cfg = GemmCfg<BN, sizeof(OutT) == 2, KC>;
  static_assert(Cfg::STAGES >= 2, "at least two pipeline stages");
  auto kern = gemm_tn_kernel<BN, IS_BF16, OutT, B_MN, KC>;
  static bool configured = false;  // one static per instantiation
  if (!configured) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES) !=
        cudaSuccess)
      return QL_STATUS_CUDA;
    configured = true;
  }
  const int units = (int)(cdiv(a.M, 128) * cdiv(a.N, BN)) * a.splits;
  const int grid = units < num_sms() ? units : num_sms();
  if (launch_k(kern, dim3(grid), dim3(192), Cfg::SMEM_BYTES, stream, ma, mb, mc, a) != cudaSuccess)
    return QL_STATUS_CUDA;
  return launched(1);
}

// Clusters of two CTAs that can be resident at once (a GPC's SM count can be odd), per kernel.
template <typename K>
static int pair_slots(K kern, int smem) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (num_sms() / 2));
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters <= 0) {
    cudaGetLastError();
    clusters = num_sms() / 2;
  }
  return clusters;
}

template <int BN, bool IS_BF16, typename OutT, bool B_MN, int KC>
static int launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const GemmArgs& a,
                       cudaStream_t stream) {
  using Cfg = PairCfg<BN, sizeof(OutT) == 2, KC>;
  static_assert(Cfg::STAGES >= 2, "at least two pipeline stages");
  auto kern = gemm_pair_kernel<BN, IS_BF16, OutT, B_MN, KC>;
  static int slots = 0;  // one per instantiation
  if (slots == 0) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES) !=
        cudaSuccess)
      return QL_STATUS_CUDA;
    slots = pair_slots(kern, Cfg::SMEM_BYTES);
  }
  const int units = (int)(cdiv(a.M, 2 * Cfg::BM) * cdiv(a.N, BN)) * a.splits;
  const int pairs = units < slots ? units : slots;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  if (cudaLaunchKernelEx(&cfg, kern, ma, mb, mc, a) != cudaSuccess) return QL_STATUS_CUDA;
  return launched(1);
}

template <int BN, bool IS_BF16, bool B_MN, int KC>
static int dispatch_pair_out(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const GemmArgs& a,
                             cudaStream_t s) {
  switch (a.out_dtype) {
    case QL_F16: return launch_pair<BN, IS_BF16, __half, B_MN, KC>(ma, mb, mc, a, s);
    case QL_BF16: return launch_pair<BN, IS_BF16, __nv_bfloat16, B_MN, KC>(ma, mb, mc, a, s);
    case QL_F32: return launch_pair<BN, IS_BF16, float, B_MN, KC>(ma, mb, mc, a, s);
  }
  return QL_STATUS_BAD_ARG;
}

template <int BN, bool B_MN>
static int dispatch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const GemmArgs& a,
                         bool bf16, int kc, cudaStream_t s) {
  if (kc != 1) return QL_STATUS_UNSUPPORTED;  // pair tiles keep single-chunk stages (gemm_core)
  return bf16 ? dispatch_pair_out<BN, true, B_MN, 1>(ma, mb, mc, a, s)
              : dispatch_pair_out<BN, false, B_MN, 1>(ma, mb, mc, a, s);
}

template <int BN, bool IS_BF16, bool B_MN, int KC>
static int dispatch_out(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const GemmArgs& a,
                        cudaStream_t s) {
  switch (a.out_dtype) {
    case QL_F16: return launch_gemm<BN, IS_BF16, __half, B_MN, KC>(ma, mb, mc, a, s);
    case QL_BF16: return launch_gemm<BN, IS_BF16, __nv_bfloat16, B_MN, KC>(ma, mb, mc, a, s);
    case QL_F32: return launch_gemm<BN, IS_BF16, float, B_MN, KC>(ma, mb, mc, a, s);
  }
  return QL_STATUS_BAD_ARG;
}

template <int BN, bool B_MN>
static int dispatch_in(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const GemmArgs& a, bool bf16,
                       int kc, cudaStream_t s) {
  if constexpr (BN <= 128) {  // two-chunk stages: tiles of up to 128 columns only (gemm_core)
    if (kc == 2)
      return bf16 ? dispatch_out<BN, true, B_MN, 2>(ma, mb, mc, a, s)
                  : dispatch_out<BN, false, B_MN, 2>(ma, mb, mc, a, s);
  }
  if (kc != 1) return QL_STATUS_UNSUPPORTED;
  return bf16 ? dispatch_out<BN, true, B_MN, 1>(ma, mb, mc, a, s)
              : dispatch_out<BN, false, B_MN, 1>(ma, mb, mc, a, s);
}

// Split-K workspace: tile counters first (a fixed region, left all-zero by every launch, so
// GEMMs of any shape can share one workspace), then the fp32 partial tiles.
constexpr int64_t kCounterBytes = 2048;  // 512 tiles: split-K only runs below 2 x SMs tiles

struct GemmPlan {
  int bn;
  int64_t tiles;
  int splits, kb_per_split;
  bool pair;  // 2-SM pair tiles (256 x bn)
};

// Tile-kind selection (mode & 3): 0 = cost model, 1 = single-CTA tiles only, 2 = pair tiles
// where possible; mode & 4: single-chunk (2-D copy) stages only.
static std::atomic<int> g_gemm_mode{0};
void gemm_set_mode(int mode) { g_gemm_mode.store(mode); }

// Clocks of one 64-deep K step of a CTA holding a 128-row tile of width w: the larger of its
// operand fill (rows of A and B x 128 B at about 64 B per clock into shared memory) and its MMA
// time (about 7,700 dense FLOP per clock per SM).
static double kstep_clocks(int a_rows, int b_rows, int w) {
  const double fill = (double)(a_rows + b_rows) * 128.0 / 64.0;
  const double mma = 2.0 * 128.0 * w * 64.0 / 7700.0;
  return fill > mma ? fill : mma;
}

// Tile width and K splits of a shape, minimising an estimate of the launch's time: waves of
// work units over the SMs x K-blocks per unit x (BN + 64) (a tile streams 128 + BN rows of A and B
// per K step and does BN columns of MMA: operand fill bounds it), plus, when split, the fp32
// partials each tile writes and its last unit reads back (4 x BN "rows" per split). Splits keep
// at least 32 K-blocks each and run only while the tiles fit in well under two waves; a
// candidate replaces the current choice only if it is 2 % cheaper (ties go to the wider tile and
// the fewer splits). Long-K products with few output tiles (the down projection, the data
// gradients of gate/up and of the LM head at ~1 k tokens) thereby take wider tiles, split in two,
// instead of narrow unsplit ones: less operand traffic per FLOP.
static GemmPlan plan_gemm_uncached(int M, int N, int K, int sms, bool b_mn, int mode);

// plan_gemm memoised per host thread: the same few shapes come back every layer of every step.
static GemmPlan plan_gemm(int M, int N, int K, int sms, bool b_mn = false) {
  struct Key {
    int M, N, K, sms, b_mn, mode;
    bool operator==(const Key& o) const {
      return M == o.M && N == o.N && K == o.K && sms == o.sms && b_mn == o.b_mn && mode == o.mode;
    }
  };
  struct Hash {
    size_t operator()(const Key& k) const {
      uint64_t h = 0x9E3779B97F4A7C15ull;
      for (uint64_t x : {(uint64_t)k.M, (uint64_t)k.N, (uint64_t)k.K,
                         (uint64_t)(k.sms * 64 + k.b_mn * 8 + k.mode)})
        h = (h ^ x) * 0x100000001B3ull;
      return (size_t)h;
    }
  };
  thread_local std::unordered_map<Key, GemmPlan, Hash> cache;
  const Key key{M, N, K, sms, (int)b_mn, g_gemm_mode.load() & 3};
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  if (cache.size() > 1024) cache.clear();
  const GemmPlan g = plan_gemm_uncached(M, N, K, sms, b_mn, key.mode);
  cache.emplace(key, g);
  return g;
}

static GemmPlan plan_gemm_uncached(int M, int N, int K, int sms, bool b_mn, int mode) {
  static const int widths[] = {256, 224, 192, 128, 96};
  GemmPlan g{256, 0, 1, 0, false};
  const int k_blocks = (int)cdiv(K, 64);
  g.kb_per_split = k_blocks;
  // 2-SM pair tiles: forced by mode 2; by default only for K-major wide products (N >= 16384,
  // K <= 4096: the gate/up and lm_head forwards), the shapes where they measured faster than the
  // single-CTA tiles at 1-4K rows. Elsewhere the 256-row pairs waste rows of M and were slower.
  // Narrow long-K data gradients at ~1 k tokens or more (gate/up's and the head's vocabulary
  // chunks', an MN-major B): 256-row pair tiles cut the operand bytes each CTA streams by a fifth
  // against the single-CTA tiles, and a K split fills the SMs (gate/up 52.8 -> 50.8 µs in the
  // step). The K-major down projection measured no better this way (35.6 -> 36.6 µs).
  if (mode == 0 && b_mn && N <= 2048 && K >= 4096 && M >= 512) {
    const int64_t ptiles = cdiv(M, 256) * cdiv(N, 256);
    const int s = (int)((sms / 2) / ptiles);
    if (s >= 2 && k_blocks / s >= 32 && 2 * ptiles * 4 <= kCounterBytes) {
      g.pair = true;
      g.bn = 256;
      g.tiles = 2 * ptiles;  // 128-row sub-tiles: one split-K partial and counter each
      g.splits = s;
      g.kb_per_split = (int)cdiv(k_blocks, s);
      g.splits = (int)cdiv(k_blocks, g.kb_per_split);
      return g;
    }
  }
  if (mode == 2 || (mode == 0 && !b_mn && N >= 16384 && K <= 4096 && M >= 512)) {
    int pbn = 0;
    int64_t punits = 0;
    double pbest = 0.0;
    for (int bn : {256, 192, 128}) {
      if (b_mn && (bn / 2) % 64 != 0) continue;  // each CTA's half of an MN-major B: whole boxes
      const int64_t units = cdiv(M, 256) * cdiv(N, bn);
      const double cost = (double)cdiv(units, sms / 2) * kstep_clocks(128, bn / 2, bn);
      if (pbn == 0 || cost < pbest) {
        pbest = cost;
        pbn = bn;
        punits = units;
      }
    }
    g.pair = true;
    g.bn = pbn;
    g.tiles = punits;
    return g;
  }
  double best = -1.0;
  for (int bn : widths) {
    if (b_mn && bn % 64 != 0) continue;  // an MN-major B tile is whole 64-column boxes
    const int64_t tiles = cdiv(M, 128) * cdiv(N, bn);
    for (int s = 1; s <= 8; ++s) {
      if (s > 1 && (tiles >= 2 * (int64_t)sms || tiles * 4 > kCounterBytes || k_blocks / s < 32)) break;
      const int kper = (int)cdiv(k_blocks, s);
      const int splits = (int)cdiv(k_blocks, kper);  // no empty split
      if (s > 1 && splits != s) continue;
      const double waves = (double)cdiv(tiles * splits, sms);
      double cost = waves * kper * (bn + 64);
      if (splits > 1) cost += waves * (splits + 1) * 4.0 * bn;
      if (best < 0.0 || cost < 0.98 * best) {
        best = cost;
        g.bn = bn;
        g.tiles = tiles;
        g.splits = splits;
        g.kb_per_split = kper;
      }
    }
  }
  return g;
}

int64_t gemm_workspace_bytes(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  GemmPlan g = plan_gemm(M, N, K, num_sms());
  const GemmPlan g2 = plan_gemm(M, N, K, num_sms(), true);  // the larger of the two layouts
  if (g2.splits > 1 && g2.tiles * g2.splits * g2.bn > g.tiles * g.splits * g.bn) g = g2;
  if (g.splits == 1) return 0;
  return kCounterBytes + g.tiles * g.splits * 128 * g.bn * 4;
}

// C = A . op(B): b_mn = false, B is [N, K] (K contiguous, C = A B^T); b_mn = true, B is [K, N]
// (N contiguous, C = A B), read by the tensor cores as an MN-major operand.
static int gemm_core(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                     const void* bias, int M, int N, int K, int in_dtype, int out_dtype,
                     int accumulate, const float* residual, int* err, cudaStream_t stream,
                     void* workspace, int64_t workspace_bytes, bool b_mn) {
  if (M < 0 || N < 0 || K < 0) return QL_STATUS_BAD_ARG;
  if (M == 0 || N == 0) return QL_STATUS_OK;
  if (in_dtype != QL_F16 && in_dtype != QL_BF16) return QL_STATUS_BAD_ARG;
  if ((accumulate || residual != nullptr) && out_dtype != QL_F32) return QL_STATUS_BAD_ARG;
  // TMA: 16-byte aligned base and row strides
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) % 16 != 0)
    return QL_STATUS_BAD_ARG;
  if ((lda * 2) % 16 != 0 || (ldb * 2) % 16 != 0 || K % 8 != 0) return QL_STATUS_BAD_ARG;
  if (b_mn && N % 8 != 0) return QL_STATUS_BAD_ARG;
  if (K == 0) return QL_STATUS_UNSUPPORTED;
  const bool bf16 = in_dtype == QL_BF16;
  ProfScope prof(PK_GEMM, 2.0 * M * N * K,
                 2.0 * ((double)M * K + (double)N * K) + (double)M * N * (out_dtype == QL_F32 ? 4 : 2),
                 stream);
  GemmPlan g = plan_gemm(M, N, K, num_sms(), b_mn);
  const int64_t need = kCounterBytes + g.tiles * g.splits * 128 * g.bn * 4;
  if (g.splits > 1 && (workspace == nullptr || workspace_bytes < need ||
                       reinterpret_cast<uintptr_t>(workspace) % 256 != 0 ||
                       accumulate /* C is read by the epilogue: keep one writer per tile */)) {
    g.splits = 1;
    g.kb_per_split = (int)cdiv(K, 64);
  }
  // Two 64-wide K chunks per pipeline stage, each operand in one 3-D copy (32 KB boxes stream
  // from L2 faster than 16 KB ones), for single-CTA tiles of up to 128 columns, where the larger
  // stages still leave three of them in flight, and K is a multiple of 128 (an MN-major B's N of
  // 64). Wider tiles would drop to two stages and measured slower (the down projection 34.7 ->
  // 40.2 us, its data gradient 29.6 -> 33.7 us, the 2-SM gate/up tiles 50 -> 52 us); the qkv and
  // o products (tiles of 96-128 columns) gained 20-25 %.
  const int kc = (!g.pair && g.bn <= 128 && K % 128 == 0 && (!b_mn || N % 64 == 0) &&
                  !(g_gemm_mode.load() & 4)) ? 2 : 1;
  const int brows = g.pair ? g.bn / 2 : g.bn;  // B rows (or MN-major columns) per CTA
  CUtensorMap ma, mb;
  int b3d = 0;
  if (kc == 2) {
    if (make_chunked_map(&ma, A, M, K, lda, 128, 2, bf16) != QL_STATUS_OK) return QL_STATUS_CUDA;
    if (b_mn ? make_chunked_map(&mb, B, K, N, ldb, 128, brows / 64, bf16) != QL_STATUS_OK
             : make_chunked_map(&mb, B, N, K, ldb, brows, 2, bf16) != QL_STATUS_OK)
      return QL_STATUS_CUDA;
    // the split-K plan is in 64-wide blocks: the same split points rounded up to whole stages
    const int kper = (int)cdiv(g.kb_per_split, 2);
    g.kb_per_split = kper;
    g.splits = (int)cdiv(cdiv(K, 128), kper);
  } else {
    if (make_kmajor_map(&ma, A, M, K, lda, 128, bf16) != QL_STATUS_OK) return QL_STATUS_CUDA;
    if (b_mn && N % 64 == 0 && !(g_gemm_mode.load() & 4)) {
      // the stage's 64-column boxes of an MN-major B in one 3-D copy (8 KB boxes are the
      // slowest to stream)
      if (make_chunked_map(&mb, B, K, N, ldb, 64, brows / 64, bf16) != QL_STATUS_OK) return QL_STATUS_CUDA;
      b3d = 1;
    } else if (b_mn) {
      if (make_kmajor_map(&mb, B, K, N, ldb, 64, bf16) != QL_STATUS_OK) return QL_STATUS_CUDA;
    } else {
      if (make_kmajor_map(&mb, B, N, K, ldb, brows, bf16) != QL_STATUS_OK) return QL_STATUS_CUDA;
    }
  }
  GemmArgs a{M, N, K, C, ldc, bias, out_dtype, accumulate, residual, err, g.splits,
             g.kb_per_split, nullptr, nullptr, 0, b3d};
  // 16-bit C with no read-modify epilogue: TMA tensor stores (needs a 16-byte aligned C and row
  // stride); otherwise per-thread row stores and an unused map
  CUtensorMap mc;
  std::memset(&mc, 0, sizeof(mc));
  if (out_dtype != QL_F32 && residual == nullptr && !accumulate &&
      reinterpret_cast<uintptr_t>(C) % 16 == 0 && (ldc * 2) % 16 == 0 &&
      make_store_map(&mc, C, M, N, ldc, out_dtype == QL_BF16) == QL_STATUS_OK)
    a.tma_c = 1;
  if (g.splits > 1) {
    uint8_t* w = static_cast<uint8_t*>(workspace);
    a.counters = reinterpret_cast<int*>(w);
    a.ws = reinterpret_cast<float*>(w + kCounterBytes);
  }
  if (g.pair) {
    if (b_mn) {
      if (g.bn == 128) return dispatch_pair<128, true>(ma, mb, mc, a, bf16, kc, stream);
      return dispatch_pair<256, true>(ma, mb, mc, a, bf16, kc, stream);
    }
    switch (g.bn) {
      case 128: return dispatch_pair<128, false>(ma, mb, mc, a, bf16, kc, stream);
      case 192: return dispatch_pair<192, false>(ma, mb, mc, a, bf16, kc, stream);
      default: return dispatch_pair<256, false>(ma, mb, mc, a, bf16, kc, stream);
    }
  }
  if (b_mn) {
    switch (g.bn) {
      case 128: return dispatch_in<128, true>(ma, mb, mc, a, bf16, kc, stream);
      case 192: return dispatch_in<192, true>(ma, mb, mc, a, bf16, kc, stream);
      default: return dispatch_in<256, true>(ma, mb, mc, a, bf16, kc, stream);
    }
  }
  switch (g.bn) {
    case 96: return dispatch_in<96, false>(ma, mb, mc, a, bf16, kc, stream);
    case 128: return dispatch_in<128, false>(ma, mb, mc, a, bf16, kc, stream);
    case 192: return dispatch_in<192, false>(ma, mb, mc, a, bf16, kc, stream);
    case 224: return dispatch_in<224, false>(ma, mb, mc, a, bf16, kc, stream);
    default: return dispatch_in<256, false>(ma, mb, mc, a, bf16, kc, stream);
  }
}

int gemm_tn(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
            const void* bias, int M, int N, int K, int in_dtype, int out_dtype, int accumulate,
            const float* residual, int* err, cudaStream_t stream, void* workspace,
            int64_t workspace_bytes) {
  return gemm_core(A, lda, B, ldb, C, ldc, bias, M, N, K, in_dtype, out_dtype, accumulate,
                   residual, err, stream, workspace, workspace_bytes, false);
}

int gemm_nn(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
            const void* bias, int M, int N, int K, int in_dtype, int out_dtype, int accumulate,
            const float* residual, int* err, cudaStream_t stream, void* workspace,
            int64_t workspace_bytes) {
  return gemm_core(A, lda, B, ldb, C, ldc, bias, M, N, K, in_dtype, out_dtype, accumulate,
                   residual, err, stream, workspace, workspace_bytes, true);
}

}  // namespace ql
