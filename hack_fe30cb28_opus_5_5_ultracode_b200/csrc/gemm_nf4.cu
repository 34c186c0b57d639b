// GEMM with the NF4 weight dequantised inside the kernel, for sm_100a:
//
//   layout 0:  C[M, N] (+)= A[M, K] . W[N, K]^T (+ bias)   (the projections of the forward)
//   layout 1:  C[M, N] (+)= A[M, K] . W[K, N]              (their data gradients, dX = dY . W)
//
// W is a bitsandbytes-layout NF4 weight [rows, cols] (element i in byte i/2, high nibble first,
// one absmax per 64 consecutive elements of a row, fp32 or double-quantised): the 16-bit weight
// is never written to HBM. This replaces the reference's dequant-then-GEMM pairs
// (solution/engine.py:103-109 + 1081-1093, 1111-1112, 1132-1139, 1163-1165, 1178-1179 and the
// backward's 1239, 1293, 1301, 1316).
//
// Structure (one CTA per SM, persistent, warp-specialised, 448 threads):
//   warp 0      TMA: the 128 x 64 tile of A (128-byte swizzle) and the tile's packed NF4 bytes
//               (BN x 32 B, or 64 x BN/2 B for layout 1) into a ring slot; mbarrier full[s];
//   warps 6-13  dequantise: each thread takes halves of 64-element NF4 blocks (one block = one
//               128-byte operand row: a K-row of W^T for layout 0, a K-row of W for layout 1),
//               value = level[nibble] * scale in fp32, rounded once to the 16-bit type (the
//               reference's nf4_dequant_kernel, solution/kernels.py:68-105), written in the
//               128-byte-swizzled layout the tensor cores read; then ready[s];
//   warp 1      tcgen05.mma (B K-major for layout 0, MN-major for layout 1) into two TMEM
//               accumulators; commit frees the slot (empty[s]) and signals the epilogue;
//   warps 2-5   epilogue: TMEM -> registers -> C (TMA tensor stores for a 16-bit C).
// Operand bytes per 64-deep K step fall from 16 KB + BN x 128 B to 16 KB + BN x 32 B.
#include "common.cuh"
#include "gemm_common.cuh"
#include "ops.h"
#include "profile.h"

namespace ql {

struct Nf4Src {
  const void* absmax;     // fp32 [blocks] or uint8 [blocks] (nested)
  const float* code2;     // nested: [256]
  const float* absmax2;   // nested: [ceil(blocks / bs2)]
  const float* offsets;   // nested: per member of a group
  const float* code;      // [16] levels
  int64_t seg1, seg2;     // first block of the 2nd / 3rd member (nested offsets)
  int64_t rows, cols;     // W [rows, cols]
  int nested, bs2;
};

template <int BN>
struct Nf4Cfg {
  static constexpr int BM = 128, BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;  // the dequantised tile
  static constexpr int P_BYTES = BN * BK / 2;  // its packed NF4 bytes
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + P_BYTES;
  static constexpr int STAGES_FIT = (225 * 1024 - 1280 - EPI_BYTES - 2048) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int TMEM_COLS = 2 * BN <= 256 ? 256 : 512;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 1024 + 512;
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "UMMA N and 32-column epilogue");
  static_assert(B_BYTES % 1024 == 0 && P_BYTES % 1024 == 0, "1 KB aligned stage regions");
};

__device__ __forceinline__ float nf4_block_scale(const Nf4Src& w, int64_t blk) {
  if (w.nested) {
    const uint8_t q = reinterpret_cast<const uint8_t*>(w.absmax)[blk];
    const float s = __fmul_rn(__ldg(w.code2 + q), __ldg(w.absmax2 + blk / w.bs2));
    const int seg = (blk >= w.seg1) + (blk >= w.seg2);
    return __fadd_rn(s, __ldg(w.offsets + seg));
  }
  return __ldg(reinterpret_cast<const float*>(w.absmax) + blk);
}

template <int BN, bool IS_BF16, typename OutT, bool B_MN>
__global__ void __launch_bounds__(448, 1)
    gemm_nf4_kernel(const __grid_constant__ CUtensorMap tma_a,
                    const __grid_constant__ CUtensorMap tma_p,
                    const __grid_constant__ CUtensorMap tma_c, GemmArgs p, Nf4Src w) {
  pdl_enter();
  using Cfg = Nf4Cfg<BN>;
  using InT = typename std::conditional<IS_BF16, __nv_bfloat16, __half>::type;
  constexpr bool kTmaC = sizeof(OutT) == 2;
  constexpr int HPT = (2 * BN + 255) / 256;  // half-blocks per dequant thread and K step
  constexpr int DQ_AHEAD = 4;                 // K steps of scales loaded ahead
  extern __shared__ uint8_t smem_raw[];
  // the 16 levels, one copy per lane (entry e of lane l in bank l): conflict-free lookups
  __shared__ float lut[16][32];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_stage = smem + Cfg::STAGES * Cfg::STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + EPI_BYTES);
  uint64_t* ready = full + Cfg::STAGES;
  uint64_t* empty = ready + Cfg::STAGES;
  uint64_t* tfull = empty + Cfg::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (int)cdiv(p.M, Cfg::BM), n_tiles = (int)cdiv(p.N, BN);
  const int num_tiles = m_tiles * n_tiles;
  const int k_blocks = (int)cdiv(p.K, Cfg::BK);

  for (int i = threadIdx.x; i < 16 * 32; i += blockDim.x) lut[i >> 5][i & 31] = __ldg(w.code + (i >> 5));
  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], 8);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    fence_barrier_init();
    prefetch_tmap(&tma_a);
    prefetch_tmap(&tma_p);
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
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
        const int mb = tile % m_tiles, nb = tile / m_tiles;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) { ok = false; break; }
          uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sp = sa + Cfg::A_BYTES + Cfg::B_BYTES;
          mbar_arrive_expect_tx(&full[stage], Cfg::A_BYTES + Cfg::P_BYTES);
          tma_load_2d(sa, &tma_a, &full[stage], kb * Cfg::BK, mb * Cfg::BM);
          if constexpr (B_MN)  // W rows kb*64.., bytes of columns nb*BN..
            tma_load_2d(sp, &tma_p, &full[stage], nb * (BN / 2), kb * Cfg::BK);
          else  // W rows nb*BN.., bytes of columns kb*64..
            tma_load_2d(sp, &tma_p, &full[stage], kb * (Cfg::BK / 2), nb * BN);
          if (++stage == Cfg::STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp >= 6) {
    // dequantisation warps 6-13: thread dt owns half-blocks (32 elements) h = dt + 256 q of each
    // K step's tile (block h / 2, half h % 2). The blocks' scales are loaded DQ_AHEAD K steps
    // ahead into a small register ring, so their latency hides behind the decoding.
    const int dt = threadIdx.x - 192;
    const int64_t wbpr = w.cols / 64;  // NF4 blocks per W row
    auto scale_of = [&](int nb, int kb, int h) -> float {
      const int i = h >> 1;
      int64_t wrow, wcb;
      if constexpr (B_MN) {
        wrow = (int64_t)kb * Cfg::BK + (i & 63);
        wcb = (int64_t)nb * (BN / 64) + (i >> 6);
      } else {
        wrow = (int64_t)nb * BN + i;
        wcb = kb;
      }
      return (i < BN && kb < k_blocks && wrow < w.rows && wcb < wbpr)
                 ? nf4_block_scale(w, wrow * wbpr + wcb) : 0.f;
    };
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      const int nb = tile / m_tiles;
      float ring[DQ_AHEAD][HPT];
#pragma unroll
      for (int d = 0; d < DQ_AHEAD; ++d)
#pragma unroll
        for (int q = 0; q < HPT; ++q) ring[d][q] = scale_of(nb, d, dt + 256 * q);
      for (int kb0 = 0; kb0 < k_blocks && ok; kb0 += DQ_AHEAD) {
#pragma unroll
        for (int d = 0; d < DQ_AHEAD; ++d) {
          const int kb = kb0 + d;
          if (kb >= k_blocks) break;
          float sc[HPT];
#pragma unroll
          for (int q = 0; q < HPT; ++q) {
            sc[q] = ring[d][q];
            ring[d][q] = scale_of(nb, kb + DQ_AHEAD, dt + 256 * q);
          }
          if (!mbar_wait(&full[stage], phase, p.err)) { ok = false; break; }
          uint8_t* bt = smem + stage * Cfg::STAGE_BYTES + Cfg::A_BYTES;
          const uint8_t* pk = bt + Cfg::B_BYTES;
#pragma unroll
          for (int q = 0; q < HPT; ++q) {
            const int h = dt + 256 * q, i = h >> 1, half = h & 1;
            if (i < BN) {
              const uint8_t* src;
              uint8_t* dst;
              int swz;
              if constexpr (B_MN) {
                const int r = i & 63, j = i >> 6;
                src = pk + r * (BN / 2) + j * 32;
                dst = bt + j * 8192 + r * 128;
                swz = r & 7;
              } else {
                src = pk + i * 32;
                dst = bt + i * 128;
                swz = i & 7;
              }
              const uint4 wv = *reinterpret_cast<const uint4*>(src + 16 * half);
              const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
              const float s = sc[q];
#pragma unroll
              for (int c = 0; c < 4; ++c) {  // 16-byte output chunk 4 half + c: 8 elements
                uint32_t o[4];
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                  const uint32_t byte = (words[c] >> (8 * b)) & 0xFFu;
                  o[b] = pack_t2<InT>(__fmul_rn(lut[byte >> 4][lane], s),
                                      __fmul_rn(lut[byte & 15u][lane], s));
                }
                *reinterpret_cast<uint4*>(dst + (((4 * half + c) ^ swz) << 4)) =
                    make_uint4(o[0], o[1], o[2], o[3]);
              }
            }
          }
          fence_proxy_async_smem();  // the tensor cores read these rows through the async proxy
          __syncwarp();
          if (lane == 0) mbar_arrive(&ready[stage]);
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
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, p.err)) break;
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err) || !mbar_wait(&ready[stage], phase, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < Cfg::BK / 16; ++k) {
            const uint64_t db = B_MN ? umma_desc_mn_sw128(sb + k * 2048, 8192, 1024)
                                     : umma_desc_k_sw128(sb + k * 32);
            umma_f16(tmem_d, umma_desc_k_sw128(sa + k * 32), db, idesc, (kb != 0 || k != 0) ? 1u : 0u);
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
    int local = 0, ebuf = 0;
    OutT* C = reinterpret_cast<OutT*>(p.C);
    const InT* bias = reinterpret_cast<const InT*>(p.bias);
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase, p.err)) break;
      tc_fence_after();
      const int mb = tile % m_tiles, nb = tile / m_tiles;
      const int row = mb * Cfg::BM + row_in_tile;
      const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        float v[32];
        tmem_ld32(taddr + c, v);
        const int col0 = nb * BN + c;
        if constexpr (kTmaC) {
          if (p.tma_c) {
            const int wrow0 = mb * Cfg::BM + quad * 32;
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
      mbar_arrive(&tempty[acc]);
    }
    if (kTmaC && p.tma_c && lane == 0) bulk_wait<0>();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
// The packed NF4 bytes as a 2-D uint8 tensor [rows, cols / 2], boxes of box_x bytes x box_y rows.
static int make_packed_map(CUtensorMap* map, const uint8_t* packed, int64_t rows, int64_t cols,
                           int box_x, int box_y) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return QL_STATUS_CUDA;
  cuuint64_t dims[2] = {(cuuint64_t)(cols / 2), (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(cols / 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_x, (cuuint32_t)box_y};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(packed), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QL_STATUS_OK : QL_STATUS_CUDA;
}

template <int BN, bool IS_BF16, typename OutT, bool B_MN>
static int launch_nf4(const CUtensorMap& ma, const CUtensorMap& mp, const CUtensorMap& mc,
                      const GemmArgs& a, const Nf4Src& w, cudaStream_t stream) {
  using Cfg = Nf4Cfg<BN>;
  auto kern = gemm_nf4_kernel<BN, IS_BF16, OutT, B_MN>;
  static bool configured = false;  // one static per instantiation
  if (!configured) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES) !=
        cudaSuccess)
      return QL_STATUS_CUDA;
    configured = true;
  }
  const int tiles = (int)(cdiv(a.M, 128) * cdiv(a.N, BN));
  const int grid = tiles < num_sms() ? tiles : num_sms();
  kern<<<grid, 448, Cfg::SMEM_BYTES, stream>>>(ma, mp, mc, a, w);
  return launched(1);
}

template <int BN, bool IS_BF16, bool B_MN>
static int nf4_out(const CUtensorMap& ma, const CUtensorMap& mp, const CUtensorMap& mc,
                   const GemmArgs& a, const Nf4Src& w, cudaStream_t s) {
  switch (a.out_dtype) {
    case QL_F16: return launch_nf4<BN, IS_BF16, __half, B_MN>(ma, mp, mc, a, w, s);
    case QL_BF16: return launch_nf4<BN, IS_BF16, __nv_bfloat16, B_MN>(ma, mp, mc, a, w, s);
    case QL_F32: return launch_nf4<BN, IS_BF16, float, B_MN>(ma, mp, mc, a, w, s);
  }
  return QL_STATUS_BAD_ARG;
}

template <int BN, bool B_MN>
static int nf4_in(const CUtensorMap& ma, const CUtensorMap& mp, const CUtensorMap& mc,
                  const GemmArgs& a, const Nf4Src& w, bool bf16, cudaStream_t s) {
  return bf16 ? nf4_out<BN, true, B_MN>(ma, mp, mc, a, w, s) : nf4_out<BN, false, B_MN>(ma, mp, mc, a, w, s);
}

// Tile width: the fewest waves of output tiles, each wave costed as BN + 64 (as the dense GEMM).
static int nf4_width(int M, int N, bool b_mn) {
  int best_bn = 128;
  int64_t best = -1;
  for (int bn : {256, 128, 96}) {
    if (b_mn && bn % 64 != 0) continue;  // MN-major tiles are whole 64-column boxes
    const int64_t cost = cdiv(cdiv(M, 128) * cdiv(N, bn), num_sms()) * (bn + 64);
    if (best < 0 || cost < best) {
      best = cost;
      best_bn = bn;
    }
  }
  return best_bn;
}

int gemm_nf4(const void* A, int64_t lda, const ql_nf4_weight& W, int layout, void* C, int64_t ldc,
             const void* bias, int M, int in_dtype, int out_dtype, int accumulate,
             const float* residual, int* err, cudaStream_t stream) {
  if (layout != 0 && layout != 1) return QL_STATUS_BAD_ARG;
  const bool b_mn = layout == 1;
  const int64_t N64 = b_mn ? W.cols : W.rows, K64 = b_mn ? W.rows : W.cols;
  if (M < 0 || W.rows <= 0 || W.cols <= 0 || N64 > INT32_MAX || K64 > INT32_MAX) return QL_STATUS_BAD_ARG;
  const int N = (int)N64, K = (int)K64;
  if (M == 0) return QL_STATUS_OK;
  if (in_dtype != QL_F16 && in_dtype != QL_BF16) return QL_STATUS_BAD_ARG;
  if ((accumulate || residual != nullptr) && out_dtype != QL_F32) return QL_STATUS_BAD_ARG;
  if (W.cols % 64 != 0 || W.packed == nullptr || W.absmax == nullptr || W.code == nullptr)
    return QL_STATUS_BAD_ARG;
  if (W.nested && (W.bs2 <= 0 || W.code2 == nullptr || W.absmax2 == nullptr || W.offsets == nullptr))
    return QL_STATUS_BAD_ARG;
  if (reinterpret_cast<uintptr_t>(A) % 16 != 0 || reinterpret_cast<uintptr_t>(W.packed) % 16 != 0 ||
      (lda * 2) % 16 != 0 || K % 8 != 0)
    return QL_STATUS_BAD_ARG;
  if (b_mn && N % 64 != 0) return QL_STATUS_BAD_ARG;
  const bool bf16 = in_dtype == QL_BF16;
  ProfScope prof(PK_GEMM, 2.0 * M * N * K,
                 2.0 * M * K + 0.5625 * (double)N * K + (double)M * N * (out_dtype == QL_F32 ? 4 : 2),
                 stream);
  const int bn = nf4_width(M, N, b_mn);
  CUtensorMap ma, mp, mc;
  std::memset(&mc, 0, sizeof(mc));
  if (make_kmajor_map(&ma, A, M, K, lda, 128, bf16) != QL_STATUS_OK) return QL_STATUS_CUDA;
  if (b_mn) {
    if (make_packed_map(&mp, W.packed, W.rows, W.cols, bn / 2, 64) != QL_STATUS_OK) return QL_STATUS_CUDA;
  } else {
    if (make_packed_map(&mp, W.packed, W.rows, W.cols, 32, bn) != QL_STATUS_OK) return QL_STATUS_CUDA;
  }
  GemmArgs a{M, N, K, C, ldc, bias, out_dtype, accumulate, residual, err, 1, (int)cdiv(K, 64),
             nullptr, nullptr, 0};
  if (out_dtype != QL_F32 && residual == nullptr && !accumulate &&
      reinterpret_cast<uintptr_t>(C) % 16 == 0 && (ldc * 2) % 16 == 0 &&
      make_store_map(&mc, C, M, N, ldc, out_dtype == QL_BF16) == QL_STATUS_OK)
    a.tma_c = 1;
  const Nf4Src w{W.absmax, W.code2, W.absmax2, W.offsets, W.code, W.seg1, W.seg2, W.rows, W.cols,
                 W.nested, W.bs2 > 0 ? W.bs2 : 1};
  if (b_mn) {
    if (bn == 128) return nf4_in<128, true>(ma, mp, mc, a, w, bf16, stream);
    return nf4_in<256, true>(ma, mp, mc, a, w, bf16, stream);
  }
  switch (bn) {
    case 96: return nf4_in<96, false>(ma, mp, mc, a, w, bf16, stream);
    case 128: return nf4_in<128, false>(ma, mp, mc, a, w, bf16, stream);
    default: return nf4_in<256, false>(ma, mp, mc, a, w, bf16, stream);
  }
}

}  // namespace ql
