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
//   warp 0      TMA producer: 128 x 64 tiles of A and BN x 64 tiles of B into a ring of STAGES
//               shared-memory slots (128-byte swizzle), completion counted on an mbarrier;
//   warp 1      allocates 2 x BN TMEM columns (two accumulators) and issues tcgen05.mma from one
//               thread, 4 x (K = 16) per 64-wide K step; tcgen05.commit frees each slot and, at
//               the end of a tile, signals the epilogue;
//   warps 2-5   epilogue: tcgen05.ld of their 32 TMEM lanes, bias add, conversion, stores.
// The accumulator of tile t+1 is written while the epilogue drains tile t.
#include "common.cuh"
#include "profile.h"

namespace ql {

struct GemmArgs {
  int M, N, K;
  void* C;
  int64_t ldc;
  const void* bias;  // [N] of the input type, or null
  int out_dtype;     // QL_F16 / QL_BF16 / QL_F32
  int accumulate;    // C += result (fp32 output only)
  const float* residual;  // fp32 [M, ldc] or null: C = residual + (result rounded to the input type)
  int* err;
};

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128, BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int TMEM_COLS = 2 * BN;  // 256 or 512: a power of two >= 32
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

template <typename OutT>
__device__ __forceinline__ void store_row32(OutT* dst, const float* v, int ncols) {
  if (ncols >= 32 && (reinterpret_cast<uintptr_t>(dst) % 16) == 0) {
    if constexpr (sizeof(OutT) == 2) {
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        OutT lo = from_f<OutT>(v[2 * i]), hi = from_f<OutT>(v[2 * i + 1]);
        w[i] = (uint32_t)(*reinterpret_cast<uint16_t*>(&lo)) |
               ((uint32_t)(*reinterpret_cast<uint16_t*>(&hi)) << 16);
      }
      uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int i = 0; i < 4; ++i) d[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    } else {
      float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
      for (int i = 0; i < 8; ++i) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < ncols) dst[i] = from_f<OutT>(v[i]);
  }
}

template <int BN, bool IS_BF16, typename OutT>
__global__ void __launch_bounds__(192, 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                   GemmArgs p) {
  using Cfg = GemmCfg<BN>;
  using InT = typename std::conditional<IS_BF16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + Cfg::STAGES;
  uint64_t* tfull = empty + Cfg::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (int)cdiv(p.M, Cfg::BM), n_tiles = (int)cdiv(p.N, BN);
  const int num_tiles = m_tiles * n_tiles;
  const int k_blocks = (int)cdiv(p.K, Cfg::BK);

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
          uint8_t* sb = sa + Cfg::A_BYTES;
          mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          tma_load_2d(sa, &tma_a, &full[stage], kb * Cfg::BK, mb * Cfg::BM);
          tma_load_2d(sb, &tma_b, &full[stage], kb * Cfg::BK, nb * BN);
          if (++stage == Cfg::STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(IS_BF16, 128, BN);
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
          if (!mbar_wait(&full[stage], phase, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < Cfg::BK / 16; ++k) {
            umma_f16(tmem_d, umma_desc_k_sw128(sa + k * 32), umma_desc_k_sw128(sb + k * 32), idesc,
                     (kb | k) != 0 ? 1u : 0u);
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
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// A row-major [rows, cols] 16-bit matrix with row stride ld (elements), boxes of box_rows x 64.
static int make_kmajor_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols,
                           int64_t ld, int box_rows, bool bf16) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return QL_STATUS_CUDA;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QL_STATUS_OK : QL_STATUS_CUDA;
}

static int num_sms() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

template <int BN, bool IS_BF16, typename OutT>
static int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& a,
                       cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  auto kern = gemm_tn_kernel<BN, IS_BF16, OutT>;
  static bool configured = false;  // one static per instantiation
  if (!configured) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES) !=
        cudaSuccess)
      return QL_STATUS_CUDA;
    configured = true;
  }
  const int tiles = (int)(cdiv(a.M, 128) * cdiv(a.N, BN));
  const int grid = tiles < num_sms() ? tiles : num_sms();
  kern<<<grid, 192, Cfg::SMEM_BYTES, stream>>>(ma, mb, a);
  return launched(1);
}

template <int BN, bool IS_BF16>
static int dispatch_out(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& a,
                        cudaStream_t s) {
  switch (a.out_dtype) {
    case QL_F16: return launch_gemm<BN, IS_BF16, __half>(ma, mb, a, s);
    case QL_BF16: return launch_gemm<BN, IS_BF16, __nv_bfloat16>(ma, mb, a, s);
    case QL_F32: return launch_gemm<BN, IS_BF16, float>(ma, mb, a, s);
  }
  return QL_STATUS_BAD_ARG;
}

int gemm_tn(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
            const void* bias, int M, int N, int K, int in_dtype, int out_dtype, int accumulate,
            const float* residual, int* err, cudaStream_t stream) {
  if (M < 0 || N < 0 || K < 0) return QL_STATUS_BAD_ARG;
  if (M == 0 || N == 0) return QL_STATUS_OK;
  if (in_dtype != QL_F16 && in_dtype != QL_BF16) return QL_STATUS_BAD_ARG;
  if ((accumulate || residual != nullptr) && out_dtype != QL_F32) return QL_STATUS_BAD_ARG;
  // TMA: 16-byte aligned base and row strides
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) % 16 != 0)
    return QL_STATUS_BAD_ARG;
  if ((lda * 2) % 16 != 0 || (ldb * 2) % 16 != 0 || K % 8 != 0) return QL_STATUS_BAD_ARG;
  if (K == 0) return QL_STATUS_UNSUPPORTED;
  const bool bf16 = in_dtype == QL_BF16;
  ProfScope prof(PK_GEMM, 2.0 * M * N * K,
                 2.0 * ((double)M * K + (double)N * K) + (double)M * N * (out_dtype == QL_F32 ? 4 : 2),
                 stream);
  // Wide N tiles when there are enough of them to fill the machine, else 128.
  const int64_t tiles256 = cdiv(M, 128) * cdiv(N, 256);
  const int BN = (tiles256 >= num_sms()) ? 256 : 128;
  CUtensorMap ma, mb;
  if (make_kmajor_map(&ma, A, M, K, lda, 128, bf16) != QL_STATUS_OK) return QL_STATUS_CUDA;
  if (make_kmajor_map(&mb, B, N, K, ldb, BN, bf16) != QL_STATUS_OK) return QL_STATUS_CUDA;
  GemmArgs a{M, N, K, C, ldc, bias, out_dtype, accumulate, residual, err};
  if (BN == 256)
    return bf16 ? dispatch_out<256, true>(ma, mb, a, stream) : dispatch_out<256, false>(ma, mb, a, stream);
  return bf16 ? dispatch_out<128, true>(ma, mb, a, stream) : dispatch_out<128, false>(ma, mb, a, stream);
}

}  // namespace ql
