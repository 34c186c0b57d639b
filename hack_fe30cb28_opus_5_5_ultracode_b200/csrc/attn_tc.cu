// Varlen causal GQA attention forward on the 5th-generation tensor cores (head dim 128).
//
// Same contract as the warp-level kernel in attn.cu (replaces _attn_fwd, solution/engine.py:
// 857-869): q [n, HQ, 128], k / v [n, HKV, 128], cu_seqlens [B + 1], causal within a sequence;
// writes out [n, HQ, 128] and the natural-log logsumexp [HQ, n].
//
// One CTA per (128-query tile, query head, sequence), the tiles with the most key blocks first.
// Six warps with fixed roles:
//   warp 0     TMA: the Q tile once, then K and V tiles of 128 keys into a two-stage ring;
//   warp 1     one thread issues tcgen05.mma: S_j = Q K_j^T into one of two TMEM score buffers,
//              then O += P_{j-1} V_{j-1} into the TMEM output accumulator (S_j runs while the
//              softmax warps work on S_{j-1});
//   warps 2-5  softmax, one query row per thread (TMEM lane = row): the row's 128 scores come
//              from TMEM with no cross-thread reduction, P is written as 16-bit values into a
//              swizzled shared-memory tile (the A operand of the next MMA; two buffers), and
//              the running row max is raised lazily: O (in TMEM) is rescaled only when a row's
//              max grows by more than 2^8, after the MMA that last added to O has completed.
// TMEM columns: O [0, 128), score buffers [128, 256) and [256, 384) (512 allocated).
// Shared memory: Q 32 KB, two (K, V) stages of 64 KB, two P tiles of 32 KB (224 KB).
// Every wait is bounded (QL_STATUS_TIMEOUT in the library's status word on expiry).
#include "common.cuh"
#include "gemm_common.cuh"
#include "ops.h"
#include "profile.h"

namespace ql {

namespace {

constexpr int TA_BM = 128;               // queries per CTA
constexpr int TA_BN = 128;               // keys per block
constexpr int TA_D = 128;                // head dim
constexpr int TA_TILE = 128 * TA_D * 2;  // a 128 x 128 16-bit tile: two 64-column boxes
constexpr int TA_BOX = TA_TILE / 2;      // one 128-row x 64-column box (128-byte rows)
constexpr int TA_SMEM = 7 * TA_TILE + 1024 /*align*/ + 256 /*barriers*/;
constexpr uint32_t TA_TMEM_COLS = 512;

// offset of the 16-byte chunk ch (0-15) of row r in a K-major 128-byte-swizzled two-box tile
__device__ __forceinline__ uint32_t ta_chunk(int r, int ch) {
  return (uint32_t)((ch >> 3) * TA_BOX + r * 128 + (((ch & 7) ^ (r & 7)) << 4));
}

template <bool IS_BF16>
__global__ void __launch_bounds__(192, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                       const __grid_constant__ CUtensorMap tv, AttnFwdC a, int* err) {
  pdl_enter();
  using T = typename std::conditional<IS_BF16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                   // [128 q][128 d]
  uint8_t* sKV = smem + TA_TILE;        // stage s: K at + 2s tiles, V at + (2s + 1) tiles
  uint8_t* sP = smem + 5 * TA_TILE;     // two [128 q][128 keys] tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 7 * TA_TILE);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;   // [2] K and V of a stage landed
  uint64_t* kv_empty = bars + 3;  // [2] the MMAs reading a stage completed
  uint64_t* s_full = bars + 5;    // [2] score buffer written
  uint64_t* s_free = bars + 7;    // [2] score buffer read by all 128 softmax threads
  uint64_t* p_full = bars + 9;    // [2] P tile written by all 128 softmax threads
  uint64_t* pv_done = bars + 11;  // [2] O += P V of the P tile completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);

  const int qb = gridDim.x - 1 - blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int start = a.cu_seqlens[b], len = a.cu_seqlens[b + 1] - start;
  if (qb * TA_BM >= len) return;  // the whole CTA, before any barrier or TMEM is set up
  const int kvh = h / (a.HQ / a.HKV);
  const int nkb = qb + 1;  // causal: key blocks 0 .. qb
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 128);
      mbar_init(&p_full[s], 128);
      mbar_init(&pv_done[s], 1);
    }
    fence_barrier_init();
    prefetch_tmap(&tq);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
  }
  if (warp == 1) tmem_alloc(tmem_slot, TA_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, TA_TILE);
      tma_load_2d(sQ, &tq, q_full, h * TA_D, start + qb * TA_BM);
      tma_load_2d(sQ + TA_BOX, &tq, q_full, h * TA_D + 64, start + qb * TA_BM);
      for (int j = 0; j < nkb; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&kv_empty[s], ((j >> 1) - 1) & 1, err)) break;
        uint8_t* k = sKV + s * 2 * TA_TILE;
        uint8_t* v = k + TA_TILE;
        const int row = start + j * TA_BN;
        mbar_arrive_expect_tx(&kv_full[s], 2 * TA_TILE);
        tma_load_2d(k, &tk, &kv_full[s], kvh * TA_D, row);
        tma_load_2d(k + TA_BOX, &tk, &kv_full[s], kvh * TA_D + 64, row);
        tma_load_2d(v, &tv, &kv_full[s], kvh * TA_D, row);
        tma_load_2d(v + TA_BOX, &tv, &kv_full[s], kvh * TA_D + 64, row);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = umma_idesc_f16(IS_BF16, 128, TA_BN, false);
      constexpr uint32_t id_o = umma_idesc_f16(IS_BF16, 128, TA_D, true);  // V is MN-major
      const uint32_t aq = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, err);
      for (int j = 0; ok && j <= nkb; ++j) {
        if (j < nkb) {  // S_j = Q K_j^T
          const int s = j & 1;
          if (!mbar_wait(&kv_full[s], (j >> 1) & 1, err)) break;
          if (j >= 2 && !mbar_wait(&s_free[s], ((j >> 1) - 1) & 1, err)) break;
          tc_fence_after();
          const uint32_t bk = smem_u32(sKV + s * 2 * TA_TILE);
          const uint32_t ts = tmem + 128 + s * TA_BN;
#pragma unroll
          for (int kk = 0; kk < TA_D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * TA_BOX + (kk & 3) * 32;
            umma_f16(ts, umma_desc_k_sw128(aq + off), umma_desc_k_sw128(bk + off), id_s, kk > 0);
          }
          umma_commit(&s_full[s]);
        }
        if (j >= 1) {  // O += P_i V_i, i = j - 1
          const int i = j - 1, s = i & 1;
          if (!mbar_wait(&p_full[s], (i >> 1) & 1, err)) break;
          tc_fence_after();
          const uint32_t ap = smem_u32(sP + s * TA_TILE);
          const uint32_t bv = smem_u32(sKV + s * 2 * TA_TILE + TA_TILE);
#pragma unroll
          for (int kk = 0; kk < TA_BN / 16; ++kk) {
            umma_f16(tmem, umma_desc_k_sw128(ap + (kk >> 2) * TA_BOX + (kk & 3) * 32),
                     umma_desc_mn_sw128(bv + kk * 2048, TA_BOX, 1024), id_o, (i > 0 || kk > 0));
          }
          umma_commit(&kv_empty[s]);
          umma_commit(&pv_done[s]);
        }
      }
    }
  } else {
    const int quad = warp & 3, r = quad * 32 + lane;  // TMEM lane quadrant = warp % 4
    const int qi = qb * TA_BM + r;                      // query row in the sequence
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const float sl2 = a.scale * 1.4426950408889634f;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      const int s = j & 1;
      if (!mbar_wait(&s_full[s], (j >> 1) & 1, err)) { ok = false; break; }
      tc_fence_after();
      float sv[TA_BN];
      {
        uint32_t su[TA_BN];
#pragma unroll
        for (int c = 0; c < TA_BN / 32; ++c) tmem_ld32_nw(lane_base + 128 + s * TA_BN + c * 32, su + c * 32);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < TA_BN; ++c) sv[c] = __uint_as_float(su[c]);
      }
      tc_fence_before();
      mbar_arrive(&s_free[s]);
      if (j == qb) {  // the diagonal block: keys after the query are masked
#pragma unroll
        for (int c = 0; c < TA_BN; ++c)
          if (j * TA_BN + c > qi) sv[c] = -INFINITY;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < TA_BN; ++c) mx = fmaxf(mx, sv[c]);
      const float ms = mx * sl2;
      float corr = 1.f;
      if (ms > m_run + 8.f) {
        corr = m_run == -INFINITY ? 0.f : exp2f(m_run - ms);
        m_run = ms;
      }
      const float mneg = m_run == -INFINITY ? 0.f : -m_run;
      // this P buffer was last read by O += P_{j-2} V_{j-2}
      if (j >= 2 && !mbar_wait(&pv_done[s], ((j >> 1) - 1) & 1, err)) { ok = false; break; }
      uint8_t* pt = sP + s * TA_TILE;
      float sum = 0.f;
#pragma unroll
      for (int ch = 0; ch < TA_BN / 8; ++ch) {
        float p[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          p[e] = exp2f(fmaf(sv[ch * 8 + e], sl2, mneg));  // exp2(-inf) = 0
          sum += p[e];
        }
        *reinterpret_cast<uint4*>(pt + ta_chunk(r, ch)) =
            make_uint4(pack_t2<T>(p[0], p[1]), pack_t2<T>(p[2], p[3]), pack_t2<T>(p[4], p[5]),
                       pack_t2<T>(p[6], p[7]));
      }
      l_run = l_run * corr + sum;
      if (j > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
        // rescale this warp's O rows once the last MMA adding to O (P_{j-1} V_{j-1}) is done
        if (!mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, err)) { ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < TA_D / 32; ++c) {
          float ov[32];
          tmem_ld32(lane_base + c * 32, ov);
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] *= corr;
          tmem_st32(lane_base + c * 32, ov);
        }
        tmem_wait_st();
      }
      fence_proxy_async_smem();  // P visible to the tensor core
      tc_fence_before();
      mbar_arrive(&p_full[s]);
    }
    if (ok && mbar_wait(&pv_done[(nkb - 1) & 1], ((nkb - 1) >> 1) & 1, err)) {
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      T* out = reinterpret_cast<T*>(a.out) + ((int64_t)(start + qi) * a.HQ + h) * TA_D;
#pragma unroll 1
      for (int c = 0; c < TA_D / 32; ++c) {
        float ov[32];
        tmem_ld32(lane_base + c * 32, ov);
        if (qi < len) {
#pragma unroll
          for (int u = 0; u < 4; ++u)
            reinterpret_cast<uint4*>(out + c * 32)[u] =
                make_uint4(pack_t2<T>(ov[8 * u] * inv, ov[8 * u + 1] * inv),
                           pack_t2<T>(ov[8 * u + 2] * inv, ov[8 * u + 3] * inv),
                           pack_t2<T>(ov[8 * u + 4] * inv, ov[8 * u + 5] * inv),
                           pack_t2<T>(ov[8 * u + 6] * inv, ov[8 * u + 7] * inv));
        }
      }
      if (qi < len) a.lse[(int64_t)h * a.n + start + qi] = (m_run + log2f(l_run)) * 0.6931471805599453f;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TA_TMEM_COLS);
  }
}

}  // namespace

// Host side: tensor maps over q [n, HQ * 128] and k / v [n, HKV * 128] (boxes of 64 columns x
// 128 rows with the 128-byte swizzle; rows past n read as zeros).
int attn_fwd_tc(const AttnFwdC& a, cudaStream_t s) {
  if (a.D != TA_D) return QL_STATUS_UNSUPPORTED;
  const bool bf = a.dtype == QL_BF16;
  CUtensorMap mq, mk, mv;
  const int64_t wq = (int64_t)a.HQ * TA_D, wk = (int64_t)a.HKV * TA_D;
  if (make_kmajor_map(&mq, a.q, a.n, wq, wq, 128, bf) != QL_STATUS_OK ||
      make_kmajor_map(&mk, a.k, a.n, wk, wk, 128, bf) != QL_STATUS_OK ||
      make_kmajor_map(&mv, a.v, a.n, wk, wk, 128, bf) != QL_STATUS_OK)
    return QL_STATUS_CUDA;
  dim3 grid((unsigned)cdiv(a.max_len, TA_BM), (unsigned)a.HQ, (unsigned)a.B);
  int* err = status_word();
  if (bf) {
    smem_optin(reinterpret_cast<const void*>(attn_fwd_tc_kernel<true>), TA_SMEM);
    launch_k(attn_fwd_tc_kernel<true>, grid, dim3(192), TA_SMEM, s, mq, mk, mv, a, err);
  } else {
    smem_optin(reinterpret_cast<const void*>(attn_fwd_tc_kernel<false>), TA_SMEM);
    launch_k(attn_fwd_tc_kernel<false>, grid, dim3(192), TA_SMEM, s, mq, mk, mv, a, err);
  }
  return QL_STATUS_OK;
}

}  // namespace ql
