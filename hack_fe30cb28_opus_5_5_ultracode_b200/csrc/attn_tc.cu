// Varlen causal GQA attention forward on the 5th-generation tensor cores (head dim 128).
//
// Same contract as the warp-level kernel in attn.cu (replaces _attn_fwd, solution/engine.py:
// 857-869): q [n, HQ, 128], k / v [n, HKV, 128], cu_seqlens [B + 1], causal within a sequence;
// writes out [n, HQ, 128] and the natural-log logsumexp [HQ, n].
//
// One CTA per (128-query tile, query head, sequence), the tiles with the most key blocks first.
// Ten warps with fixed roles:
//   warp 0     TMA: the Q tile once, then K and V tiles of 128 keys into a two-stage ring;
//   warp 1     one thread issues tcgen05.mma: S_j = Q K_j^T into one of two TMEM score buffers,
//              then O += P_{j-1} V_{j-1} into the TMEM output accumulator (S_j runs while the
//              softmax warps work on S_{j-1});
//   warps 2-9  softmax, two threads per query row (TMEM lane = row; warps w and w + 4 share a
//              lane quadrant): both read the row's 128 scores from TMEM and take the same row
//              max with no exchange, and each exponentiates its own 64 of them, writing P as
//              16-bit values into a swizzled shared-memory tile (the A operand of the next MMA;
//              two buffers). The running row max is raised lazily: O (in TMEM) is rescaled,
//              each thread its 64 columns, only when a row's max grows by more than 2^8, after
//              the MMA that last added to O has completed. The two partial row sums are added
//              once, at the end, through shared memory.
// TMEM columns: O [0, 128), score buffers [128, 256) and [256, 384) (512 allocated).
// Shared memory: Q 32 KB, two (K, V) stages of 64 KB, two P tiles of 32 KB (224 KB), barriers,
// the row sums' exchange (1 KB).
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
constexpr int TA_SOFTMAX = 256;          // softmax threads: two per query row
constexpr int TA_SMEM = 7 * TA_TILE + 1024 /*align*/ + 256 /*barriers*/ + 2 * TA_BM * 4 /*sums*/;
constexpr uint32_t TA_TMEM_COLS = 512;

// offset of the 16-byte chunk ch (0-15) of row r in a K-major 128-byte-swizzled two-box tile
__device__ __forceinline__ uint32_t ta_chunk(int r, int ch) {
  return (uint32_t)((ch >> 3) * TA_BOX + r * 128 + (((ch & 7) ^ (r & 7)) << 4));
}

template <bool IS_BF16>
__global__ void __launch_bounds__(64 + TA_SOFTMAX, 1)
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
  uint64_t* l_bar = bars + 13;    // both halves' row sums stored
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  float* sL = reinterpret_cast<float*>(smem + 7 * TA_TILE + 256);  // [2 halves][128 rows]

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
      mbar_init(&s_free[s], TA_SOFTMAX);
      mbar_init(&p_full[s], TA_SOFTMAX);
      mbar_init(&pv_done[s], 1);
    }
    mbar_init(l_bar, TA_SOFTMAX);
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
      // each tile in one 3-D copy of both 64-column halves of the head ([2][128 rows][64])
      tma_load_3d(sQ, &tq, q_full, 0, start + qb * TA_BM, h * 2);
      for (int j = 0; j < nkb; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&kv_empty[s], ((j >> 1) - 1) & 1, err)) break;
        uint8_t* k = sKV + s * 2 * TA_TILE;
        uint8_t* v = k + TA_TILE;
        const int row = start + j * TA_BN;
        mbar_arrive_expect_tx(&kv_full[s], 2 * TA_TILE);
        tma_load_3d(k, &tk, &kv_full[s], 0, row, kvh * 2);
        tma_load_3d(v, &tv, &kv_full[s], 0, row, kvh * 2);
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
    const int half = (warp - 2) >> 2;                   // this thread's 64 score / O columns
    const int qi = qb * TA_BM + r;                      // query row in the sequence
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const float sl2 = a.scale * 1.4426950408889634f;
    constexpr int HC = TA_BN / 2;  // columns per thread
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      const int s = j & 1;
      if (!mbar_wait(&s_full[s], (j >> 1) & 1, err)) { ok = false; break; }
      tc_fence_after();
      // the whole row for its max (both threads of the row find the same one), this thread's
      // half for the exponentials
      float sv[HC];
      float mx = -INFINITY;
      {
        uint32_t su[TA_BN];
#pragma unroll
        for (int c = 0; c < TA_BN / 32; ++c) tmem_ld32_nw(lane_base + 128 + s * TA_BN + c * 32, su + c * 32);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < TA_BN; ++c) {
          float x = __uint_as_float(su[c]);
          if (j == qb && j * TA_BN + c > qi) x = -INFINITY;  // the diagonal block: causal mask
          mx = fmaxf(mx, x);
          if ((c >= HC) == (half == 1)) sv[c % HC] = x;
        }
      }
      tc_fence_before();
      mbar_arrive(&s_free[s]);
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
      // off the diagonal every other group of 8 exponentials runs on the FMA pipe (exp2_fma),
      // halving the special-function-unit load; the diagonal block keeps exp2f (exact zeros for
      // the masked keys)
      auto emit = [&](auto mix) {
#pragma unroll
        for (int cc = 0; cc < HC / 8; ++cc) {
          float p[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float x = fmaf(sv[cc * 8 + e], sl2, mneg);
            p[e] = (decltype(mix)::value && (cc & 1)) ? exp2_fma(x) : exp2f(x);  // exp2f(-inf) = 0
            sum += p[e];
          }
          *reinterpret_cast<uint4*>(pt + ta_chunk(r, half * (HC / 8) + cc)) =
              make_uint4(pack_t2<T>(p[0], p[1]), pack_t2<T>(p[2], p[3]), pack_t2<T>(p[4], p[5]),
                         pack_t2<T>(p[6], p[7]));
        }
      };
      if (j == qb) emit(std::false_type{});
      else emit(std::true_type{});
      l_run = l_run * corr + sum;
      if (j > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
        // rescale this thread's O columns once the last MMA adding to O (P_{j-1} V_{j-1}) is done
        if (!mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, err)) { ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < TA_D / 64; ++c) {
          float ov[32];
          const uint32_t col = lane_base + half * (TA_D / 2) + c * 32;
          tmem_ld32(col, ov);
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] *= corr;
          tmem_st32(col, ov);
        }
        tmem_wait_st();
      }
      fence_proxy_async_smem();  // P visible to the tensor core
      tc_fence_before();
      mbar_arrive(&p_full[s]);
    }
    // the row sum: both halves' partial sums, added in a fixed order
    sL[half * TA_BM + r] = l_run;
    mbar_arrive(l_bar);
    if (ok) ok = mbar_wait(l_bar, 0, err);
    if (ok && mbar_wait(&pv_done[(nkb - 1) & 1], ((nkb - 1) >> 1) & 1, err)) {
      tc_fence_after();
      const float l_row = sL[r] + sL[TA_BM + r];
      const float inv = l_row > 0.f ? 1.f / l_row : 0.f;
      T* out = reinterpret_cast<T*>(a.out) + ((int64_t)(start + qi) * a.HQ + h) * TA_D +
               half * (TA_D / 2);
#pragma unroll 1
      for (int c = 0; c < TA_D / 64; ++c) {
        float ov[32];
        tmem_ld32(lane_base + half * (TA_D / 2) + c * 32, ov);
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
      if (qi < len && half == 0)
        a.lse[(int64_t)h * a.n + start + qi] = (m_run + log2f(l_row)) * 0.6931471805599453f;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TA_TMEM_COLS);
  }
}


// ---------------------------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------------------------
// One CTA per (128-key block, query chunk of attn_bwd_qch queries, query head, sequence). The
// key block's K and V stay in shared memory; the chunk's query blocks of 64 stream through a
// two-stage ring (Q, dO, lse * log2(e), Dvec). Per query block j, all on tcgen05 with fp32
// accumulators in TMEM (lane = the M row):
//   S^T  = K Q_j^T          [128 keys x 64 q]   K-major A and B
//   dP^T = V dO_j^T         [128 keys x 64 q]
//   (softmax warps, one key row per thread) P^T = exp2(S^T sl2 - lse2), masked causally;
//   dS^T = P^T (dP^T - Dvec); both to shared memory as 16-bit [key][q] tiles (128-byte swizzle)
//   dV  += P^T dO_j         [128 keys x 128 d]  A K-major, B (dO) MN-major
//   dK  += dS^T Q_j         [128 keys x 128 d]
//   dQ^T = K^T dS^T         [128 d x 64 q]      A (K) MN-major, B (dS^T) MN-major
// dQ^T is read by four more warps (one d row per thread), scaled, staged as [64 q][128 d] fp32
// and added to dq by bulk reductions; at the end dK (scaled) and dV are staged the same way and
// bulk-added to the KV head's fp32 rows (the chunks and the group's query heads all add there).
// Warps: 0 loads (all lanes: lse / Dvec; lane 0: TMA), 1 MMA, 2-5 softmax + final dK / dV,
// 6-9 dQ. TMEM: S^T [0, 64), dP^T [64, 128), dQ^T [128, 192), dV [192, 320), dK [320, 448).
constexpr int TB_BK = 128;           // keys per CTA
constexpr int TB_BQ = 64;            // queries per block

constexpr int TB_KT = TB_BK * 256;   // K or V tile: 128 rows x 128 d (two 64-column boxes)
constexpr int TB_KBOX = TB_KT / 2;
constexpr int TB_QT = TB_BQ * 256;   // Q or dO tile: 64 rows x 128 d
constexpr int TB_QBOX = TB_QT / 2;
constexpr int TB_PT = TB_BK * 128;   // P^T or dS^T tile: 128 keys x 64 q (one box)
constexpr int TB_OFF_K = 0, TB_OFF_V = TB_KT, TB_OFF_STAGE = 2 * TB_KT;  // stage s at + 2 s TB_QT
constexpr int TB_OFF_P = TB_OFF_STAGE + 4 * TB_QT, TB_OFF_DS = TB_OFF_P + TB_PT;
constexpr int TB_OFF_DQ = TB_OFF_DS + TB_PT;              // [64 q][128 d] fp32
constexpr int TB_OFF_L = TB_OFF_DQ + TB_BQ * 128 * 4;     // [2][64] lse2, [2][64] Dvec
constexpr int TB_OFF_BAR = TB_OFF_L + 4 * TB_BQ * 4;
constexpr int TB_SMEM = TB_OFF_BAR + 256 + 1024;
constexpr int TB_KV_PITCH = 128 * 4 + 16;  // final dK / dV staging rows (conflict-free float4)
static_assert(2 * TB_BK * TB_KV_PITCH <= TB_OFF_DQ, "dK / dV staging over the dead tiles");

template <bool IS_BF16>
__global__ void __launch_bounds__(320, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                       const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                       AttnBwdC a, int* err) {
  pdl_enter();
  using T = typename std::conditional<IS_BF16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* sL = reinterpret_cast<float*>(smem + TB_OFF_L);  // [2][64]
  float* sDv = sL + 2 * TB_BQ;                              // [2][64]
  float* sDQ = reinterpret_cast<float*>(smem + TB_OFF_DQ);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TB_OFF_BAR);
  uint64_t* kv_full = bars;
  uint64_t* qd_full = bars + 1;   // [2] Q, dO landed and lse2 / Dvec stored
  uint64_t* qd_empty = bars + 3;  // [2] the MMAs reading the stage completed
  uint64_t* st_full = bars + 5;   // S^T, dP^T written
  uint64_t* st_free = bars + 6;   // S^T, dP^T read by the 128 softmax threads
  uint64_t* p_full = bars + 7;    // P^T, dS^T tiles written by the 128 softmax threads
  uint64_t* p_free = bars + 8;    // the MMAs reading P^T / dS^T completed
  uint64_t* dq_full = bars + 9;   // dQ^T written
  uint64_t* dq_free = bars + 10;  // dQ^T read by the 128 dQ threads
  uint64_t* dkv_full = bars + 11; // the last dV / dK MMAs completed
  uint64_t* dqs_free = bars + 12; // dQ staging read out by the previous block's reductions
  uint64_t* dqs_full = bars + 13; // dQ staging written by the 128 dQ threads
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);

  const int nkb = (int)cdiv(a.max_len, TB_BK);
  const int kb = blockIdx.x % nkb, chunk = blockIdx.x / nkb, h = blockIdx.y, b = blockIdx.z;
  const int start = a.cu_seqlens[b], len = a.cu_seqlens[b + 1] - start;
  const int qch = attn_bwd_qch(a.max_len);
  const int key0 = kb * TB_BK, q_first = key0 + chunk * qch;
  if (key0 >= len || q_first >= len) return;  // the whole CTA, before any setup
  const int q_end = min(len, q_first + qch);
  const int nq = (int)cdiv(q_end - q_first, TB_BQ);
  const int kvh = h / (a.HQ / a.HKV);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&qd_full[s], 33);  // lane 0's expect_tx arrival + all 32 lanes after their stores
      mbar_init(&qd_empty[s], 1);
    }
    mbar_init(st_full, 1);
    mbar_init(st_free, 128);
    mbar_init(p_full, 128);
    mbar_init(p_free, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 128);
    mbar_init(dkv_full, 1);
    mbar_init(dqs_free, 32);
    mbar_init(dqs_full, 128);
    fence_barrier_init();
    prefetch_tmap(&tq);
    prefetch_tmap(&tdo);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  constexpr uint32_t C_ST = 0, C_DPT = 64, C_DQT = 128, C_DV = 192, C_DK = 320;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * TB_KT);
      // each tile in one 3-D copy of both 64-column halves of the head
      tma_load_3d(smem + TB_OFF_K, &tk, kv_full, 0, start + key0, kvh * 2);
      tma_load_3d(smem + TB_OFF_V, &tv, kv_full, 0, start + key0, kvh * 2);
    }
    const float* lse = a.lse + (int64_t)h * a.n + start;
    const float* dvec = a.dvec + (int64_t)h * a.n + start;
    for (int j = 0; j < nq; ++j) {
      const int s = j & 1, q0 = q_first + j * TB_BQ;
      if (j >= 2 && !mbar_wait(&qd_empty[s], ((j >> 1) - 1) & 1, err)) break;
      if (lane == 0) {
        uint8_t* st = smem + TB_OFF_STAGE + s * 2 * TB_QT;
        mbar_arrive_expect_tx(&qd_full[s], 2 * TB_QT);
        tma_load_3d(st, &tq, &qd_full[s], 0, start + q0, h * 2);
        tma_load_3d(st + TB_QT, &tdo, &qd_full[s], 0, start + q0, h * 2);
      }
#pragma unroll
      for (int t = lane; t < TB_BQ; t += 32) {
        const int q = q0 + t;
        sL[s * TB_BQ + t] = q < len ? lse[q] * 1.4426950408889634f : INFINITY;  // p = 0 past len
        sDv[s * TB_BQ + t] = q < len ? dvec[q] : 0.f;
      }
      mbar_arrive(&qd_full[s]);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_st = umma_idesc_f16(IS_BF16, 128, TB_BQ);              // S^T, dP^T
      constexpr uint32_t id_kv = umma_idesc_f16(IS_BF16, 128, 128, true);           // dV, dK
      constexpr uint32_t id_dq = umma_idesc_f16(IS_BF16, 128, TB_BQ, true, true);   // dQ^T
      const uint32_t sk = smem_u32(smem + TB_OFF_K), sv = smem_u32(smem + TB_OFF_V);
      const uint32_t sp = smem_u32(smem + TB_OFF_P), sds = smem_u32(smem + TB_OFF_DS);
      bool ok = mbar_wait(kv_full, 0, err);
      for (int j = 0; ok && j <= nq; ++j) {
        if (j < nq) {
          const int s = j & 1;
          if (!mbar_wait(&qd_full[s], (j >> 1) & 1, err)) break;
          if (j >= 1 && !mbar_wait(st_free, (j - 1) & 1, err)) break;
          tc_fence_after();
          const uint32_t sq = smem_u32(smem + TB_OFF_STAGE + s * 2 * TB_QT), sdo = sq + TB_QT;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t ok_ = (kk >> 2) * TB_KBOX + (kk & 3) * 32, oq = (kk >> 2) * TB_QBOX + (kk & 3) * 32;
            umma_f16(tmem + C_ST, umma_desc_k_sw128(sk + ok_), umma_desc_k_sw128(sq + oq), id_st, kk > 0);
          }
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t ok_ = (kk >> 2) * TB_KBOX + (kk & 3) * 32, oq = (kk >> 2) * TB_QBOX + (kk & 3) * 32;
            umma_f16(tmem + C_DPT, umma_desc_k_sw128(sv + ok_), umma_desc_k_sw128(sdo + oq), id_st, kk > 0);
          }
          umma_commit(st_full);
        }
        if (j >= 1) {
          const int i = j - 1, s = i & 1;
          if (!mbar_wait(p_full, i & 1, err)) break;
          tc_fence_after();
          const uint32_t sq = smem_u32(smem + TB_OFF_STAGE + s * 2 * TB_QT), sdo = sq + TB_QT;
#pragma unroll
          for (int kk = 0; kk < TB_BQ / 16; ++kk) {  // dV += P^T dO ; dK += dS^T Q  (k = queries)
            umma_f16(tmem + C_DV, umma_desc_k_sw128(sp + kk * 32),
                     umma_desc_mn_sw128(sdo + kk * 2048, TB_QBOX, 1024), id_kv, (i > 0 || kk > 0));
            umma_f16(tmem + C_DK, umma_desc_k_sw128(sds + kk * 32),
                     umma_desc_mn_sw128(sq + kk * 2048, TB_QBOX, 1024), id_kv, (i > 0 || kk > 0));
          }
          if (i >= 1 && !mbar_wait(dq_free, (i - 1) & 1, err)) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < TB_BK / 16; ++kk)  // dQ^T = K^T dS^T  (k = keys)
            umma_f16(tmem + C_DQT, umma_desc_mn_sw128(sk + kk * 2048, TB_KBOX, 1024),
                     umma_desc_mn_sw128(sds + kk * 2048, TB_PT, 1024), id_dq, kk > 0);
          umma_commit(&qd_empty[s]);
          umma_commit(p_free);
          umma_commit(dq_full);
        }
      }
      umma_commit(dkv_full);
    }
  } else if (warp < 6) {
    // softmax: thread = key row r of the block
    const int quad = warp & 3, r = quad * 32 + lane, key = key0 + r;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const float sl2 = a.scale * 1.4426950408889634f;
    uint8_t* pP = smem + TB_OFF_P + r * 128;
    uint8_t* pS = smem + TB_OFF_DS + r * 128;
    bool ok = true;
    for (int j = 0; j < nq; ++j) {
      const int s = j & 1, q0 = q_first + j * TB_BQ;
      if (!mbar_wait(st_full, j & 1, err)) { ok = false; break; }
      tc_fence_after();
      uint32_t su[TB_BQ], du[TB_BQ];
      tmem_ld32_nw(lane_base + C_ST, su);
      tmem_ld32_nw(lane_base + C_ST + 32, su + 32);
      tmem_ld32_nw(lane_base + C_DPT, du);
      tmem_ld32_nw(lane_base + C_DPT + 32, du + 32);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(st_free);
      if (!mbar_wait(&qd_full[s], (j >> 1) & 1, err)) { ok = false; break; }
      if (j >= 1 && !mbar_wait(p_free, (j - 1) & 1, err)) { ok = false; break; }
      const float* l2 = sL + s * TB_BQ;
      const float* dv = sDv + s * TB_BQ;
      const bool diag = q0 < key0 + TB_BK;  // some query of the block precedes some key
#pragma unroll
      for (int ch = 0; ch < TB_BQ / 8; ++ch) {
        float p[8], ds[8];
        const float4 la = *reinterpret_cast<const float4*>(l2 + ch * 8);
        const float4 lb = *reinterpret_cast<const float4*>(l2 + ch * 8 + 4);
        const float4 da = *reinterpret_cast<const float4*>(dv + ch * 8);
        const float4 db = *reinterpret_cast<const float4*>(dv + ch * 8 + 4);
        const float lv[8] = {la.x, la.y, la.z, la.w, lb.x, lb.y, lb.z, lb.w};
        const float dd[8] = {da.x, da.y, da.z, da.w, db.x, db.y, db.z, db.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int c = ch * 8 + e;
          float pv = exp2f(fmaf(__uint_as_float(su[c]), sl2, -lv[e]));
          if (diag && q0 + c < key) pv = 0.f;
          p[e] = pv;
          ds[e] = pv * (__uint_as_float(du[c]) - dd[e]);
        }
        const uint32_t off = (uint32_t)(((ch ^ (r & 7))) << 4);
        *reinterpret_cast<uint4*>(pP + off) =
            make_uint4(pack_t2<T>(p[0], p[1]), pack_t2<T>(p[2], p[3]), pack_t2<T>(p[4], p[5]), pack_t2<T>(p[6], p[7]));
        *reinterpret_cast<uint4*>(pS + off) =
            make_uint4(pack_t2<T>(ds[0], ds[1]), pack_t2<T>(ds[2], ds[3]), pack_t2<T>(ds[4], ds[5]), pack_t2<T>(ds[6], ds[7]));
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // dK (scaled) and dV: TMEM -> staging over the dead tiles -> bulk reductions
    if (ok && mbar_wait(dkv_full, 0, err)) {
      tc_fence_after();
      uint8_t* stk = smem + r * TB_KV_PITCH;
      uint8_t* stv = smem + TB_BK * TB_KV_PITCH + r * TB_KV_PITCH;
#pragma unroll 1
      for (int c = 0; c < 128; c += 32) {
        float vk[32], vv[32];
        tmem_ld32(lane_base + C_DK + c, vk);
        tmem_ld32(lane_base + C_DV + c, vv);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          reinterpret_cast<float4*>(stk + c * 4)[u] =
              make_float4(vk[4 * u] * a.scale, vk[4 * u + 1] * a.scale, vk[4 * u + 2] * a.scale, vk[4 * u + 3] * a.scale);
          reinterpret_cast<float4*>(stv + c * 4)[u] = make_float4(vv[4 * u], vv[4 * u + 1], vv[4 * u + 2], vv[4 * u + 3]);
        }
      }
      fence_proxy_async_smem();
      if (key < len) {
        const int64_t row = ((int64_t)(start + key) * a.HKV + kvh) * 128;
        if (a.partials == nullptr) {
          bulk_reduce_add_f32(a.dk + row, reinterpret_cast<const float*>(stk), 512);
          bulk_reduce_add_f32(a.dv + row, reinterpret_cast<const float*>(stv), 512);
        } else {  // this (query head of the group, chunk)'s own slot
          const int group = a.HQ / a.HKV, nch = (int)cdiv(a.max_len, qch);
          const int64_t slot = ((int64_t)(h - kvh * group) * nch + chunk) * a.n * a.HKV * 128;
          float* pk = a.partials + attn_part_q_floats(a) + slot;
          float* pv = pk + attn_part_kv_floats(a);
          bulk_store(pk + row, reinterpret_cast<const float*>(stk), 512);
          bulk_store(pv + row, reinterpret_cast<const float*>(stv), 512);
        }
      }
      bulk_commit();
      bulk_wait<0>();
    }
  } else {
    // dQ: thread = d row of dQ^T
    const int quad = warp & 3, d = quad * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    for (int i = 0; i < nq; ++i) {
      const int q0 = q_first + i * TB_BQ;
      if (!mbar_wait(dq_full, i & 1, err)) break;
      tc_fence_after();
      float v[TB_BQ];
      tmem_ld32(lane_base + C_DQT, v);
      tmem_ld32(lane_base + C_DQT + 32, v + 32);
      tc_fence_before();
      mbar_arrive(dq_free);
      if (warp == 6) {  // the previous block's reductions have read the staging
        bulk_wait_read<0>();
        mbar_arrive(dqs_free);
      }
      if (!mbar_wait(dqs_free, i & 1, err)) break;
#pragma unroll
      for (int q = 0; q < TB_BQ; ++q) sDQ[q * 128 + d] = v[q] * a.scale;
      fence_proxy_async_smem();
      mbar_arrive(dqs_full);
      if (warp == 6) {
        if (!mbar_wait(dqs_full, i & 1, err)) break;
#pragma unroll
        for (int t = lane; t < TB_BQ; t += 32)
          if (q0 + t < len) {
            const int64_t off = ((int64_t)(start + q0 + t) * a.HQ + h) * 128;
            if (a.partials == nullptr) bulk_reduce_add_f32(a.dq + off, sDQ + t * 128, 512);
            else bulk_store(a.partials + (int64_t)kb * a.n * a.HQ * 128 + off, sDQ + t * 128, 512);
          }
        bulk_commit();
      }
    }
    if (warp == 6) bulk_wait<0>();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}
__global__ void exp2_fma_eval_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i < n) y[i] = exp2_fma(x[i]);
}

}  // namespace

int exp2_fma_eval(const float* x, float* y, int64_t n, cudaStream_t s) {
  if (n < 0 || (n > 0 && (x == nullptr || y == nullptr))) return QL_STATUS_BAD_ARG;
  if (n == 0) return QL_STATUS_OK;
  exp2_fma_eval_kernel<<<(unsigned)cdiv(n, 256), 256, 0, s>>>(x, y, n);
  return launched(1);
}

// Host side: tensor maps over q [n, HQ * 128] and k / v [n, HKV * 128] seen as {64 columns, n rows,
// 2 H column chunks} (128-byte swizzle; a box of {64, 128, 2} is one head's tile of 128 rows, both
// halves, in one copy; rows past n read as zeros).
int attn_fwd_tc(const AttnFwdC& a, cudaStream_t s) {
  if (a.D != TA_D) return QL_STATUS_UNSUPPORTED;
  const bool bf = a.dtype == QL_BF16;
  CUtensorMap mq, mk, mv;
  const int64_t wq = (int64_t)a.HQ * TA_D, wk = (int64_t)a.HKV * TA_D;
  if (make_chunked_map(&mq, a.q, a.n, wq, wq, 128, 2, bf) != QL_STATUS_OK ||
      make_chunked_map(&mk, a.k, a.n, wk, wk, 128, 2, bf) != QL_STATUS_OK ||
      make_chunked_map(&mv, a.v, a.n, wk, wk, 128, 2, bf) != QL_STATUS_OK)
    return QL_STATUS_CUDA;
  dim3 grid((unsigned)cdiv(a.max_len, TA_BM), (unsigned)a.HQ, (unsigned)a.B);
  int* err = status_word();
  if (bf) {
    smem_optin(reinterpret_cast<const void*>(attn_fwd_tc_kernel<true>), TA_SMEM);
    launch_k(attn_fwd_tc_kernel<true>, grid, dim3(64 + TA_SOFTMAX), TA_SMEM, s, mq, mk, mv, a, err);
  } else {
    smem_optin(reinterpret_cast<const void*>(attn_fwd_tc_kernel<false>), TA_SMEM);
    launch_k(attn_fwd_tc_kernel<false>, grid, dim3(64 + TA_SOFTMAX), TA_SMEM, s, mq, mk, mv, a, err);
  }
  return QL_STATUS_OK;
}

int attn_bwd_tc(const AttnBwdC& a, cudaStream_t s) {
  if (a.D != 128) return QL_STATUS_UNSUPPORTED;
  const bool bf = a.dtype == QL_BF16;
  CUtensorMap mq, mdo, mk, mv;
  const int64_t wq = (int64_t)a.HQ * 128, wk = (int64_t)a.HKV * 128;
  if (make_chunked_map(&mq, a.q, a.n, wq, wq, TB_BQ, 2, bf) != QL_STATUS_OK ||
      make_chunked_map(&mdo, a.dout, a.n, wq, wq, TB_BQ, 2, bf) != QL_STATUS_OK ||
      make_chunked_map(&mk, a.k, a.n, wk, wk, TB_BK, 2, bf) != QL_STATUS_OK ||
      make_chunked_map(&mv, a.v, a.n, wk, wk, TB_BK, 2, bf) != QL_STATUS_OK)
    return QL_STATUS_CUDA;
  dim3 grid((unsigned)(cdiv(a.max_len, TB_BK) * cdiv(a.max_len, attn_bwd_qch(a.max_len))),
            (unsigned)a.HQ, (unsigned)a.B);
  int* err = status_word();
  if (bf) {
    smem_optin(reinterpret_cast<const void*>(attn_bwd_tc_kernel<true>), TB_SMEM);
    launch_k(attn_bwd_tc_kernel<true>, grid, dim3(320), TB_SMEM, s, mq, mdo, mk, mv, a, err);
  } else {
    smem_optin(reinterpret_cast<const void*>(attn_bwd_tc_kernel<false>), TB_SMEM);
    launch_k(attn_bwd_tc_kernel<false>, grid, dim3(320), TB_SMEM, s, mq, mdo, mk, mv, a, err);
  }
  return QL_STATUS_OK;
}

}  // namespace ql
