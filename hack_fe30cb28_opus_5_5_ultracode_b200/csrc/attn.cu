// Varlen causal attention with grouped-query heads over the packed tokens of one step.
//
// Replaces PyTorch's memory-efficient attention in its cu_seqlens form (_attn_fwd / _attn_bwd,
// solution/engine.py:857-869): q [n, HQ, D], k and v [n, HKV, D] (one copy per KV head, shared by
// the HQ / HKV query heads of its group), sequences given by cu_seqlens [B + 1], causal within a
// sequence, scale D^-1/2. Forward writes out [n, HQ, D] and the natural-log logsumexp [HQ, n];
// backward recomputes the probabilities from it (FlashAttention-2 scheme, Dao 2023) and writes
// dq [n, HQ, D], dk and dv [n, HKV, D] in fp32 (accumulated over the GQA group and query blocks).
//
// Runs on the warp-level tensor-core path (mma.sync m16n8k16, fp32 accumulation); the tiles are
// 64 queries x 64 keys, head dim D = 128 (Qwen2.5) or 64, staged by cp.async into XOR-swizzled
// shared memory read with ldmatrix. The forward's online softmax raises its running row max
// lazily (output rescaled only on a rise of more than 2^8); the backward's fp32 gradient tiles are
// added to dq / dk / dv by bulk reductions from shared memory (cp.reduce.async.bulk).
#include <atomic>

#include "common.cuh"
#include "profile.h"
#include "ops.h"

namespace ql {

constexpr int AT_BM = 64;   // queries per forward CTA (= AT_BN: the Q tile borrows a K buffer)
constexpr int AT_BN = 64;   // keys per step / per backward CTA
constexpr int AT_BQ = 32;   // queries per backward step
constexpr int AT_LONG = 1024; // max_len from which the forward takes its long-sequence shape
constexpr int AT_QCH = 128; // queries per backward CTA (a chunk of a key block's rows)

// element offset of (row, col) in a [rows][D] 16-bit tile (D = 64 or 128) with its 16-byte
// chunks XOR-swizzled by the row (conflict-free ldmatrix)
template <int D>
__device__ __forceinline__ int sw(int row, int col) {
  return row * D + ((((col >> 3) ^ (row & 7))) << 3) + (col & 7);
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(pred ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Loads rows [r0, r0 + ROWS) of a [len, heads, D] sequence slice (row stride ld elements) into a
// swizzled [ROWS][D] tile; rows at or past len are zero-filled.
template <typename T, int D, int ROWS, int NT>
__device__ __forceinline__ void load_tile(T* tile, const T* base, int64_t ld, int r0, int len) {
  constexpr int CPR = D / 8;  // 16-byte chunks per row
  constexpr int CHUNKS = ROWS * CPR;
  for (int i = threadIdx.x; i < CHUNKS; i += NT) {
    const int r = i / CPR, ch = i % CPR;
    const bool ok = r0 + r < len;
    const T* src = ok ? base + (int64_t)(r0 + r) * ld + ch * 8 : base;
    cp_async16(tile + sw<D>(r, ch * 8), src, ok);
  }
}

// ---------------------------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------------------------
// Two shapes of the same kernel. kShare (long sequences, many key blocks per CTA): the Q tile is
// staged in the second K buffer and its fragments move to registers before the first prefetch
// overwrites it, so a CTA holds 64 KB (D = 128) and three CTAs share an SM. Otherwise (short
// sequences, one wave of CTAs whose latency is the kernel's time): Q has its own buffer, the
// second key block is prefetched at once, and the register budget is that of two CTAs per SM.
template <typename T, int AT_D, bool kShare>
__global__ void __launch_bounds__(128, kShare ? 3 : 2) attn_fwd_kernel(AttnFwdC a) {
  pdl_enter();
  extern __shared__ __align__(16) uint8_t at_smem[];
  T* sK = reinterpret_cast<T*>(at_smem);  // [2][64][D]
  T* sV = sK + 2 * AT_BN * AT_D;          // [2][64][D]
  T* sQ = kShare ? sK + AT_BN * AT_D : sV + 2 * AT_BN * AT_D;
  // the longest causal rows first: the last query blocks of a sequence run the most key blocks
  const int qb = gridDim.x - 1 - blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int start = a.cu_seqlens[b], len = a.cu_seqlens[b + 1] - start;
  if (qb * AT_BM >= len) return;
  const int group = a.HQ / a.HKV, kvh = h / group;
  const int64_t ldq = (int64_t)a.HQ * AT_D, ldk = (int64_t)a.HKV * AT_D;
  const T* Q = reinterpret_cast<const T*>(a.q) + (int64_t)start * ldq + h * AT_D;
  const T* K = reinterpret_cast<const T*>(a.k) + (int64_t)start * ldk + kvh * AT_D;
  const T* V = reinterpret_cast<const T*>(a.v) + (int64_t)start * ldk + kvh * AT_D;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const float sl2 = a.scale * 1.4426950408889634f;  // scale * log2(e)

  load_tile<T, AT_D, AT_BM, 128>(sQ, Q, ldq, qb * AT_BM, len);
  const int nkb = qb + 1;  // causal: key blocks 0 .. qb
  load_tile<T, AT_D, AT_BN, 128>(sK, K, ldk, 0, len);
  load_tile<T, AT_D, AT_BN, 128>(sV, V, ldk, 0, len);
  cp_async_commit();

  constexpr int NT = AT_D / 8;   // 8-wide d tiles
  constexpr int KS = AT_D / 16;  // 16-wide k steps over d
  float o[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  uint32_t qf[KS][4];
  const int qrow0 = qb * AT_BM + warp * 16;  // first query row of this warp (in the sequence)

  auto load_q_fragments = [&]() {
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      const int c = kk * 16 + (lane >> 4) * 8;
      ldsm_x4(sQ + sw<AT_D>(r, c), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
    }
  };
  if (kShare) {
    cp_async_wait<0>();
    __syncthreads();
    load_q_fragments();
    __syncthreads();  // every warp holds its Q fragments: K buffer 1 is free
  }

  for (int kb = 0; kb < nkb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < nkb) {
      load_tile<T, AT_D, AT_BN, 128>(sK + (buf ^ 1) * AT_BN * AT_D, K, ldk, (kb + 1) * AT_BN, len);
      load_tile<T, AT_D, AT_BN, 128>(sV + (buf ^ 1) * AT_BN * AT_D, V, ldk, (kb + 1) * AT_BN, len);
      cp_async_commit();
      cp_async_wait<1>();
      __syncthreads();
    } else if (!kShare || kb > 0) {
      cp_async_wait<0>();
      __syncthreads();
    }
    if (!kShare && kb == 0) load_q_fragments();
    const T* tK = sK + buf * AT_BN * AT_D;
    const T* tV = sV + buf * AT_BN * AT_D;
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {  // pairs of 8-key n-tiles
        uint32_t b0, b1, b2, b3;
        const int r = jp * 16 + (lane & 7) + (lane >> 4) * 8;
        const int c = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(tK + sw<AT_D>(r, c), b0, b1, b2, b3);
        mma16816<T>(s[2 * jp], qf[kk], b0, b1);
        mma16816<T>(s[2 * jp + 1], qf[kk], b2, b3);
      }
    }
    // causal / length mask and online softmax (rows g and g + 8 of this warp). The running max
    // mrow is in the scaled log2 domain and is raised lazily: only when a row's new max exceeds
    // it by more than 8 (probabilities up to 2^8 stay exact in the 16-bit P and fp32 sums) are O
    // and l rescaled, and never unless some row of the warp needs it.
    const bool diag = kb == qb;
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int qi = qrow0 + g + hr * 8;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          if (diag) {
            const int kj = kb * AT_BN + j * 8 + 2 * t4 + e;
            if (kj > qi || kj >= len) s[j][hr * 2 + e] = -INFINITY;
          }
          mx = fmaxf(mx, s[j][hr * 2 + e]);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float ms = mx * sl2;  // this block's row max, scaled
      const bool raise = ms > mrow[hr] + 8.f;
      if (__any_sync(0xffffffffu, raise)) {
        const float m_new = raise ? ms : mrow[hr];
        const float corr = mrow[hr] == -INFINITY ? 0.f : exp2f(mrow[hr] - m_new);
        mrow[hr] = m_new;
        lrow[hr] *= corr;
#pragma unroll
        for (int i = 0; i < NT; ++i) {
          o[i][hr * 2] *= corr;
          o[i][hr * 2 + 1] *= corr;
        }
      }
      const float mneg = mrow[hr] == -INFINITY ? 0.f : -mrow[hr];
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float p = exp2f(fmaf(s[j][hr * 2 + e], sl2, mneg));  // exp2(-inf) = 0
          s[j][hr * 2 + e] = p;
          sum += p;
        }
      }
      lrow[hr] += sum;
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // 16 keys per k-step
      uint32_t pa[4];
      pa[0] = pack_t2<T>(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_t2<T>(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_t2<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_t2<T>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {  // pairs of 8-wide d tiles
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = np * 16 + (lane >> 4) * 8;
        ldsm_x4_t(tV + sw<AT_D>(r, c), b0, b1, b2, b3);
        mma16816<T>(o[2 * np], pa, b0, b1);
        mma16816<T>(o[2 * np + 1], pa, b2, b3);
      }
    }
    __syncthreads();  // the buffer is reloaded two steps later
  }
  // finalize
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    float l = lrow[hr];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const int qi = qrow0 + g + hr * 8;
    if (qi < len) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T* out = reinterpret_cast<T*>(a.out) + ((int64_t)(start + qi) * a.HQ + h) * AT_D;
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        *reinterpret_cast<uint32_t*>(out + i * 8 + 2 * t4) = pack_t2<T>(o[i][hr * 2] * inv, o[i][hr * 2 + 1] * inv);
      }
      if (t4 == 0) a.lse[(int64_t)h * a.n + start + qi] = (mrow[hr] + log2f(l)) * 0.6931471805599453f;
    }
  }
}

template <typename T, int D, bool kShare>
static void launch_attn_fwd_shape(const AttnFwdC& a, cudaStream_t s) {
  const int smem = (kShare ? 4 * AT_BN : 4 * AT_BN + AT_BM) * D * 2;
  static bool cfg = false;
  if (!cfg) {
    cudaFuncSetAttribute(attn_fwd_kernel<T, D, kShare>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cfg = true;
  }
  dim3 grid((unsigned)cdiv(a.max_len, AT_BM), (unsigned)a.HQ, (unsigned)a.B);
  launch_k(attn_fwd_kernel<T, D, kShare>, grid, dim3(128), smem, s, a);
}
template <typename T, int D>
static void launch_attn_fwd(const AttnFwdC& a, cudaStream_t s) {
  if (a.max_len >= AT_LONG) launch_attn_fwd_shape<T, D, true>(a, s);
  else launch_attn_fwd_shape<T, D, false>(a, s);
}

static std::atomic<int> g_attn_impl{0};
void attn_set_impl(int impl) { g_attn_impl.store(impl); }

int attn_fwd(const AttnFwdC& a, cudaStream_t s) {
  if (a.D != 128 && a.D != 64) return QL_STATUS_UNSUPPORTED;
  if (a.n < 0 || a.B < 0 || a.HKV <= 0 || a.HQ % a.HKV != 0 || a.max_len < 0) return QL_STATUS_BAD_ARG;
  if (a.n == 0 || a.B == 0 || a.max_len == 0) return QL_STATUS_OK;
  ProfScope prof(PK_ATTN_FWD, 0, 0, s);
  if (a.D == 128 && (a.dtype == QL_F16 || a.dtype == QL_BF16) && g_attn_impl.load() != 1) {
    const int st = attn_fwd_tc(a, s);
    return st == QL_STATUS_OK ? launched(1) : st;
  }
  if (a.dtype == QL_F16) {
    if (a.D == 128) launch_attn_fwd<__half, 128>(a, s); else launch_attn_fwd<__half, 64>(a, s);
  } else if (a.dtype == QL_BF16) {
    if (a.D == 128) launch_attn_fwd<__nv_bfloat16, 128>(a, s); else launch_attn_fwd<__nv_bfloat16, 64>(a, s);
  } else {
    return QL_STATUS_BAD_ARG;
  }
  return launched(1);
}

}  // namespace ql

namespace ql {

// ---------------------------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------------------------
// Dvec[h][t] = sum_d dO[t, h, d] * O[t, h, d] (the softmax-gradient row term).
template <typename T, int AT_D>
__global__ void attn_bwd_pre_kernel(const T* __restrict__ dout, const T* __restrict__ out,
                                    float* __restrict__ dvec, int64_t n, int HQ,
                                    float* __restrict__ dq, float* __restrict__ dk,
                                    float* __restrict__ dv, int64_t kv_vec4) {
  pdl_enter();
  // the gradients the backward kernel bulk-adds into start from zero: one float4 of dq per thread
  // (n HQ rows of 32 float4), and of dk and dv for the first kv_vec4 threads (null: not needed)
  const int64_t gid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  if (dq != nullptr && gid < n * HQ * (AT_D / 4)) reinterpret_cast<float4*>(dq)[gid] = zero;
  if (dk != nullptr && gid < kv_vec4) {
    reinterpret_cast<float4*>(dk)[gid] = zero;
    reinterpret_cast<float4*>(dv)[gid] = zero;
  }
  const int64_t row = blockIdx.x * (int64_t)(blockDim.x / 32) + (threadIdx.x >> 5);  // (t, h)
  const int lane = threadIdx.x & 31;
  if (row >= n * HQ) return;
  const T* a = dout + row * AT_D;
  const T* b = out + row * AT_D;
  float s = 0.f;
  constexpr int PER = AT_D / 32;
#pragma unroll
  for (int j = 0; j < PER; ++j) s += to_f<T>(a[lane * PER + j]) * to_f<T>(b[lane * PER + j]);
  s = warp_sum(s);
  if (lane == 0) {
    const int64_t t = row / HQ;
    const int h = (int)(row % HQ);
    dvec[(int64_t)h * n + t] = s;
  }
}

// One CTA per (64-key block, query head, sequence); 4 warps, warp w owns keys 16w .. 16w + 15.
// Steps over the query rows from the key block's start in blocks of 32: recomputes P^T, then
// dV += P^T dO, dP^T = V dO^T, dS^T = P^T (dP^T - Dvec), dK += dS^T Q, and dQ += dS K through a
// shared-memory copy of dS^T. The step's dQ tile is staged in shared memory and added to the
// fp32 dq rows by bulk reductions (one 4D-byte row per query, issued by warp 0's lanes); dK and dV
// are staged the same way at the end and bulk-added into the KV head's fp32 rows (the query
// chunks and the group's query heads all contribute).
template <typename T, int AT_D>
__global__ void __launch_bounds__(128) attn_bwd_kernel(AttnBwdC a) {
  pdl_enter();
  extern __shared__ __align__(16) uint8_t at_smem[];
  T* sK = reinterpret_cast<T*>(at_smem);   // [64][D]
  T* sV = sK + AT_BN * AT_D;                // [64][D]
  T* sQ = sV + AT_BN * AT_D;                // [2][32][D]
  T* sO = sQ + 2 * AT_BQ * AT_D;            // [2][32][D] (dO)
  T* sS = sO + 2 * AT_BQ * AT_D;            // [64][40] dS^T (padded rows)
  float* sL = reinterpret_cast<float*>(sS + AT_BN * 40);  // [2][32] lse * log2(e)
  float* sD = sL + 2 * AT_BQ;                              // [2][32] Dvec
  float* sDQ = sD + 2 * AT_BQ;                             // [32][D + 8] dQ tile (fp32)
  constexpr int SROW = 40;
  constexpr int FROW = AT_D + 8;  // fp32 staging pitch: 16-byte rows, conflict-free float2 stores

  // blockIdx.x = (query chunk) x (key block): the key block's query rows are cut into chunks of
  // AT_QCH so that no CTA walks a long sequence alone (dK / dV are added atomically anyway)
  const int nkb = (int)cdiv(a.max_len, AT_BN);
  const int kb = blockIdx.x % nkb, chunk = blockIdx.x / nkb, h = blockIdx.y, b = blockIdx.z;
  const int start = a.cu_seqlens[b], len = a.cu_seqlens[b + 1] - start;
  if (kb * AT_BN >= len || kb * AT_BN + chunk * AT_QCH >= len) return;
  const int group = a.HQ / a.HKV, kvh = h / group;
  const int64_t ldq = (int64_t)a.HQ * AT_D, ldk = (int64_t)a.HKV * AT_D;
  const T* Q = reinterpret_cast<const T*>(a.q) + (int64_t)start * ldq + h * AT_D;
  const T* dO = reinterpret_cast<const T*>(a.dout) + (int64_t)start * ldq + h * AT_D;
  const T* K = reinterpret_cast<const T*>(a.k) + (int64_t)start * ldk + kvh * AT_D;
  const T* V = reinterpret_cast<const T*>(a.v) + (int64_t)start * ldk + kvh * AT_D;
  const float* lse = a.lse + (int64_t)h * a.n + start;
  const float* dvec = a.dvec + (int64_t)h * a.n + start;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const float sl2 = a.scale * 1.4426950408889634f;

  load_tile<T, AT_D, AT_BN, 128>(sK, K, ldk, kb * AT_BN, len);
  load_tile<T, AT_D, AT_BN, 128>(sV, V, ldk, kb * AT_BN, len);
  const int q_first = kb * AT_BN + chunk * AT_QCH;
  const int q_end = min(len, q_first + AT_QCH);
  const int nsteps = (int)cdiv(q_end - q_first, AT_BQ);
  auto load_q = [&](int step, int buf) {
    const int r0 = q_first + step * AT_BQ;
    load_tile<T, AT_D, AT_BQ, 128>(sQ + buf * AT_BQ * AT_D, Q, ldq, r0, len);
    load_tile<T, AT_D, AT_BQ, 128>(sO + buf * AT_BQ * AT_D, dO, ldq, r0, len);
    if (threadIdx.x < AT_BQ) {
      const int qi = r0 + threadIdx.x;
      sL[buf * AT_BQ + threadIdx.x] = qi < len ? lse[qi] * 1.4426950408889634f : INFINITY;  // masked: p = 0
      sD[buf * AT_BQ + threadIdx.x] = qi < len ? dvec[qi] : 0.f;
    }
  };
  load_q(0, 0);
  cp_async_commit();

  constexpr int NT = AT_D / 8, KS = AT_D / 16;
  float dk[NT][4], dv[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    dk[i][0] = dk[i][1] = dk[i][2] = dk[i][3] = 0.f;
    dv[i][0] = dv[i][1] = dv[i][2] = dv[i][3] = 0.f;
  }
  const int key0 = kb * AT_BN + warp * 16;  // this warp's first key (in the sequence)

  for (int st = 0; st < nsteps; ++st) {
    const int buf = st & 1;
    if (st + 1 < nsteps) {
      load_q(st + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    if (warp == 0) bulk_wait_read<0>();  // the previous step's dQ tile has been read out
    __syncthreads();
    const T* tQ = sQ + buf * AT_BQ * AT_D;
    const T* tO = sO + buf * AT_BQ * AT_D;
    const float* tL = sL + buf * AT_BQ;
    const float* tD = sD + buf * AT_BQ;
    const int qbase = q_first + st * AT_BQ;

    // S^T = K_w Q^T and dP^T = V_w dO^T: 16 keys x 32 queries each
    float s[4][4], dp[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
      dp[j][0] = dp[j][1] = dp[j][2] = dp[j][3] = 0.f;
    }
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      uint32_t ka[4], va[4];
      const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      const int c = kk * 16 + (lane >> 4) * 8;
      ldsm_x4(sK + sw<AT_D>(r, c), ka[0], ka[1], ka[2], ka[3]);
      ldsm_x4(sV + sw<AT_D>(r, c), va[0], va[1], va[2], va[3]);
#pragma unroll
      for (int jp = 0; jp < 2; ++jp) {
        uint32_t b0, b1, b2, b3;
        const int qr = jp * 16 + (lane & 7) + (lane >> 4) * 8;
        const int qc = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(tQ + sw<AT_D>(qr, qc), b0, b1, b2, b3);
        mma16816<T>(s[2 * jp], ka, b0, b1);
        mma16816<T>(s[2 * jp + 1], ka, b2, b3);
        ldsm_x4(tO + sw<AT_D>(qr, qc), b0, b1, b2, b3);
        mma16816<T>(dp[2 * jp], va, b0, b1);
        mma16816<T>(dp[2 * jp + 1], va, b2, b3);
      }
    }
    // P^T and dS^T (rows: keys g, g + 8 of the warp; columns: queries)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = key0 + g + (e >> 1) * 8;
        const int ql = j * 8 + 2 * t4 + (e & 1);  // query within the step
        const int qi = qbase + ql;
        float p = exp2f(fmaf(s[j][e], sl2, -tL[ql]));
        if (key > qi || qi >= len || key >= len) p = 0.f;
        s[j][e] = p;
        dp[j][e] = p * (dp[j][e] - tD[ql]);
      }
    }
    // dV += P^T dO ; dK += dS^T Q   (k = 32 queries: 2 k-steps)
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      uint32_t pa[4], sa[4];
      pa[0] = pack_t2<T>(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_t2<T>(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_t2<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_t2<T>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
      sa[0] = pack_t2<T>(dp[2 * kk][0], dp[2 * kk][1]);
      sa[1] = pack_t2<T>(dp[2 * kk][2], dp[2 * kk][3]);
      sa[2] = pack_t2<T>(dp[2 * kk + 1][0], dp[2 * kk + 1][1]);
      sa[3] = pack_t2<T>(dp[2 * kk + 1][2], dp[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = np * 16 + (lane >> 4) * 8;
        ldsm_x4_t(tO + sw<AT_D>(r, c), b0, b1, b2, b3);
        mma16816<T>(dv[2 * np], pa, b0, b1);
        mma16816<T>(dv[2 * np + 1], pa, b2, b3);
        ldsm_x4_t(tQ + sw<AT_D>(r, c), b0, b1, b2, b3);
        mma16816<T>(dk[2 * np], sa, b0, b1);
        mma16816<T>(dk[2 * np + 1], sa, b2, b3);
      }
    }
    // dS^T to shared memory: sS[key][query]
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int kr = warp * 16 + g + hr * 8;
        *reinterpret_cast<uint32_t*>(sS + kr * SROW + j * 8 + 2 * t4) =
            pack_t2<T>(dp[j][hr * 2], dp[j][hr * 2 + 1]);
      }
    }
    __syncthreads();
    // dQ (32 queries x D) = dS (32 x 64 keys) K (64 x D): warp -> 16 queries x D/2
    {
      constexpr int HT = AT_D / 16;  // 8-wide d tiles per warp
      const int qm = (warp & 1) * 16, dn = (warp >> 1) * (AT_D / 2);
      float dq[HT][4];
#pragma unroll
      for (int i = 0; i < HT; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t aq[4];
        // A[m = query][k = key] from sS[key][query] (transposed load)
        const int mi = lane >> 3;
        const int kr = kk * 16 + (lane & 7) + (mi >> 1) * 8;
        const int qc = qm + (mi & 1) * 8;
        ldsm_x4_t(sS + kr * SROW + qc, aq[0], aq[1], aq[2], aq[3]);
#pragma unroll
        for (int np = 0; np < HT / 2; ++np) {
          uint32_t b0, b1, b2, b3;
          const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = dn + np * 16 + (lane >> 4) * 8;
          ldsm_x4_t(sK + sw<AT_D>(r, c), b0, b1, b2, b3);
          mma16816<T>(dq[2 * np], aq, b0, b1);
          mma16816<T>(dq[2 * np + 1], aq, b2, b3);
        }
      }
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        float* row = sDQ + (qm + g + hr * 8) * FROW + dn + 2 * t4;
#pragma unroll
        for (int i = 0; i < HT; ++i)
          *reinterpret_cast<float2*>(row + i * 8) = make_float2(dq[i][hr * 2] * a.scale, dq[i][hr * 2 + 1] * a.scale);
      }
      fence_proxy_async_smem();
    }
    __syncthreads();  // sS and the dQ tile written; the Q / dO buffer is reloaded next step
    if (warp == 0) {
      const int qi = qbase + lane;
      if (qi < len)
        bulk_reduce_add_f32(a.dq + ((int64_t)(start + qi) * a.HQ + h) * AT_D, sDQ + lane * FROW, AT_D * 4);
      bulk_commit();
    }
  }
  // dK (scaled) and dV staged over the K / V / Q / dO / dS^T tiles (all dead after the last
  // step's closing barrier), then bulk-added into the KV head's fp32 rows
  float* sDK = reinterpret_cast<float*>(at_smem);  // [64][D + 8]
  float* sDV = sDK + AT_BN * FROW;                  // [64][D + 8]
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int kr = warp * 16 + g + hr * 8;
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      *reinterpret_cast<float2*>(sDK + kr * FROW + i * 8 + 2 * t4) = make_float2(dk[i][hr * 2] * a.scale, dk[i][hr * 2 + 1] * a.scale);
      *reinterpret_cast<float2*>(sDV + kr * FROW + i * 8 + 2 * t4) = make_float2(dv[i][hr * 2], dv[i][hr * 2 + 1]);
    }
  }
  fence_proxy_async_smem();
  __syncthreads();
  {
    const int r = threadIdx.x & (AT_BN - 1);  // threads 0-63: dK rows, 64-127: dV rows
    const int key = kb * AT_BN + r;
    if (key < len) {
      float* dst = (threadIdx.x < AT_BN ? a.dk : a.dv) + ((int64_t)(start + key) * a.HKV + kvh) * AT_D;
      bulk_reduce_add_f32(dst, (threadIdx.x < AT_BN ? sDK : sDV) + r * FROW, AT_D * 4);
    }
    bulk_commit();
    bulk_wait<0>();  // dQ, dK and dV reductions of this thread complete before the CTA exits
  }
}

template <typename T, int D>
static void launch_attn_bwd(const AttnBwdC& a, cudaStream_t s) {
  const int64_t rows = (int64_t)a.n * a.HQ;
  launch_k(attn_bwd_pre_kernel<T, D>, dim3((unsigned)cdiv(rows, 8)), dim3(256), 0, s,
      (const T*)a.dout, (const T*)a.out, a.dvec, a.n, a.HQ, a.dq, a.dk, a.dv,
      (int64_t)a.n * a.HKV * (D / 4));
  if (a.max_len == 0) return;  // every sequence empty: the zeroed gradients are the answer
  const int smem = (2 * AT_BN + 4 * AT_BQ) * D * 2 + AT_BN * 40 * 2 + 4 * AT_BQ * 4 +
                   AT_BQ * (D + 8) * 4;
  static_assert(AT_BQ == 32 && 2 * AT_BN == 128, "one dQ row per lane of warp 0; one dK / dV row per thread");
  static bool cfg = false;
  if (!cfg) {
    cudaFuncSetAttribute(attn_bwd_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cfg = true;
  }
  dim3 grid((unsigned)(cdiv(a.max_len, AT_BN) * cdiv(a.max_len, AT_QCH)), (unsigned)a.HQ,
            (unsigned)a.B);
  launch_k(attn_bwd_kernel<T, D>, grid, dim3(128), smem, s, a);
}

static std::atomic<bool> g_attn_det{false};
void attn_set_deterministic(bool on) { g_attn_det.store(on); }
bool attn_deterministic() { return g_attn_det.load(); }

// The deterministic backward's sums: thread = (row, head, 4 columns). dq of query row p (position
// in its sequence) adds the contributions of key blocks 0 .. p / 128; dk / dv of key row j add,
// over the GQA group's query heads g and the query chunks c (attn_bwd_qch queries each) that
// exist for j's key block, slot (g, c), in that order.
__global__ void attn_bwd_det_reduce_kernel(const float* __restrict__ parts, AttnBwdC a) {
  pdl_enter();  // the backward kernel's partials are complete and visible from here on
  const int hh_all = a.HQ + 2 * a.HKV;
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= (int64_t)a.n * hh_all * 32) return;
  const int c4 = (int)(idx % 32), hh = (int)((idx / 32) % hh_all);
  const int64_t row = idx / (32 * (int64_t)hh_all);
  int lo = 0, hi = a.B;  // the sequence holding row: cu[lo] <= row < cu[lo + 1]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (a.cu_seqlens[mid] <= row) lo = mid; else hi = mid;
  }
  const int start = a.cu_seqlens[lo], len = a.cu_seqlens[lo + 1] - start;
  const int p = (int)(row - start), kb = p / 128;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  auto add = [&](const float* src) {
    const float4 v = *reinterpret_cast<const float4*>(src + 4 * c4);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  };
  if (hh < a.HQ) {
    const float* q = parts + (row * a.HQ + hh) * 128;
    for (int b = 0; b <= kb; ++b) add(q + (int64_t)b * a.n * a.HQ * 128);
    *reinterpret_cast<float4*>(a.dq + (row * a.HQ + hh) * 128 + 4 * c4) = acc;
  } else {
    const int which = (hh - a.HQ) / a.HKV, j = (hh - a.HQ) % a.HKV;
    const int qch = attn_bwd_qch(a.max_len);
    const int group = a.HQ / a.HKV, nch = (a.max_len + qch - 1) / qch;
    const int chunks = (len - kb * 128 + qch - 1) / qch;
    const float* base = parts + attn_part_q_floats(a) + which * attn_part_kv_floats(a) +
                        (row * a.HKV + j) * 128;
    for (int g = 0; g < group; ++g)
      for (int c = 0; c < chunks; ++c) add(base + ((int64_t)g * nch + c) * a.n * a.HKV * 128);
    float* dst = which == 0 ? a.dk : a.dv;
    *reinterpret_cast<float4*>(dst + (row * a.HKV + j) * 128 + 4 * c4) = acc;
  }
}

int attn_bwd(const AttnBwdC& a, cudaStream_t s) {
  if (a.D != 128 && a.D != 64) return QL_STATUS_UNSUPPORTED;
  if (a.n < 0 || a.B < 0 || a.HKV <= 0 || a.HQ % a.HKV != 0 || a.max_len < 0) return QL_STATUS_BAD_ARG;
  if (a.n == 0 || a.B == 0) return QL_STATUS_OK;
  if (a.dvec == nullptr) return QL_STATUS_BAD_ARG;
  // dq, dk and dv rows are bulk-reduced: 16-byte aligned bases
  if ((reinterpret_cast<uintptr_t>(a.dq) | reinterpret_cast<uintptr_t>(a.dk) |
       reinterpret_cast<uintptr_t>(a.dv)) & 15)
    return QL_STATUS_BAD_ARG;
  const bool tc = a.D == 128 && (a.dtype == QL_F16 || a.dtype == QL_BF16) && g_attn_impl.load() != 1;
  if (a.partials != nullptr && (!tc || (reinterpret_cast<uintptr_t>(a.partials) & 15)))
    return QL_STATUS_UNSUPPORTED;  // the deterministic form: tcgen05 kernels, 16-byte aligned
  ProfScope prof(PK_ATTN_BWD, 0, 0, s);
  if (a.partials != nullptr) {  // every contribution to its own slot, then one ordered sum
    if (a.max_len == 0) return QL_STATUS_OK;
    const int64_t rows = (int64_t)a.n * a.HQ;
    if (a.dtype == QL_F16)
      launch_k(attn_bwd_pre_kernel<__half, 128>, dim3((unsigned)cdiv(rows, 8)), dim3(256), 0, s,
               (const __half*)a.dout, (const __half*)a.out, a.dvec, a.n, a.HQ, (float*)nullptr,
               (float*)nullptr, (float*)nullptr, (int64_t)0);
    else
      launch_k(attn_bwd_pre_kernel<__nv_bfloat16, 128>, dim3((unsigned)cdiv(rows, 8)), dim3(256), 0, s,
               (const __nv_bfloat16*)a.dout, (const __nv_bfloat16*)a.out, a.dvec, a.n, a.HQ,
               (float*)nullptr, (float*)nullptr, (float*)nullptr, (int64_t)0);
    const int st = attn_bwd_tc(a, s);
    if (st != QL_STATUS_OK) return st;
    const int64_t threads = (int64_t)a.n * (a.HQ + 2 * a.HKV) * 32;
    launch_k(attn_bwd_det_reduce_kernel, dim3((unsigned)cdiv(threads, 256)), dim3(256), 0, s,
             (const float*)a.partials, a);
    return launched(3);
  }
  // the gradients accumulate by bulk reductions from zero: the pre-kernel (which every path runs
  // first) zeroes them, so no separate memset breaks the launch chain
  if (tc) {
    const int64_t rows = (int64_t)a.n * a.HQ;
    const int64_t kv4 = (int64_t)a.n * a.HKV * 32;
    if (a.dtype == QL_F16)
      launch_k(attn_bwd_pre_kernel<__half, 128>, dim3((unsigned)cdiv(rows, 8)), dim3(256), 0, s,
               (const __half*)a.dout, (const __half*)a.out, a.dvec, a.n, a.HQ, a.dq, a.dk, a.dv,
               kv4);
    else
      launch_k(attn_bwd_pre_kernel<__nv_bfloat16, 128>, dim3((unsigned)cdiv(rows, 8)), dim3(256), 0, s,
               (const __nv_bfloat16*)a.dout, (const __nv_bfloat16*)a.out, a.dvec, a.n, a.HQ, a.dq,
               a.dk, a.dv, kv4);
    if (a.max_len == 0) return launched(1);
    const int st = attn_bwd_tc(a, s);
    return st == QL_STATUS_OK ? launched(2) : st;
  }
  if (a.dtype == QL_F16) {
    if (a.D == 128) launch_attn_bwd<__half, 128>(a, s); else launch_attn_bwd<__half, 64>(a, s);
  } else if (a.dtype == QL_BF16) {
    if (a.D == 128) launch_attn_bwd<__nv_bfloat16, 128>(a, s); else launch_attn_bwd<__nv_bfloat16, 64>(a, s);
  } else {
    return QL_STATUS_BAD_ARG;
  }
  return launched(a.max_len == 0 ? 1 : 2);
}

}  // namespace ql
