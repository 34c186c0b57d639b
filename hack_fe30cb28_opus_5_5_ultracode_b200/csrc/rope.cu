// qkv + LoRA + rotary embedding, forward and backward, CTA tiles of up to 16 tokens.
//
// Forward (reference qkv_rope_fwd_kernel, solution/kernels.py:212-264): splits the biased qkv
// GEMM output into q, k, v, adds lora_scale * (the LoRA-B output) to q and v in fp32, and rotates
// q and k with Qwen2's rotate-half RoPE: out[:h] = x1 cos - x2 sin, out[h:] = x2 cos + x1 sin.
// The LoRA-B output is either given ([n, HQ*D], [n, HKV*D]) or formed here from the rank-16
// factor, lq = x_lo . B^T rounded to the 16-bit type (the reference's separate fp16 GEMM,
// solution/engine.py:1088-1093). k and v are written per KV head ([n, HKV, D]); the attention
// kernels share them across the GQA group instead of an expanded copy.
//
// Backward (reference qkv_rope_bwd_kernel, solution/kernels.py:267-306): the inverse rotation of
// dq and dk, dk / dv summed over the GQA group when given per query head, written as the
// pre-rotary [dq | dk | dv] row of the qkv data-gradient GEMM. New here: the LoRA input gradients
// dx_lo = s * (g . B) of q and v (solution/engine.py:1322-1326) as a per-token reduction in the
// same pass, rounded like the reference's fp16 GEMM and scale.
#include "common.cuh"
#include "profile.h"
#include "ops.h"

namespace ql {

constexpr int RANK = 16;

// 8 consecutive values of a 16-bit or fp32 row as floats, and back.
template <typename T>
__device__ __forceinline__ void ld8(const T* p, float* v) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = to_f<T>(h[j]);
  }
}
template <typename T>
__device__ __forceinline__ void st8(T* p, const float* v) {
  T h[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) h[j] = from_f<T>(v[j]);
  *reinterpret_cast<uint4*>(p) = *reinterpret_cast<const uint4*>(h);
}

constexpr int ROPE_MAXR = 16;  // tokens per CTA tile at most (the tensor-core fragments' rows)

// Tiles of `rows` tokens (at most 16, picked by the launcher so the tiles fill one balanced
// wave; tiles strided over the grid), WPR warps per token (rows x WPR <= 16). With LoRA, the
// tile's LoRA-B outputs lq / lv = x_lo . B^T are formed first on the tensor cores (mma.sync
// m16n8k16, fp32 accumulation; the tokens are rows 0 .. rows-1 of the A fragment), rounded to
// the 16-bit type into shared memory. Then the warps of a token take chunks of 8 consecutive
// positions d .. d+7 of the first half of a head together with their partners d + D/2 (16-byte
// loads and stores).
template <typename T, int WPR>
__global__ void __launch_bounds__(512) rope_fwd_kernel(RopeFwdC a, int rows) {
  pdl_enter();
  const int NW = rows * WPR;
  extern __shared__ __align__(16) uint8_t rope_smem[];
  const int HQ = a.HQ, HKV = a.HKV, D = a.D, HALF = D / 2;
  const int C = (HQ + 2 * HKV) * D, QD = HQ * D, VD = HKV * D, ld = QD + VD + 8;
  T* sL = reinterpret_cast<T*>(rope_smem);  // [rows][ld]: [lq | lv] of the tile's tokens
  const bool fq = a.lq == nullptr && a.xq != nullptr, fv = a.lv == nullptr && a.xv != nullptr;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rrow = warp / WPR, part = warp % WPR;
  const float s = a.lora_scale;
  const int cph = HALF / 8;                 // chunks per head
  const int rot_chunks = (HQ + HKV) * cph;  // q and k heads
  const int v_chunks = VD / 8;
  const int ntiles = (a.n + rows - 1) / rows;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    if (fq || fv) {
      const int g = lane >> 2, t = lane & 3;
      uint32_t aq[4] = {0u, 0u, 0u, 0u}, av[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int half = 0; half < 2; ++half) {  // fragment rows g and g + 8
        const int r = g + 8 * half;
        const int64_t tg = (int64_t)tile * rows + r;
        if (r < rows && tg < a.n) {
          if (fq) {
            const uint32_t* x = reinterpret_cast<const uint32_t*>(reinterpret_cast<const T*>(a.xq) + tg * RANK);
            aq[half] = x[t];
            aq[2 + half] = x[4 + t];
          }
          if (fv) {
            const uint32_t* x = reinterpret_cast<const uint32_t*>(reinterpret_cast<const T*>(a.xv) + tg * RANK);
            av[half] = x[t];
            av[2 + half] = x[4 + t];
          }
        }
      }
      // 8-column groups n0 = 8 (warp + NW j) of [q | v], RB at a time: the RB groups' B fragments
      // are loaded first (independent L2 reads in flight together), then multiplied
      constexpr int RB = 8;
      for (int j0 = 0; warp * 8 + j0 * 8 * NW < QD + VD; j0 += RB) {
        uint32_t b0[RB], b1[RB];
#pragma unroll
        for (int j = 0; j < RB; ++j) {
          const int n0 = warp * 8 + (j0 + j) * 8 * NW;
          const bool isq = n0 < QD;
          b0[j] = b1[j] = 0u;
          if (n0 < QD + VD && (isq ? fq : fv)) {
            const unsigned int* Bw = reinterpret_cast<const unsigned int*>(
                isq ? reinterpret_cast<const T*>(a.Bq) + (int64_t)(n0 + g) * RANK
                    : reinterpret_cast<const T*>(a.Bv) + (int64_t)(n0 - QD + g) * RANK);
            b0[j] = __ldg(Bw + t);
            b1[j] = __ldg(Bw + 4 + t);
          }
        }
#pragma unroll
        for (int j = 0; j < RB; ++j) {
          const int n0 = warp * 8 + (j0 + j) * 8 * NW;
          const bool isq = n0 < QD;
          if (n0 >= QD + VD || (isq ? !fq : !fv)) continue;
          float c[4] = {0.f, 0.f, 0.f, 0.f};
          mma16816<T>(c, isq ? aq : av, b0[j], b1[j]);
          if (g < rows) *reinterpret_cast<uint32_t*>(sL + g * ld + n0 + 2 * t) = pack_t2<T>(c[0], c[1]);
          if (g + 8 < rows)
            *reinterpret_cast<uint32_t*>(sL + (g + 8) * ld + n0 + 2 * t) = pack_t2<T>(c[2], c[3]);
        }
      }
      __syncthreads();
    }
    const int64_t tok = (int64_t)tile * rows + rrow;
    if (tok < a.n) {
      const T* row = reinterpret_cast<const T*>(a.qkv) + tok * C;
      const T* lrow = sL + rrow * ld;
      const int pos = a.pos[tok];
      const float* cs = a.cos + (int64_t)pos * HALF;
      const float* sn = a.sin + (int64_t)pos * HALF;
      for (int ch = part * 32 + lane; ch < rot_chunks; ch += 32 * WPR) {
        const int hh = ch / cph, d = (ch % cph) * 8;
        const bool is_q = hh < HQ;
        const int src = hh * D + d;
        float x1[8], x2[8], c[8], sv[8];
        ld8<T>(row + src, x1);
        ld8<T>(row + src + HALF, x2);
        ld8<float>(cs + d, c);
        ld8<float>(sn + d, sv);
        if (is_q && (a.lq != nullptr || fq)) {
          float l1[8], l2[8];
          if (a.lq != nullptr) {
            const T* lq = reinterpret_cast<const T*>(a.lq) + tok * QD;
            ld8<T>(lq + src, l1);
            ld8<T>(lq + src + HALF, l2);
          } else {
            ld8<T>(lrow + src, l1);
            ld8<T>(lrow + src + HALF, l2);
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) { x1[j] += l1[j] * s; x2[j] += l2[j] * s; }
        }
        float o1[8], o2[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          o1[j] = x1[j] * c[j] - x2[j] * sv[j];
          o2[j] = x2[j] * c[j] + x1[j] * sv[j];
        }
        T* out = is_q ? reinterpret_cast<T*>(a.q) + tok * QD + hh * D
                      : reinterpret_cast<T*>(a.k) + tok * VD + (hh - HQ) * D;
        st8<T>(out + d, o1);
        st8<T>(out + d + HALF, o2);
      }
      for (int ch = part * 32 + lane; ch < v_chunks; ch += 32 * WPR) {
        const int idx = ch * 8;
        float v[8];
        ld8<T>(row + (HQ + HKV) * D + idx, v);
        if (a.lv != nullptr || fv) {
          float l[8];
          if (a.lv != nullptr) ld8<T>(reinterpret_cast<const T*>(a.lv) + tok * VD + idx, l);
          else ld8<T>(lrow + QD + idx, l);
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] += l[j] * s;
        }
        st8<T>(reinterpret_cast<T*>(a.v) + tok * VD + idx, v);
      }
    }
    __syncthreads();  // sL is refilled by the next tile
  }
}

// Backward, tiles of `rows` tokens (as the forward), WPR warps per token: the rotation pass
// writes the pre-rotary gradient row and keeps its q and v parts (16-bit) in shared memory; then
// dx_lo[rows][16] = g[rows][K] . B[K][16] on the tensor cores over K slices of 64 columns of
// [q | v] strided over the warps, the slices' partials added in a fixed order.
template <typename T, typename TIn, int WPR>
__global__ void __launch_bounds__(512) rope_bwd_kernel(RopeBwdC a, int rows) {
  pdl_enter();
  const int NW = rows * WPR;
  extern __shared__ __align__(16) uint8_t rope_smem[];
  const int HQ = a.HQ, HKV = a.HKV, D = a.D, HALF = D / 2;
  const int C = (HQ + 2 * HKV) * D, QD = HQ * D, VD = HKV * D, ld = QD + VD + 8;
  const int KVIN = a.kv_heads_in;  // HKV, or HQ (per query head: summed over the group)
  const int group = KVIN / HKV;
  T* sG = reinterpret_cast<T*>(rope_smem);                   // [rows][ld] [g_q | g_v]
  float* sRed = reinterpret_cast<float*>(sG + rows * ld);     // [NW][2][16][16]
  const bool lq = a.dxlo_q != nullptr, lv = a.dxlo_v != nullptr;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rrow = warp / WPR, part = warp % WPR;
  const int cph = HALF / 8;
  const int rot_chunks = (HQ + HKV) * cph;
  const int v_chunks = VD / 8;
  const int ntiles = (a.n + rows - 1) / rows;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int64_t tok = (int64_t)tile * rows + rrow;
    T* grow = sG + rrow * ld;
    if (tok < a.n) {
      const int pos = a.pos[tok];
      const float* cs = a.cos + (int64_t)pos * HALF;
      const float* sn = a.sin + (int64_t)pos * HALF;
      const TIn* dq = reinterpret_cast<const TIn*>(a.dq) + tok * QD;
      const TIn* dk = reinterpret_cast<const TIn*>(a.dk) + tok * KVIN * D;
      const TIn* dv = reinterpret_cast<const TIn*>(a.dv) + tok * KVIN * D;
      T* out = reinterpret_cast<T*>(a.dqkv) + tok * C;
      for (int ch = part * 32 + lane; ch < rot_chunks; ch += 32 * WPR) {
        const int hh = ch / cph, d = (ch % cph) * 8;
        float g1[8], g2[8], c[8], sv[8];
        if (hh < HQ) {
          ld8<TIn>(dq + hh * D + d, g1);
          ld8<TIn>(dq + hh * D + d + HALF, g2);
        } else {
          const int j = hh - HQ;
#pragma unroll
          for (int t = 0; t < 8; ++t) g1[t] = g2[t] = 0.f;
          for (int r = 0; r < group; ++r) {
            float t1[8], t2[8];
            ld8<TIn>(dk + (j * group + r) * D + d, t1);
            ld8<TIn>(dk + (j * group + r) * D + d + HALF, t2);
#pragma unroll
            for (int t = 0; t < 8; ++t) { g1[t] += t1[t]; g2[t] += t2[t]; }
          }
        }
        ld8<float>(cs + d, c);
        ld8<float>(sn + d, sv);
        float o1[8], o2[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          o1[t] = g1[t] * c[t] + g2[t] * sv[t];
          o2[t] = g2[t] * c[t] - g1[t] * sv[t];
        }
        const int col = hh * D + d;
        st8<T>(out + col, o1);
        st8<T>(out + col + HALF, o2);
        if (hh < HQ && lq) {
          st8<T>(grow + col, o1);
          st8<T>(grow + col + HALF, o2);
        }
      }
      for (int ch = part * 32 + lane; ch < v_chunks; ch += 32 * WPR) {
        const int idx = ch * 8, j = idx / D, d = idx % D;
        float g[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) g[t] = 0.f;
        for (int r = 0; r < group; ++r) {
          float t1[8];
          ld8<TIn>(dv + (j * group + r) * D + d, t1);
#pragma unroll
          for (int t = 0; t < 8; ++t) g[t] += t1[t];
        }
        st8<T>(out + (HQ + HKV) * D + idx, g);
        if (lv) st8<T>(grow + QD + idx, g);
      }
    }
    if (lq || lv) {
      __syncthreads();
      const int g = lane >> 2, t = lane & 3;
      float accq[2][4] = {}, accv[2][4] = {};  // [n tile][fragment] per adapter
      for (int k0 = warp * 64; k0 < QD + VD; k0 += 64 * NW) {
        const bool isq = k0 < QD;
        if (isq ? !lq : !lv) continue;
        const unsigned short* B = reinterpret_cast<const unsigned short*>(isq ? a.Bq : a.Bv) +
                                  (int64_t)(isq ? k0 : k0 - QD) * RANK;
#pragma unroll
        for (int kk = 0; kk < 64; kk += 16) {
          const T* Y0 = sG + g * ld + k0 + kk + 2 * t;
          const T* Y1 = Y0 + 8 * ld;
          const uint32_t af[4] = {g < rows ? *reinterpret_cast<const uint32_t*>(Y0) : 0u,
                                  g + 8 < rows ? *reinterpret_cast<const uint32_t*>(Y1) : 0u,
                                  g < rows ? *reinterpret_cast<const uint32_t*>(Y0 + 8) : 0u,
                                  g + 8 < rows ? *reinterpret_cast<const uint32_t*>(Y1 + 8) : 0u};
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const unsigned short* bp = B + (kk + 2 * t) * RANK + nt * 8 + g;
            const uint32_t b0 = (uint32_t)__ldg(bp) | ((uint32_t)__ldg(bp + RANK) << 16);
            const uint32_t b1 = (uint32_t)__ldg(bp + 8 * RANK) | ((uint32_t)__ldg(bp + 9 * RANK) << 16);
            if (isq) mma16816<T>(accq[nt], af, b0, b1);
            else mma16816<T>(accv[nt], af, b0, b1);
          }
        }
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        float* rq = sRed + ((warp * 2 + 0) * ROPE_MAXR + g) * RANK + nt * 8 + 2 * t;
        float* rv = sRed + ((warp * 2 + 1) * ROPE_MAXR + g) * RANK + nt * 8 + 2 * t;
        rq[0] = accq[nt][0];
        rq[1] = accq[nt][1];
        rq[8 * RANK] = accq[nt][2];
        rq[8 * RANK + 1] = accq[nt][3];
        rv[0] = accv[nt][0];
        rv[1] = accv[nt][1];
        rv[8 * RANK] = accv[nt][2];
        rv[8 * RANK + 1] = accv[nt][3];
      }
      __syncthreads();
      for (int idx = threadIdx.x; idx < 2 * rows * RANK; idx += blockDim.x) {
        const int ad = idx / (rows * RANK), rr = (idx / RANK) % rows, r = idx % RANK;
        const int64_t orow = (int64_t)tile * rows + rr;
        if (orow < a.n && (ad == 0 ? lq : lv)) {
          float sum = 0.f;
          for (int w = 0; w < NW; ++w) sum += sRed[((w * 2 + ad) * ROPE_MAXR + rr) * RANK + r];
          // (g @ B) rounded to the 16-bit type, then * s rounded again (fp16 tensor times a scalar)
          const float v = to_f<T>(from_f<T>(to_f<T>(from_f<T>(sum)) * a.lora_scale));
          (ad == 0 ? a.dxlo_q : a.dxlo_v)[orow * RANK + r] = v;
        }
      }
    }
    __syncthreads();  // sG and sRed are refilled by the next tile
  }
}

// Launch shape: tokens per tile balanced so the tiles fill whole waves of one CTA per SM (up to
// 16 tokens per tile), two warps per token for up to 8 tokens per tile, else one.
struct RopeShape {
  int wpr, rows, grid;
};

static RopeShape rope_shape(int64_t n) {
  const int sms = sm_count();
  const int64_t waves = cdiv(n, (int64_t)sms * ROPE_MAXR);
  RopeShape r;
  if (waves > 1) {
    // more rows than one wave of 16-row tiles: 8-row tiles of one warp per token (256 threads),
    // two CTAs resident per SM, so one CTA's loads overlap the other's arithmetic
    r.rows = 8;
    r.wpr = 1;
  } else {
    r.rows = (int)cdiv(n, (int64_t)sms * waves);
    r.wpr = r.rows <= 8 ? 2 : 1;
  }
  r.grid = (int)cdiv(n, r.rows);
  return r;
}

// Opts a kernel into more than 48 KB of dynamic shared memory, once per kernel (and size).
template <typename K>
static void rope_smem_attr(K kern, int bytes) {
  if (bytes > 48 * 1024) smem_optin(reinterpret_cast<const void*>(kern), bytes);
}

int rope_fwd(const RopeFwdC& a, cudaStream_t s) {
  if (a.n < 0 || a.D % 16 != 0 || a.HKV <= 0 || a.HQ % a.HKV != 0) return QL_STATUS_BAD_ARG;
  if (a.n == 0) return QL_STATUS_OK;
  if ((a.xq != nullptr && a.Bq == nullptr) || (a.xv != nullptr && a.Bv == nullptr)) return QL_STATUS_BAD_ARG;
  if ((a.xq != nullptr || a.xv != nullptr) && a.rank != RANK) return QL_STATUS_UNSUPPORTED;
  ProfScope prof(PK_ROPE_FWD, 0, (double)a.n * (a.HQ + 2 * a.HKV) * a.D * 2 * 2, s);
  const bool lora = (a.lq == nullptr && a.xq != nullptr) || (a.lv == nullptr && a.xv != nullptr);
  const RopeShape sh = rope_shape(a.n);
  const int smem = lora ? sh.rows * ((a.HQ + a.HKV) * a.D + 8) * 2 : 0;
#define QL_ROPEF(TT, WW)                                                                  \
  do {                                                                                    \
    rope_smem_attr(rope_fwd_kernel<TT, WW>, smem);                                        \
    launch_k(rope_fwd_kernel<TT, WW>, dim3(sh.grid), dim3(32 * WW * sh.rows), smem, s, a, sh.rows); \
  } while (0)
  if (a.dtype == QL_F16) {
    if (sh.wpr == 2) QL_ROPEF(__half, 2); else QL_ROPEF(__half, 1);
  } else if (a.dtype == QL_BF16) {
    if (sh.wpr == 2) QL_ROPEF(__nv_bfloat16, 2); else QL_ROPEF(__nv_bfloat16, 1);
  } else {
    return QL_STATUS_BAD_ARG;
  }
#undef QL_ROPEF
  return launched(1);
}

int rope_bwd(const RopeBwdC& a, cudaStream_t s) {
  if (a.n < 0 || a.D % 16 != 0 || a.HKV <= 0 || a.HQ % a.HKV != 0) return QL_STATUS_BAD_ARG;
  if (a.kv_heads_in != a.HKV && a.kv_heads_in != a.HQ) return QL_STATUS_BAD_ARG;
  if (a.n == 0) return QL_STATUS_OK;
  if ((a.dxlo_q != nullptr && a.Bq == nullptr) || (a.dxlo_v != nullptr && a.Bv == nullptr)) return QL_STATUS_BAD_ARG;
  if ((a.dxlo_q != nullptr || a.dxlo_v != nullptr) && a.rank != RANK) return QL_STATUS_UNSUPPORTED;
  const bool f32in = a.grad_dtype == QL_F32;
  if (a.grad_dtype != QL_F32 && a.grad_dtype != a.dtype) return QL_STATUS_BAD_ARG;
  ProfScope prof(PK_ROPE_BWD, 0, (double)a.n * (a.HQ + 2 * a.HKV) * a.D * (4 + 2), s);
  const bool lora = a.dxlo_q != nullptr || a.dxlo_v != nullptr;
  if (lora && a.D % 64 != 0) return QL_STATUS_UNSUPPORTED;  // 64-column K slices of [q | v]
  const RopeShape sh = rope_shape(a.n);
  const int smem = lora ? sh.rows * ((a.HQ + a.HKV) * a.D + 8) * 2 +
                              sh.rows * sh.wpr * 2 * ROPE_MAXR * RANK * 4
                        : 0;
#define QL_ROPEB(TT, TI)                                                                      \
  do {                                                                                        \
    if (sh.wpr == 2) {                                                                        \
      rope_smem_attr(rope_bwd_kernel<TT, TI, 2>, smem);                                       \
      launch_k(rope_bwd_kernel<TT, TI, 2>, dim3(sh.grid), dim3(64 * sh.rows), smem, s, a, sh.rows); \
    } else {                                                                                  \
      rope_smem_attr(rope_bwd_kernel<TT, TI, 1>, smem);                                       \
      launch_k(rope_bwd_kernel<TT, TI, 1>, dim3(sh.grid), dim3(32 * sh.rows), smem, s, a, sh.rows); \
    }                                                                                         \
  } while (0)
  if (a.dtype == QL_F16) {
    if (f32in) QL_ROPEB(__half, float); else QL_ROPEB(__half, __half);
  } else if (a.dtype == QL_BF16) {
    if (f32in) QL_ROPEB(__nv_bfloat16, float); else QL_ROPEB(__nv_bfloat16, __nv_bfloat16);
  } else {
    return QL_STATUS_BAD_ARG;
  }
#undef QL_ROPEB
  return launched(1);
}

}  // namespace ql
