// qkv + LoRA + rotary embedding, forward and backward, one CTA per token.
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

// lo[j] = sum_r x[r] B[idx + j][r] for 8 consecutive rows of a [rows, 16] factor in smem,
// rounded to the 16-bit type (the reference's fp16 GEMM output).
template <typename T>
__device__ __forceinline__ void lora_rows8(const T* B, int idx, const float* x, float* lo) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint4* b4 = reinterpret_cast<const uint4*>(B + (int64_t)(idx + j) * RANK);
    const uint4 u0 = b4[0], u1 = b4[1];
    const T* b0 = reinterpret_cast<const T*>(&u0);
    const T* b1 = reinterpret_cast<const T*>(&u1);
    float acc = 0.f;
#pragma unroll
    for (int r = 0; r < 8; ++r) acc += x[r] * to_f<T>(b0[r]);
#pragma unroll
    for (int r = 0; r < 8; ++r) acc += x[8 + r] * to_f<T>(b1[r]);
    lo[j] = to_f<T>(from_f<T>(acc));
  }
}

// One warp per token (8 per CTA, tokens strided over the grid). A lane takes chunks of 8
// consecutive positions d .. d+7 of the first half of a head together with their partners
// d + D/2 (16-byte loads and stores); the LoRA-B factors sit in shared memory.
template <typename T>
__global__ void __launch_bounds__(256) rope_fwd_kernel(RopeFwdC a) {
  extern __shared__ __align__(16) uint8_t rope_smem[];
  const int HQ = a.HQ, HKV = a.HKV, D = a.D, HALF = D / 2;
  const int C = (HQ + 2 * HKV) * D;
  T* sBq = reinterpret_cast<T*>(rope_smem);
  T* sBv = sBq + (int64_t)HQ * D * RANK;
  const bool fq = a.lq == nullptr && a.xq != nullptr, fv = a.lv == nullptr && a.xv != nullptr;
  if (fq || fv) {
    if (fq) stage_to_smem(sBq, a.Bq, HQ * D * RANK * (int)sizeof(T));
    if (fv) stage_to_smem(sBv, a.Bv, HKV * D * RANK * (int)sizeof(T));
    stage_wait();
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float s = a.lora_scale;
  const int cph = HALF / 8;                 // chunks per head
  const int rot_chunks = (HQ + HKV) * cph;  // q and k heads
  const int v_chunks = HKV * D / 8;
  for (int64_t tok = blockIdx.x * 8 + warp; tok < a.n; tok += (int64_t)gridDim.x * 8) {
    const T* row = reinterpret_cast<const T*>(a.qkv) + tok * C;
    float mine = 0.f;
    if (lane < RANK) { if (fq) mine = to_f<T>(reinterpret_cast<const T*>(a.xq)[tok * RANK + lane]); }
    else if (fv) mine = to_f<T>(reinterpret_cast<const T*>(a.xv)[tok * RANK + lane - RANK]);
    float xl[2 * RANK];
#pragma unroll
    for (int r = 0; r < 2 * RANK; ++r) xl[r] = __shfl_sync(0xffffffffu, mine, r);
    const int pos = a.pos[tok];
    const float* cs = a.cos + (int64_t)pos * HALF;
    const float* sn = a.sin + (int64_t)pos * HALF;
#pragma unroll 2
    for (int ch = lane; ch < rot_chunks; ch += 32) {
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
          const T* lq = reinterpret_cast<const T*>(a.lq) + tok * HQ * D;
          ld8<T>(lq + src, l1);
          ld8<T>(lq + src + HALF, l2);
        } else {
          lora_rows8<T>(sBq, src, xl, l1);
          lora_rows8<T>(sBq, src + HALF, xl, l2);
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
      T* out = is_q ? reinterpret_cast<T*>(a.q) + tok * HQ * D + hh * D
                    : reinterpret_cast<T*>(a.k) + tok * HKV * D + (hh - HQ) * D;
      st8<T>(out + d, o1);
      st8<T>(out + d + HALF, o2);
    }
    for (int ch = lane; ch < v_chunks; ch += 32) {
      const int idx = ch * 8;
      float v[8];
      ld8<T>(row + (HQ + HKV) * D + idx, v);
      if (a.lv != nullptr || fv) {
        float l[8];
        if (a.lv != nullptr) ld8<T>(reinterpret_cast<const T*>(a.lv) + tok * HKV * D + idx, l);
        else lora_rows8<T>(sBv, idx, xl + RANK, l);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] += l[j] * s;
      }
      st8<T>(reinterpret_cast<T*>(a.v) + tok * HKV * D + idx, v);
    }
  }
}

// Sum over the warp of 32 per-lane values; afterwards lane l holds the total of value l.
__device__ __forceinline__ float rs32(float* v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float send = upper ? v[i] : v[i + off];
      const float keep = upper ? v[i + off] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return v[0];
}

// acc[off + r] += sum_j g[j] B[idx + j][r] (8 consecutive rows of a [rows, 16] factor in smem)
template <typename T>
__device__ __forceinline__ void lora_acc8(const T* B, int idx, const float* g, float* acc, int off) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint4* b4 = reinterpret_cast<const uint4*>(B + (int64_t)(idx + j) * RANK);
    const uint4 u0 = b4[0], u1 = b4[1];
    const T* b0 = reinterpret_cast<const T*>(&u0);
    const T* b1 = reinterpret_cast<const T*>(&u1);
#pragma unroll
    for (int r = 0; r < 8; ++r) acc[off + r] += g[j] * to_f<T>(b0[r]);
#pragma unroll
    for (int r = 0; r < 8; ++r) acc[off + 8 + r] += g[j] * to_f<T>(b1[r]);
  }
}

template <typename T, typename TIn>
__global__ void __launch_bounds__(256) rope_bwd_kernel(RopeBwdC a) {
  extern __shared__ __align__(16) uint8_t rope_smem[];
  const int HQ = a.HQ, HKV = a.HKV, D = a.D, HALF = D / 2;
  const int C = (HQ + 2 * HKV) * D;
  const int KVIN = a.kv_heads_in;  // HKV, or HQ (per query head: summed over the group)
  const int group = KVIN / HKV;
  T* sBq = reinterpret_cast<T*>(rope_smem);
  T* sBv = sBq + (int64_t)HQ * D * RANK;
  const bool lq = a.dxlo_q != nullptr, lv = a.dxlo_v != nullptr;
  if (lq || lv) {
    if (lq) stage_to_smem(sBq, a.Bq, HQ * D * RANK * (int)sizeof(T));
    if (lv) stage_to_smem(sBv, a.Bv, HKV * D * RANK * (int)sizeof(T));
    stage_wait();
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cph = HALF / 8;
  const int rot_chunks = (HQ + HKV) * cph;
  const int v_chunks = HKV * D / 8;
  for (int64_t tok = blockIdx.x * 8 + warp; tok < a.n; tok += (int64_t)gridDim.x * 8) {
    const int pos = a.pos[tok];
    const float* cs = a.cos + (int64_t)pos * HALF;
    const float* sn = a.sin + (int64_t)pos * HALF;
    const TIn* dq = reinterpret_cast<const TIn*>(a.dq) + tok * HQ * D;
    const TIn* dk = reinterpret_cast<const TIn*>(a.dk) + tok * KVIN * D;
    const TIn* dv = reinterpret_cast<const TIn*>(a.dv) + tok * KVIN * D;
    T* out = reinterpret_cast<T*>(a.dqkv) + tok * C;
    float acc[2 * RANK];
#pragma unroll
    for (int r = 0; r < 2 * RANK; ++r) acc[r] = 0.f;
#pragma unroll 2
    for (int ch = lane; ch < rot_chunks; ch += 32) {
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
        o1[t] = to_f<T>(from_f<T>(g1[t] * c[t] + g2[t] * sv[t]));
        o2[t] = to_f<T>(from_f<T>(g2[t] * c[t] - g1[t] * sv[t]));
      }
      const int col = hh * D + d;
      st8<T>(out + col, o1);
      st8<T>(out + col + HALF, o2);
      if (hh < HQ && lq) {
        lora_acc8<T>(sBq, col, o1, acc, 0);
        lora_acc8<T>(sBq, col + HALF, o2, acc, 0);
      }
    }
    for (int ch = lane; ch < v_chunks; ch += 32) {
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
#pragma unroll
      for (int t = 0; t < 8; ++t) g[t] = to_f<T>(from_f<T>(g[t]));
      st8<T>(out + (HQ + HKV) * D + idx, g);
      if (lv) lora_acc8<T>(sBv, idx, g, acc, RANK);
    }
    if (lq || lv) {
      const float sum = rs32(acc);  // lane l: value l (q: 0..15, v: 16..31)
      // (g @ B) rounded to the 16-bit type, then * s rounded again (fp16 tensor times a scalar)
      const float v = to_f<T>(from_f<T>(to_f<T>(from_f<T>(sum)) * a.lora_scale));
      if (lane < RANK) {
        if (lq) a.dxlo_q[tok * RANK + lane] = v;
      } else if (lv) {
        a.dxlo_v[tok * RANK + lane - RANK] = v;
      }
    }
  }
}

static int rope_grid(int64_t n) {
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = cdiv(n, 8), cap = (int64_t)sms * 4;
  return (int)(want < cap ? want : cap);
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
  const int smem = lora ? (a.HQ + a.HKV) * a.D * RANK * 2 : 0;
  const int grid = rope_grid(a.n);
  if (a.dtype == QL_F16) {
    rope_smem_attr(rope_fwd_kernel<__half>, smem);
    rope_fwd_kernel<__half><<<grid, 256, smem, s>>>(a);
  } else if (a.dtype == QL_BF16) {
    rope_smem_attr(rope_fwd_kernel<__nv_bfloat16>, smem);
    rope_fwd_kernel<__nv_bfloat16><<<grid, 256, smem, s>>>(a);
  } else {
    return QL_STATUS_BAD_ARG;
  }
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
  const int smem = lora ? (a.HQ + a.HKV) * a.D * RANK * 2 : 0;
  const int grid = rope_grid(a.n);
#define QL_ROPEB(TT, TI)                                          \
  do {                                                            \
    rope_smem_attr(rope_bwd_kernel<TT, TI>, smem);                \
    rope_bwd_kernel<TT, TI><<<grid, 256, smem, s>>>(a);           \
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
