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

// One warp per token (8 per CTA, tokens strided over the grid); the LoRA-B factors (rows of 16)
// are staged in shared memory once per CTA.
template <typename T>
__global__ void __launch_bounds__(256) rope_fwd_kernel(RopeFwdC a) {
  extern __shared__ __align__(16) uint8_t rope_smem[];
  const int HQ = a.HQ, HKV = a.HKV, D = a.D, HALF = D / 2;
  const int C = (HQ + 2 * HKV) * D;
  T* sBq = reinterpret_cast<T*>(rope_smem);
  T* sBv = sBq + (int64_t)HQ * D * RANK;
  const bool fq = a.lq == nullptr && a.xq != nullptr, fv = a.lv == nullptr && a.xv != nullptr;
  if (fq || fv) {
    for (int i = threadIdx.x; i < HQ * D * RANK / 8; i += blockDim.x)
      if (fq) reinterpret_cast<uint4*>(sBq)[i] = reinterpret_cast<const uint4*>(a.Bq)[i];
    for (int i = threadIdx.x; i < HKV * D * RANK / 8; i += blockDim.x)
      if (fv) reinterpret_cast<uint4*>(sBv)[i] = reinterpret_cast<const uint4*>(a.Bv)[i];
    __syncthreads();
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float s = a.lora_scale;
  for (int64_t tok = blockIdx.x * 8 + warp; tok < a.n; tok += (int64_t)gridDim.x * 8) {
    const T* row = reinterpret_cast<const T*>(a.qkv) + tok * C;
    // this token's LoRA-A outputs, broadcast from lanes 0..15 (q) and 16..31 (v)
    float mine = 0.f;
    if (lane < RANK) { if (fq) mine = to_f<T>(reinterpret_cast<const T*>(a.xq)[tok * RANK + lane]); }
    else if (fv) mine = to_f<T>(reinterpret_cast<const T*>(a.xv)[tok * RANK + lane - RANK]);
    float xl[2 * RANK];
#pragma unroll
    for (int r = 0; r < 2 * RANK; ++r) xl[r] = __shfl_sync(0xffffffffu, mine, r);
    const int pos = a.pos[tok];
    const float* cs = a.cos + (int64_t)pos * HALF;
    const float* sn = a.sin + (int64_t)pos * HALF;
    auto lora_b = [&](const T* B, const float* x, int idx) -> float {  // rounded like a GEMM output
      const uint4* b4 = reinterpret_cast<const uint4*>(B + (int64_t)idx * RANK);
      const uint4 u0 = b4[0], u1 = b4[1];
      const T* b0 = reinterpret_cast<const T*>(&u0);
      const T* b1 = reinterpret_cast<const T*>(&u1);
      float acc = 0.f;
#pragma unroll
      for (int r = 0; r < 8; ++r) acc += x[r] * to_f<T>(b0[r]);
#pragma unroll
      for (int r = 0; r < 8; ++r) acc += x[8 + r] * to_f<T>(b1[r]);
      return to_f<T>(from_f<T>(acc));
    };
    for (int idx = lane; idx < (HQ + HKV) * HALF; idx += 32) {
      const int hh = idx / HALF, d = idx % HALF;
      const bool is_q = hh < HQ;
      const int src = hh * D + d;
      float x1 = to_f<T>(row[src]), x2 = to_f<T>(row[src + HALF]);
      if (is_q) {
        if (a.lq != nullptr) {
          const T* lq = reinterpret_cast<const T*>(a.lq) + tok * HQ * D;
          x1 += to_f<T>(lq[src]) * s;
          x2 += to_f<T>(lq[src + HALF]) * s;
        } else if (fq) {
          x1 += lora_b(sBq, xl, src) * s;
          x2 += lora_b(sBq, xl, src + HALF) * s;
        }
      }
      const float c = cs[d], sv = sn[d];
      T* out = is_q ? reinterpret_cast<T*>(a.q) + tok * HQ * D + hh * D
                    : reinterpret_cast<T*>(a.k) + tok * HKV * D + (hh - HQ) * D;
      out[d] = from_f<T>(x1 * c - x2 * sv);
      out[d + HALF] = from_f<T>(x2 * c + x1 * sv);
    }
    for (int idx = lane; idx < HKV * D; idx += 32) {
      float v = to_f<T>(row[(HQ + HKV) * D + idx]);
      if (a.lv != nullptr) v += to_f<T>(reinterpret_cast<const T*>(a.lv)[tok * HKV * D + idx]) * s;
      else if (fv) v += lora_b(sBv, xl + RANK, idx) * s;
      reinterpret_cast<T*>(a.v)[tok * HKV * D + idx] = from_f<T>(v);
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
    for (int i = threadIdx.x; i < HQ * D * RANK / 8; i += blockDim.x)
      if (lq) reinterpret_cast<uint4*>(sBq)[i] = reinterpret_cast<const uint4*>(a.Bq)[i];
    for (int i = threadIdx.x; i < HKV * D * RANK / 8; i += blockDim.x)
      if (lv) reinterpret_cast<uint4*>(sBv)[i] = reinterpret_cast<const uint4*>(a.Bv)[i];
    __syncthreads();
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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
    auto accum = [&](const T* B, int idx, float g, int off) {
      const uint4* b4 = reinterpret_cast<const uint4*>(B + (int64_t)idx * RANK);
      const uint4 u0 = b4[0], u1 = b4[1];
      const T* b0 = reinterpret_cast<const T*>(&u0);
      const T* b1 = reinterpret_cast<const T*>(&u1);
#pragma unroll
      for (int r = 0; r < 8; ++r) acc[off + r] += g * to_f<T>(b0[r]);
#pragma unroll
      for (int r = 0; r < 8; ++r) acc[off + 8 + r] += g * to_f<T>(b1[r]);
    };
    for (int idx = lane; idx < (HQ + HKV) * HALF; idx += 32) {
      const int hh = idx / HALF, d = idx % HALF;
      float g1 = 0.f, g2 = 0.f;
      if (hh < HQ) {
        g1 = to_f<TIn>(dq[hh * D + d]);
        g2 = to_f<TIn>(dq[hh * D + d + HALF]);
      } else {
        const int j = hh - HQ;
        for (int r = 0; r < group; ++r) {
          g1 += to_f<TIn>(dk[(j * group + r) * D + d]);
          g2 += to_f<TIn>(dk[(j * group + r) * D + d + HALF]);
        }
      }
      const float c = cs[d], sv = sn[d];
      const T o1 = from_f<T>(g1 * c + g2 * sv), o2 = from_f<T>(g2 * c - g1 * sv);
      const int col = hh * D + d;
      out[col] = o1;
      out[col + HALF] = o2;
      if (hh < HQ && lq) {
        accum(sBq, col, to_f<T>(o1), 0);
        accum(sBq, col + HALF, to_f<T>(o2), 0);
      }
    }
    for (int idx = lane; idx < HKV * D; idx += 32) {
      const int j = idx / D, d = idx % D;
      float g = 0.f;
      for (int r = 0; r < group; ++r) g += to_f<TIn>(dv[(j * group + r) * D + d]);
      const T o = from_f<T>(g);
      out[(HQ + HKV) * D + idx] = o;
      if (lv) accum(sBv, idx, to_f<T>(o), RANK);
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

// Opts a kernel into more than 48 KB of dynamic shared memory, once per kernel.
template <typename K>
static void rope_smem_attr(K kern, int bytes) {
  static int done = 0;  // one flag per kernel instantiation
  if (bytes > 48 * 1024 && bytes > done) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    done = bytes;
  }
}

int rope_fwd(const RopeFwdC& a, cudaStream_t s) {
  if (a.n < 0 || a.D % 2 != 0 || a.HKV <= 0 || a.HQ % a.HKV != 0) return QL_STATUS_BAD_ARG;
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
  if (a.n < 0 || a.D % 2 != 0 || a.HKV <= 0 || a.HQ % a.HKV != 0) return QL_STATUS_BAD_ARG;
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
