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
#include "ops.h"

namespace ql {

constexpr int ROPE_THREADS = 128;
constexpr int RANK = 16;

template <typename T>
__global__ void __launch_bounds__(ROPE_THREADS) rope_fwd_kernel(RopeFwdC a) {
  __shared__ float xq[RANK], xv[RANK];
  const int64_t tok = blockIdx.x;
  const int HQ = a.HQ, HKV = a.HKV, D = a.D, HALF = D / 2;
  const int C = (HQ + 2 * HKV) * D;
  const T* row = reinterpret_cast<const T*>(a.qkv) + tok * C;
  const bool lora_q = a.lq != nullptr || a.xq != nullptr;
  const bool lora_v = a.lv != nullptr || a.xv != nullptr;
  if (threadIdx.x < RANK) {
    xq[threadIdx.x] = a.xq != nullptr ? to_f<T>(reinterpret_cast<const T*>(a.xq)[tok * RANK + threadIdx.x]) : 0.f;
    xv[threadIdx.x] = a.xv != nullptr ? to_f<T>(reinterpret_cast<const T*>(a.xv)[tok * RANK + threadIdx.x]) : 0.f;
  }
  __syncthreads();
  const int pos = a.pos[tok];
  const float* cs = a.cos + (int64_t)pos * HALF;
  const float* sn = a.sin + (int64_t)pos * HALF;
  const float s = a.lora_scale;

  auto lora_val = [&](bool on, const void* explicit_, const void* Bmat, const float* x, int ld,
                      int idx) -> float {
    if (!on) return 0.f;
    if (explicit_ != nullptr) return to_f<T>(reinterpret_cast<const T*>(explicit_)[tok * ld + idx]);
    const T* b = reinterpret_cast<const T*>(Bmat) + (int64_t)idx * RANK;
    float acc = 0.f;
#pragma unroll
    for (int r = 0; r < RANK; ++r) acc += x[r] * to_f<T>(b[r]);
    return to_f<T>(from_f<T>(acc));
  };

  // q and k pairs: index over (HQ + HKV) heads x HALF
  for (int idx = threadIdx.x; idx < (HQ + HKV) * HALF; idx += ROPE_THREADS) {
    const int hh = idx / HALF, d = idx % HALF;
    const bool is_q = hh < HQ;
    const int src = hh * D + d;  // column in the qkv row (q heads then k heads)
    float x1 = to_f<T>(row[src]), x2 = to_f<T>(row[src + HALF]);
    if (is_q && lora_q) {
      x1 += lora_val(true, a.lq, a.Bq, xq, HQ * D, src) * s;
      x2 += lora_val(true, a.lq, a.Bq, xq, HQ * D, src + HALF) * s;
    }
    const float c = cs[d], sv = sn[d];
    T* out = is_q ? reinterpret_cast<T*>(a.q) + tok * HQ * D + hh * D
                  : reinterpret_cast<T*>(a.k) + tok * HKV * D + (hh - HQ) * D;
    out[d] = from_f<T>(x1 * c - x2 * sv);
    out[d + HALF] = from_f<T>(x2 * c + x1 * sv);
  }
  for (int idx = threadIdx.x; idx < HKV * D; idx += ROPE_THREADS) {
    float v = to_f<T>(row[(HQ + HKV) * D + idx]);
    if (lora_v) v += lora_val(true, a.lv, a.Bv, xv, HKV * D, idx) * s;
    reinterpret_cast<T*>(a.v)[tok * HKV * D + idx] = from_f<T>(v);
  }
}

template <typename T, typename TIn>
__global__ void __launch_bounds__(ROPE_THREADS) rope_bwd_kernel(RopeBwdC a) {
  __shared__ float scratch[4][2 * RANK];
  const int64_t tok = blockIdx.x;
  const int HQ = a.HQ, HKV = a.HKV, D = a.D, HALF = D / 2;
  const int C = (HQ + 2 * HKV) * D;
  const int KVIN = a.kv_heads_in;  // HKV, or HQ (per query head: summed over the group)
  const int group = KVIN / HKV;
  const int pos = a.pos[tok];
  const float* cs = a.cos + (int64_t)pos * HALF;
  const float* sn = a.sin + (int64_t)pos * HALF;
  const TIn* dq = reinterpret_cast<const TIn*>(a.dq) + tok * HQ * D;
  const TIn* dk = reinterpret_cast<const TIn*>(a.dk) + tok * KVIN * D;
  const TIn* dv = reinterpret_cast<const TIn*>(a.dv) + tok * KVIN * D;
  T* out = reinterpret_cast<T*>(a.dqkv) + tok * C;
  const bool lq = a.dxlo_q != nullptr, lv = a.dxlo_v != nullptr;
  float accq[RANK], accv[RANK];
#pragma unroll
  for (int r = 0; r < RANK; ++r) accq[r] = accv[r] = 0.f;

  for (int idx = threadIdx.x; idx < (HQ + HKV) * HALF; idx += ROPE_THREADS) {
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
      const T* b1 = reinterpret_cast<const T*>(a.Bq) + (int64_t)col * RANK;
      const T* b2 = b1 + (int64_t)HALF * RANK;
      const float f1 = to_f<T>(o1), f2 = to_f<T>(o2);
#pragma unroll
      for (int r = 0; r < RANK; ++r) accq[r] += f1 * to_f<T>(b1[r]) + f2 * to_f<T>(b2[r]);
    }
  }
  for (int idx = threadIdx.x; idx < HKV * D; idx += ROPE_THREADS) {
    const int j = idx / D, d = idx % D;
    float g = 0.f;
    for (int r = 0; r < group; ++r) g += to_f<TIn>(dv[(j * group + r) * D + d]);
    const T o = from_f<T>(g);
    out[(HQ + HKV) * D + idx] = o;
    if (lv) {
      const T* b = reinterpret_cast<const T*>(a.Bv) + (int64_t)idx * RANK;
      const float f = to_f<T>(o);
#pragma unroll
      for (int r = 0; r < RANK; ++r) accv[r] += f * to_f<T>(b[r]);
    }
  }
  if (lq || lv) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < RANK; ++r) {
      accq[r] = warp_sum(accq[r]);
      accv[r] = warp_sum(accv[r]);
    }
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < RANK; ++r) {
        scratch[warp][r] = accq[r];
        scratch[warp][RANK + r] = accv[r];
      }
    }
    __syncthreads();
    if (threadIdx.x < 2 * RANK) {
      const int i = threadIdx.x;
      const float sum = scratch[0][i] + scratch[1][i] + scratch[2][i] + scratch[3][i];
      // (g @ B) rounded to the 16-bit type, then * s rounded again (fp16 tensor times a scalar)
      const float v = to_f<T>(from_f<T>(to_f<T>(from_f<T>(sum)) * a.lora_scale));
      if (i < RANK) {
        if (lq) a.dxlo_q[tok * RANK + i] = v;
      } else if (lv) {
        a.dxlo_v[tok * RANK + i - RANK] = v;
      }
    }
  }
}

int rope_fwd(const RopeFwdC& a, cudaStream_t s) {
  if (a.n < 0 || a.D % 2 != 0 || a.HKV <= 0 || a.HQ % a.HKV != 0) return QL_STATUS_BAD_ARG;
  if (a.n == 0) return QL_STATUS_OK;
  if ((a.xq != nullptr && a.Bq == nullptr) || (a.xv != nullptr && a.Bv == nullptr)) return QL_STATUS_BAD_ARG;
  if ((a.xq != nullptr || a.xv != nullptr) && a.rank != RANK) return QL_STATUS_UNSUPPORTED;
  if (a.dtype == QL_F16) rope_fwd_kernel<__half><<<a.n, ROPE_THREADS, 0, s>>>(a);
  else if (a.dtype == QL_BF16) rope_fwd_kernel<__nv_bfloat16><<<a.n, ROPE_THREADS, 0, s>>>(a);
  else return QL_STATUS_BAD_ARG;
  return cudaPeekAtLastError() == cudaSuccess ? QL_STATUS_OK : QL_STATUS_CUDA;
}

int rope_bwd(const RopeBwdC& a, cudaStream_t s) {
  if (a.n < 0 || a.D % 2 != 0 || a.HKV <= 0 || a.HQ % a.HKV != 0) return QL_STATUS_BAD_ARG;
  if (a.kv_heads_in != a.HKV && a.kv_heads_in != a.HQ) return QL_STATUS_BAD_ARG;
  if (a.n == 0) return QL_STATUS_OK;
  if ((a.dxlo_q != nullptr && a.Bq == nullptr) || (a.dxlo_v != nullptr && a.Bv == nullptr)) return QL_STATUS_BAD_ARG;
  if ((a.dxlo_q != nullptr || a.dxlo_v != nullptr) && a.rank != RANK) return QL_STATUS_UNSUPPORTED;
  const bool f32in = a.grad_dtype == QL_F32;
  if (a.grad_dtype != QL_F32 && a.grad_dtype != a.dtype) return QL_STATUS_BAD_ARG;
  if (a.dtype == QL_F16) {
    if (f32in) rope_bwd_kernel<__half, float><<<a.n, ROPE_THREADS, 0, s>>>(a);
    else rope_bwd_kernel<__half, __half><<<a.n, ROPE_THREADS, 0, s>>>(a);
  } else if (a.dtype == QL_BF16) {
    if (f32in) rope_bwd_kernel<__nv_bfloat16, float><<<a.n, ROPE_THREADS, 0, s>>>(a);
    else rope_bwd_kernel<__nv_bfloat16, __nv_bfloat16><<<a.n, ROPE_THREADS, 0, s>>>(a);
  } else {
    return QL_STATUS_BAD_ARG;
  }
  return cudaPeekAtLastError() == cudaSuccess ? QL_STATUS_OK : QL_STATUS_CUDA;
}

}  // namespace ql
