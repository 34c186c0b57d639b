// RMSNorm forward / backward with the LoRA dropout inputs fused in.
//
// Forward (reference rms_fwd_kernel, solution/kernels.py:145-175): optional residual add of a
// 16-bit delta to the fp32 residual (written back as xsum), rstd = 1 / sqrt(mean(x^2) + eps),
// y = w * (x * rstd) in fp32, stored in the 16-bit compute type; for each LoRA target (q, v) the
// dropped copy keep ? y * 1/(1-p) : 0 with PyTorch's own mask (philox.cuh). New here: the LoRA-A
// product x_lo = drop(y) . A^T ([n, R], R = 16) is formed in the same pass from the rounded
// dropped values (what the reference's separate fp16 GEMM reads, solution/engine.py:1088-1093).
//
// Backward (reference rms_bwd_kernel, solution/kernels.py:178-205):
//   dx = dres + rstd * (g - xhat * mean(g * xhat)) * grad_scale,  g = w * (dy + drop_q(tq) + drop_v(tv))
// with the masks regenerated. tq / tv are either given ([n, H]) or formed in-kernel from the
// LoRA factors, tq = dx_lo . A (solution/engine.py:1326-1330), rounded like the reference's fp16
// GEMM output. Optionally also writes dx in the 16-bit type (the next data-gradient GEMM's A).
//
// One CTA of 128 threads per row, each thread holding groups of 4 consecutive columns in
// registers (H <= 4096): one HBM read of the row, one write per output.
#include "common.cuh"
#include "ops.h"
#include "philox.cuh"

namespace ql {

constexpr int RMS_THREADS = 128;
constexpr int RMS_MAXG = 8;  // groups of 4 per thread: H <= 4 * 128 * 8 = 4096
constexpr int LORA_R = 16;

struct RmsFwdArgs {
  const float* x;
  const void* delta;  // [n, H] T or null
  const float* w;
  float* xsum;        // [n, H] fp32 (required with delta)
  void* y;            // [n, H] T or null
  void* yq;           // [n, H] T or null (the dropped copy for the q LoRA)
  void* yv;
  float* rstd;
  const void* Aq;     // [R, H] T or null: writes xq = drop_q(y) . Aq^T
  const void* Av;
  void* xq;           // [n, R] T
  void* xv;
  int n, H;
  float eps;
  DropoutArgs drop;
};

struct RmsBwdArgs {
  const void* dy;     // [n, ld_dy] T
  int64_t ld_dy;
  const float* x;     // the normalised input (xsum of the forward)
  const float* rstd;
  const float* w;
  const float* dres;  // [n, H] fp32 or null
  float* dx;          // [n, H] fp32
  void* dx16;         // [n, H] T or null
  const void* tq;     // [n, H] T or null (explicit LoRA input gradients)
  const void* tv;
  const float* dxlo_q;  // [n, R] fp32 or null: tq = dxlo_q . Aq
  const float* dxlo_v;
  const void* Aq;     // [R, H] T
  const void* Av;
  int n, H;
  float grad_scale;
  DropoutArgs drop;
};

template <typename T>
__device__ __forceinline__ float4 load4(const T* p) {
  if constexpr (sizeof(T) == 4) {
    return *reinterpret_cast<const float4*>(p);
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const T* h = reinterpret_cast<const T*>(&u);
    return make_float4(to_f<T>(h[0]), to_f<T>(h[1]), to_f<T>(h[2]), to_f<T>(h[3]));
  }
}

template <typename T>
__device__ __forceinline__ void store4(T* p, float4 v) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4*>(p) = v;
  } else {
    T h[4] = {from_f<T>(v.x), from_f<T>(v.y), from_f<T>(v.z), from_f<T>(v.w)};
    *reinterpret_cast<uint2*>(p) = *reinterpret_cast<const uint2*>(h);
  }
}

template <typename T>
__device__ __forceinline__ float4 round4(float4 v) {
  return make_float4(to_f<T>(from_f<T>(v.x)), to_f<T>(from_f<T>(v.y)), to_f<T>(from_f<T>(v.z)),
                     to_f<T>(from_f<T>(v.w)));
}

__device__ __forceinline__ float4 masked4(float4 v, uint32_t keep, float s) {
  return make_float4((keep & 1u) ? v.x * s : 0.f, (keep & 2u) ? v.y * s : 0.f,
                     (keep & 4u) ? v.z * s : 0.f, (keep & 8u) ? v.w * s : 0.f);
}

// Sums NV values held by every thread of the CTA; the result is valid in all threads.
template <int NV>
__device__ __forceinline__ void block_sum(float* v, float* scratch /* [4][NV] */) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < NV; ++i) v[i] = warp_sum(v[i]);
  __syncthreads();
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < NV; ++i) scratch[warp * NV + i] = v[i];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < NV; ++i) v[i] = scratch[i] + scratch[NV + i] + scratch[2 * NV + i] + scratch[3 * NV + i];
}

template <typename T>
__global__ void __launch_bounds__(RMS_THREADS) rms_fwd_kernel(RmsFwdArgs a) {
  __shared__ float scratch[4 * 2 * LORA_R];
  const int row = blockIdx.x;
  const int H = a.H, ngroups = H / 4;
  const int64_t base = (int64_t)row * H;
  float4 xv[RMS_MAXG];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < RMS_MAXG; ++k) {
    const int gi = threadIdx.x + k * RMS_THREADS;
    if (gi < ngroups) {
      float4 x = *reinterpret_cast<const float4*>(a.x + base + 4 * gi);
      if (a.delta != nullptr) {
        const float4 d = load4<T>(reinterpret_cast<const T*>(a.delta) + base + 4 * gi);
        x = make_float4(x.x + d.x, x.y + d.y, x.z + d.z, x.w + d.w);
        *reinterpret_cast<float4*>(a.xsum + base + 4 * gi) = x;
      }
      xv[k] = x;
      ss += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
    }
  }
  float tot[1] = {ss};
  block_sum<1>(tot, scratch);
  const float rstd = 1.0f / sqrtf(tot[0] / (float)H + a.eps);
  if (threadIdx.x == 0) a.rstd[row] = rstd;

  const bool lora_q = a.drop.drop_q && a.Aq != nullptr, lora_v = a.drop.drop_v && a.Av != nullptr;
  float accq[LORA_R], accv[LORA_R];
#pragma unroll
  for (int r = 0; r < LORA_R; ++r) accq[r] = accv[r] = 0.f;
  const int64_t e_row = (a.drop.drop_q || a.drop.drop_v) ? a.drop.tok[row] * (int64_t)H : 0;
#pragma unroll
  for (int k = 0; k < RMS_MAXG; ++k) {
    const int gi = threadIdx.x + k * RMS_THREADS;
    if (gi < ngroups) {
      const int c = 4 * gi;
      const float4 w = *reinterpret_cast<const float4*>(a.w + c);
      const float4 x = xv[k];
      const float4 y = make_float4(w.x * (x.x * rstd), w.y * (x.y * rstd), w.z * (x.z * rstd),
                                   w.w * (x.w * rstd));
      if (a.y != nullptr) store4<T>(reinterpret_cast<T*>(a.y) + base + c, y);
      if (a.drop.drop_q) {
        const float4 yq = round4<T>(masked4(y, keep4(e_row + c, a.drop.ctr_q, a.drop), a.drop.keep_scale));
        if (a.yq != nullptr) store4<T>(reinterpret_cast<T*>(a.yq) + base + c, yq);
        if (lora_q) {
          const T* A = reinterpret_cast<const T*>(a.Aq);
#pragma unroll
          for (int r = 0; r < LORA_R; ++r) {
            const float4 av = load4<T>(A + (int64_t)r * H + c);
            accq[r] += yq.x * av.x + yq.y * av.y + yq.z * av.z + yq.w * av.w;
          }
        }
      }
      if (a.drop.drop_v) {
        const float4 yv = round4<T>(masked4(y, keep4(e_row + c, a.drop.ctr_v, a.drop), a.drop.keep_scale));
        if (a.yv != nullptr) store4<T>(reinterpret_cast<T*>(a.yv) + base + c, yv);
        if (lora_v) {
          const T* A = reinterpret_cast<const T*>(a.Av);
#pragma unroll
          for (int r = 0; r < LORA_R; ++r) {
            const float4 av = load4<T>(A + (int64_t)r * H + c);
            accv[r] += yv.x * av.x + yv.y * av.y + yv.z * av.z + yv.w * av.w;
          }
        }
      }
    }
  }
  if (lora_q || lora_v) {
    float v[2 * LORA_R];
#pragma unroll
    for (int r = 0; r < LORA_R; ++r) {
      v[r] = accq[r];
      v[LORA_R + r] = accv[r];
    }
    block_sum<2 * LORA_R>(v, scratch);
    if (threadIdx.x < LORA_R) {
      const int r = threadIdx.x;
      float q = 0.f, vv = 0.f;
#pragma unroll
      for (int i = 0; i < LORA_R; ++i) {
        if (i == r) { q = v[i]; vv = v[LORA_R + i]; }
      }
      if (lora_q) reinterpret_cast<T*>(a.xq)[(int64_t)row * LORA_R + r] = from_f<T>(q);
      if (lora_v) reinterpret_cast<T*>(a.xv)[(int64_t)row * LORA_R + r] = from_f<T>(vv);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(RMS_THREADS) rms_bwd_kernel(RmsBwdArgs a) {
  __shared__ float scratch[4];
  __shared__ float lq[LORA_R], lv[LORA_R];
  const int row = blockIdx.x;
  const int H = a.H, ngroups = H / 4;
  const int64_t base = (int64_t)row * H;
  if (threadIdx.x < LORA_R) {
    lq[threadIdx.x] = a.dxlo_q != nullptr ? a.dxlo_q[(int64_t)row * LORA_R + threadIdx.x] : 0.f;
    lv[threadIdx.x] = a.dxlo_v != nullptr ? a.dxlo_v[(int64_t)row * LORA_R + threadIdx.x] : 0.f;
  }
  __syncthreads();
  const float rstd = a.rstd[row];
  const int64_t e_row = (a.drop.drop_q || a.drop.drop_v) ? a.drop.tok[row] * (int64_t)H : 0;
  float4 gv[RMS_MAXG], xh[RMS_MAXG];
  float dot = 0.f;
#pragma unroll
  for (int k = 0; k < RMS_MAXG; ++k) {
    const int gi = threadIdx.x + k * RMS_THREADS;
    if (gi < ngroups) {
      const int c = 4 * gi;
      float4 dy = load4<T>(reinterpret_cast<const T*>(a.dy) + (int64_t)row * a.ld_dy + c);
      for (int which = 0; which < 2; ++which) {
        const bool on = which == 0 ? a.drop.drop_q : a.drop.drop_v;
        if (!on) continue;
        const void* tex = which == 0 ? a.tq : a.tv;
        const float* lo = which == 0 ? lq : lv;
        const void* A = which == 0 ? a.Aq : a.Av;
        float4 t;
        if (tex != nullptr) {
          t = load4<T>(reinterpret_cast<const T*>(tex) + base + c);
        } else {
          const T* At = reinterpret_cast<const T*>(A);
          t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int r = 0; r < LORA_R; ++r) {
            const float4 av = load4<T>(At + (int64_t)r * H + c);
            t.x += lo[r] * av.x; t.y += lo[r] * av.y; t.z += lo[r] * av.z; t.w += lo[r] * av.w;
          }
          t = round4<T>(t);
        }
        const uint32_t keep = keep4(e_row + c, which == 0 ? a.drop.ctr_q : a.drop.ctr_v, a.drop);
        const float4 m = masked4(t, keep, a.drop.keep_scale);
        dy = make_float4(dy.x + m.x, dy.y + m.y, dy.z + m.z, dy.w + m.w);
      }
      const float4 w = *reinterpret_cast<const float4*>(a.w + c);
      const float4 x = *reinterpret_cast<const float4*>(a.x + base + c);
      const float4 g = make_float4(dy.x * w.x, dy.y * w.y, dy.z * w.z, dy.w * w.w);
      const float4 h = make_float4(x.x * rstd, x.y * rstd, x.z * rstd, x.w * rstd);
      gv[k] = g;
      xh[k] = h;
      dot += g.x * h.x + g.y * h.y + g.z * h.z + g.w * h.w;
    }
  }
  float tot[1] = {dot};
  block_sum<1>(tot, scratch);
  const float mean = tot[0] / (float)H;
#pragma unroll
  for (int k = 0; k < RMS_MAXG; ++k) {
    const int gi = threadIdx.x + k * RMS_THREADS;
    if (gi < ngroups) {
      const int c = 4 * gi;
      const float4 g = gv[k], h = xh[k];
      float4 d = make_float4(rstd * (g.x - h.x * mean) * a.grad_scale,
                             rstd * (g.y - h.y * mean) * a.grad_scale,
                             rstd * (g.z - h.z * mean) * a.grad_scale,
                             rstd * (g.w - h.w * mean) * a.grad_scale);
      if (a.dres != nullptr) {
        const float4 r = *reinterpret_cast<const float4*>(a.dres + base + c);
        d = make_float4(d.x + r.x, d.y + r.y, d.z + r.z, d.w + r.w);
      }
      *reinterpret_cast<float4*>(a.dx + base + c) = d;
      if (a.dx16 != nullptr) store4<T>(reinterpret_cast<T*>(a.dx16) + base + c, d);
    }
  }
}

int rms_fwd(const RmsFwdC& c, cudaStream_t s) {
  if (c.n < 0 || c.H <= 0 || c.H % 4 != 0 || c.H > 4 * RMS_THREADS * RMS_MAXG) return QL_STATUS_BAD_ARG;
  if (c.n == 0) return QL_STATUS_OK;
  if (c.delta != nullptr && c.xsum == nullptr) return QL_STATUS_BAD_ARG;
  if ((c.drop_q || c.drop_v) && c.tok == nullptr) return QL_STATUS_BAD_ARG;
  if ((c.Aq != nullptr && c.xq == nullptr) || (c.Av != nullptr && c.xv == nullptr)) return QL_STATUS_BAD_ARG;
  if ((c.Aq != nullptr || c.Av != nullptr) && c.rank != LORA_R) return QL_STATUS_UNSUPPORTED;
  RmsFwdArgs a{c.x, c.delta, c.w, c.xsum, c.y, c.yq, c.yv, c.rstd, c.Aq, c.Av, c.xq, c.xv, c.n,
               c.H, c.eps,
               DropoutArgs{c.tok, c.seed, c.ctr_q, c.ctr_v, c.threads > 0 ? c.threads : 1,
                           c.p_keep, c.keep_scale, c.vec, c.drop_q, c.drop_v}};
  if (c.vec != 4 && c.vec != 8) return QL_STATUS_BAD_ARG;
  if (c.dtype == QL_F16) rms_fwd_kernel<__half><<<c.n, RMS_THREADS, 0, s>>>(a);
  else if (c.dtype == QL_BF16) rms_fwd_kernel<__nv_bfloat16><<<c.n, RMS_THREADS, 0, s>>>(a);
  else return QL_STATUS_BAD_ARG;
  return cudaPeekAtLastError() == cudaSuccess ? QL_STATUS_OK : QL_STATUS_CUDA;
}

int rms_bwd(const RmsBwdC& c, cudaStream_t s) {
  if (c.n < 0 || c.H <= 0 || c.H % 4 != 0 || c.H > 4 * RMS_THREADS * RMS_MAXG) return QL_STATUS_BAD_ARG;
  if (c.n == 0) return QL_STATUS_OK;
  if ((c.drop_q || c.drop_v) && c.tok == nullptr) return QL_STATUS_BAD_ARG;
  if (c.drop_q && c.tq == nullptr && (c.dxlo_q == nullptr || c.Aq == nullptr)) return QL_STATUS_BAD_ARG;
  if (c.drop_v && c.tv == nullptr && (c.dxlo_v == nullptr || c.Av == nullptr)) return QL_STATUS_BAD_ARG;
  if ((c.dxlo_q != nullptr || c.dxlo_v != nullptr) && c.rank != LORA_R) return QL_STATUS_UNSUPPORTED;
  if (c.ld_dy % 4 != 0) return QL_STATUS_BAD_ARG;
  if (c.vec != 4 && c.vec != 8) return QL_STATUS_BAD_ARG;
  RmsBwdArgs a{c.dy, c.ld_dy, c.x, c.rstd, c.w, c.dres, c.dx, c.dx16, c.tq, c.tv, c.dxlo_q,
               c.dxlo_v, c.Aq, c.Av, c.n, c.H, c.grad_scale,
               DropoutArgs{c.tok, c.seed, c.ctr_q, c.ctr_v, c.threads > 0 ? c.threads : 1,
                           c.p_keep, c.keep_scale, c.vec, c.drop_q, c.drop_v}};
  if (c.dtype == QL_F16) rms_bwd_kernel<__half><<<c.n, RMS_THREADS, 0, s>>>(a);
  else if (c.dtype == QL_BF16) rms_bwd_kernel<__nv_bfloat16><<<c.n, RMS_THREADS, 0, s>>>(a);
  else return QL_STATUS_BAD_ARG;
  return cudaPeekAtLastError() == cudaSuccess ? QL_STATUS_OK : QL_STATUS_CUDA;
}

}  // namespace ql

namespace ql {

__global__ void dropout_keep_kernel(int8_t* out, int64_t nelem, DropoutArgs d) {
  const int64_t e0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) * 4;
  if (e0 >= nelem) return;
  const uint32_t k = keep4(e0, d.ctr_q, d);
  for (int j = 0; j < 4 && e0 + j < nelem; ++j) out[e0 + j] = (k >> j) & 1u;
}

int dropout_keep(int8_t* out, int64_t nelem, int64_t seed, int64_t ctr, int64_t threads,
                 float p_keep, int vec, cudaStream_t s) {
  if (nelem < 0 || threads <= 0 || (vec != 4 && vec != 8)) return QL_STATUS_BAD_ARG;
  if (nelem == 0) return QL_STATUS_OK;
  DropoutArgs d{nullptr, seed, ctr, 0, threads, p_keep, 1.f, vec, 1, 0};
  const int64_t groups = cdiv(nelem, 4);
  dropout_keep_kernel<<<(unsigned)cdiv(groups, 256), 256, 0, s>>>(out, nelem, d);
  return cudaPeekAtLastError() == cudaSuccess ? QL_STATUS_OK : QL_STATUS_CUDA;
}

}  // namespace ql
