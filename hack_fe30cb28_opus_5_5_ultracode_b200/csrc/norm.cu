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
// One warp per row, each lane holding groups of 4 consecutive columns in registers (H <= 4096):
// one HBM read of the row, one write per output; the LoRA factors A (2 x 16 x H 16-bit) are
// staged in shared memory once per CTA, and the 32 LoRA-A sums of a row leave the warp by one
// reduce-scatter.
#include "common.cuh"
#include "profile.h"
#include "ops.h"
#include "philox.cuh"

namespace ql {

constexpr int RMS_THREADS = 128;  // (used for the H bound below)
constexpr int RMS_MAXG = 8;       // H <= 4 * 128 * 8 = 4096
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

// Sum over the warp of 32 per-lane values v[0..31]; afterwards lane l holds the total of value l
// (reduce-scatter: 31 shuffles instead of 32 x 5).
__device__ __forceinline__ float reduce_scatter32(float* v) {
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

// One warp per row (8 rows in flight per CTA, rows strided over the grid); the row's groups of
// 4 columns g = lane + 32 k stay in registers between the two passes (G = groups per lane).
// The LoRA-A factors are staged once per CTA in shared memory.
template <typename T, int G>
__global__ void __launch_bounds__(256) rms_fwd_kernel(RmsFwdArgs a) {
  extern __shared__ __align__(16) uint8_t rms_smem[];
  T* sAq = reinterpret_cast<T*>(rms_smem);
  T* sAv = sAq + LORA_R * a.H;
  const int H = a.H, ngroups = H / 4;
  const bool lora_q = a.drop.drop_q && a.Aq != nullptr, lora_v = a.drop.drop_v && a.Av != nullptr;
  if (lora_q || lora_v) {
    if (lora_q) stage_to_smem(sAq, a.Aq, LORA_R * H * (int)sizeof(T));
    if (lora_v) stage_to_smem(sAv, a.Av, LORA_R * H * (int)sizeof(T));
    stage_wait();
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int row = blockIdx.x * 8 + warp; row < a.n; row += gridDim.x * 8) {
    const int64_t base = (int64_t)row * H;
    float4 xv[G];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < G; ++k) {
      const int gi = lane + 32 * k;
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
    ss = warp_sum(ss);
    const float rstd = 1.0f / sqrtf(ss / (float)H + a.eps);
    if (lane == 0) a.rstd[row] = rstd;
    float acc[2 * LORA_R];
#pragma unroll
    for (int r = 0; r < 2 * LORA_R; ++r) acc[r] = 0.f;
    const int64_t e_row = (a.drop.drop_q || a.drop.drop_v) ? a.drop.tok[row] * (int64_t)H : 0;
#pragma unroll
    for (int k = 0; k < G; ++k) {
      const int gi = lane + 32 * k;
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
#pragma unroll
            for (int r = 0; r < LORA_R; ++r) {
              const float4 av = load4<T>(sAq + r * H + c);
              acc[r] += yq.x * av.x + yq.y * av.y + yq.z * av.z + yq.w * av.w;
            }
          }
        }
        if (a.drop.drop_v) {
          const float4 yv = round4<T>(masked4(y, keep4(e_row + c, a.drop.ctr_v, a.drop), a.drop.keep_scale));
          if (a.yv != nullptr) store4<T>(reinterpret_cast<T*>(a.yv) + base + c, yv);
          if (lora_v) {
#pragma unroll
            for (int r = 0; r < LORA_R; ++r) {
              const float4 av = load4<T>(sAv + r * H + c);
              acc[LORA_R + r] += yv.x * av.x + yv.y * av.y + yv.z * av.z + yv.w * av.w;
            }
          }
        }
      }
    }
    if (lora_q || lora_v) {
      const float tot = reduce_scatter32(acc);  // lane l: value l (q: 0..15, v: 16..31)
      if (lane < LORA_R) {
        if (lora_q) reinterpret_cast<T*>(a.xq)[(int64_t)row * LORA_R + lane] = from_f<T>(tot);
      } else if (lora_v) {
        reinterpret_cast<T*>(a.xv)[(int64_t)row * LORA_R + lane - LORA_R] = from_f<T>(tot);
      }
    }
  }
}

template <typename T, int G>
__global__ void __launch_bounds__(256) rms_bwd_kernel(RmsBwdArgs a) {
  extern __shared__ __align__(16) uint8_t rms_smem[];
  T* sAq = reinterpret_cast<T*>(rms_smem);
  T* sAv = sAq + LORA_R * a.H;
  const int H = a.H, ngroups = H / 4;
  const bool fq = a.drop.drop_q && a.tq == nullptr, fv = a.drop.drop_v && a.tv == nullptr;
  if (fq || fv) {
    if (fq) stage_to_smem(sAq, a.Aq, LORA_R * H * (int)sizeof(T));
    if (fv) stage_to_smem(sAv, a.Av, LORA_R * H * (int)sizeof(T));
    stage_wait();
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int row = blockIdx.x * 8 + warp; row < a.n; row += gridDim.x * 8) {
    const int64_t base = (int64_t)row * H;
    const float rstd = a.rstd[row];
    // this row's LoRA input gradients dx_lo (q: lanes 0..15, v: lanes 16..31), broadcast below
    float lo_mine = 0.f;
    if (lane < LORA_R) { if (a.dxlo_q != nullptr) lo_mine = a.dxlo_q[(int64_t)row * LORA_R + lane]; }
    else if (a.dxlo_v != nullptr) lo_mine = a.dxlo_v[(int64_t)row * LORA_R + lane - LORA_R];
    float lo[2 * LORA_R];
#pragma unroll
    for (int r = 0; r < 2 * LORA_R; ++r) lo[r] = __shfl_sync(0xffffffffu, lo_mine, r);
    const int64_t e_row = (a.drop.drop_q || a.drop.drop_v) ? a.drop.tok[row] * (int64_t)H : 0;
    float4 gv[G], xh[G];
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < G; ++k) {
      const int gi = lane + 32 * k;
      if (gi < ngroups) {
        const int c = 4 * gi;
        float4 dy = load4<T>(reinterpret_cast<const T*>(a.dy) + (int64_t)row * a.ld_dy + c);
#pragma unroll
        for (int which = 0; which < 2; ++which) {
          const bool on = which == 0 ? a.drop.drop_q : a.drop.drop_v;
          if (!on) continue;
          const void* tex = which == 0 ? a.tq : a.tv;
          float4 t;
          if (tex != nullptr) {
            t = load4<T>(reinterpret_cast<const T*>(tex) + base + c);
          } else {
            const T* At = which == 0 ? sAq : sAv;
            t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int r = 0; r < LORA_R; ++r) {
              const float l = lo[which * LORA_R + r];
              const float4 av = load4<T>(At + r * H + c);
              t.x += l * av.x; t.y += l * av.y; t.z += l * av.z; t.w += l * av.w;
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
    const float mean = warp_sum(dot) / (float)H;
#pragma unroll
    for (int k = 0; k < G; ++k) {
      const int gi = lane + 32 * k;
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
}

static int rms_grid(int64_t n) {
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = cdiv(n, 8);
  const int64_t cap = (int64_t)sms * 4;
  return (int)(want < cap ? want : cap);
}

// Opts a kernel into more than 48 KB of dynamic shared memory, once per kernel (and size).
template <typename K>
static void set_smem(K kern, int bytes) {
  if (bytes > 48 * 1024) smem_optin(reinterpret_cast<const void*>(kern), bytes);
}

int rms_fwd(const RmsFwdC& c, cudaStream_t s) {
  if (c.n < 0 || c.H <= 0 || c.H % 4 != 0 || c.H > 4 * RMS_THREADS * RMS_MAXG) return QL_STATUS_BAD_ARG;
  if (c.n == 0) return QL_STATUS_OK;
  if (c.delta != nullptr && c.xsum == nullptr) return QL_STATUS_BAD_ARG;
  if ((c.drop_q || c.drop_v) && c.tok == nullptr) return QL_STATUS_BAD_ARG;
  if ((c.Aq != nullptr && c.xq == nullptr) || (c.Av != nullptr && c.xv == nullptr)) return QL_STATUS_BAD_ARG;
  if ((c.Aq != nullptr || c.Av != nullptr) && c.rank != LORA_R) return QL_STATUS_UNSUPPORTED;
  ProfScope prof(PK_RMS_FWD, 0, (double)c.n * c.H * (4 + (c.delta ? 6 : 0) + (c.y ? 2 : 0) +
                                                     (c.yq ? 2 : 0) + (c.yv ? 2 : 0)), s);
  RmsFwdArgs a{c.x, c.delta, c.w, c.xsum, c.y, c.yq, c.yv, c.rstd, c.Aq, c.Av, c.xq, c.xv, c.n,
               c.H, c.eps,
               DropoutArgs{c.tok, c.seed, c.ctr_q, c.ctr_v, c.threads > 0 ? c.threads : 1,
                           c.p_keep, c.keep_scale, c.vec, c.drop_q, c.drop_v, FastDiv{}}};
  if (c.vec != 4 && c.vec != 8) return QL_STATUS_BAD_ARG;
  if (!prepare_dropout(a.drop)) return QL_STATUS_BAD_ARG;
  const bool lora = (c.drop_q && c.Aq != nullptr) || (c.drop_v && c.Av != nullptr);
  const int smem = lora ? 2 * LORA_R * c.H * 2 : 0;
  const int grid = rms_grid(c.n);
#define QL_RMSF(TT, GG)                                              \
  do {                                                               \
    set_smem(rms_fwd_kernel<TT, GG>, smem);                          \
    rms_fwd_kernel<TT, GG><<<grid, 256, smem, s>>>(a);               \
  } while (0)
  const int G = (int)cdiv(c.H / 4, 32);
  if (c.dtype == QL_F16) {
    if (G <= 4) QL_RMSF(__half, 4); else if (G <= 12) QL_RMSF(__half, 12); else QL_RMSF(__half, 32);
  } else if (c.dtype == QL_BF16) {
    if (G <= 4) QL_RMSF(__nv_bfloat16, 4); else if (G <= 12) QL_RMSF(__nv_bfloat16, 12);
    else QL_RMSF(__nv_bfloat16, 32);
  } else {
    return QL_STATUS_BAD_ARG;
  }
#undef QL_RMSF
  return launched(1);
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
  ProfScope prof(PK_RMS_BWD, 0, (double)c.n * c.H * (2 + 4 + 4 + (c.dres ? 4 : 0) +
                                                     (c.dx16 ? 2 : 0)), s);
  RmsBwdArgs a{c.dy, c.ld_dy, c.x, c.rstd, c.w, c.dres, c.dx, c.dx16, c.tq, c.tv, c.dxlo_q,
               c.dxlo_v, c.Aq, c.Av, c.n, c.H, c.grad_scale,
               DropoutArgs{c.tok, c.seed, c.ctr_q, c.ctr_v, c.threads > 0 ? c.threads : 1,
                           c.p_keep, c.keep_scale, c.vec, c.drop_q, c.drop_v, FastDiv{}}};
  if (!prepare_dropout(a.drop)) return QL_STATUS_BAD_ARG;
  const bool lora = (c.drop_q && c.tq == nullptr) || (c.drop_v && c.tv == nullptr);
  const int smem = lora ? 2 * LORA_R * c.H * 2 : 0;
  const int grid = rms_grid(c.n);
#define QL_RMSB(TT, GG)                                              \
  do {                                                               \
    set_smem(rms_bwd_kernel<TT, GG>, smem);                          \
    rms_bwd_kernel<TT, GG><<<grid, 256, smem, s>>>(a);               \
  } while (0)
  const int G = (int)cdiv(c.H / 4, 32);
  if (c.dtype == QL_F16) {
    if (G <= 4) QL_RMSB(__half, 4); else if (G <= 12) QL_RMSB(__half, 12); else QL_RMSB(__half, 32);
  } else if (c.dtype == QL_BF16) {
    if (G <= 4) QL_RMSB(__nv_bfloat16, 4); else if (G <= 12) QL_RMSB(__nv_bfloat16, 12);
    else QL_RMSB(__nv_bfloat16, 32);
  } else {
    return QL_STATUS_BAD_ARG;
  }
#undef QL_RMSB
  return launched(1);
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
  DropoutArgs d{nullptr, seed, ctr, 0, threads, p_keep, 1.f, vec, 1, 0, FastDiv{}};
  if (!prepare_dropout(d)) return QL_STATUS_BAD_ARG;
  const int64_t groups = cdiv(nelem, 4);
  dropout_keep_kernel<<<(unsigned)cdiv(groups, 256), 256, 0, s>>>(out, nelem, d);
  return launched(1);
}

}  // namespace ql
