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
// CTA tiles of 8 rows, one warp per row, each lane holding groups of 4 consecutive columns in
// registers (H <= 4096): one HBM read of the row, one write per output. The rank-16 LoRA products
// run on the tensor cores (mma.sync m16n8k16, fp32 accumulation) over the tile: forward, the
// dropped rows go to shared memory and 8 warps (2 adapters x 4 quarters of K) multiply them by
// A^T; backward, tq = dx_lo . A is formed per tile into shared memory before the row pass reads
// it. The dropout masks can be kept as bits by the forward and read by the backward instead of
// drawing the Philox numbers again.
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
  uint32_t* keep_q;   // [n, H / 32] or null: masks out as bits
  uint32_t* keep_v;
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
  const uint32_t* keep_q;  // [n, H / 32] or null: masks in as bits
  const uint32_t* keep_v;
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

constexpr int RMS_MAXR = 16;  // rows per CTA tile at most (the tensor-core fragments' 16 rows)
constexpr int RMS_PAD = 8;    // 16-bit elements of padding per shared row: conflict-free fragments

// OR of 4-bit masks over the 8 lanes that share a 32-column word; lane 8j returns word j.
__device__ __forceinline__ uint32_t gather_bits(uint32_t nib) {
  const int lane = threadIdx.x & 31;
  uint32_t w = nib << (4 * (lane & 7));
  w |= __shfl_xor_sync(0xffffffffu, w, 1);
  w |= __shfl_xor_sync(0xffffffffu, w, 2);
  w |= __shfl_xor_sync(0xffffffffu, w, 4);
  return w;
}

// The A fragment of m16n8k16 for tile rows g and g + 8 from 16-bit rows in shared memory at
// column k0 (rows at or past `rows` read as zero).
template <typename T>
__device__ __forceinline__ void frag_rows(uint32_t (&af)[4], const T* base, int ld, int g, int t,
                                          int rows, int k0) {
  const T* r0 = base + g * ld + k0 + 2 * t;
  const T* r1 = base + (g + 8) * ld + k0 + 2 * t;
  af[0] = g < rows ? *reinterpret_cast<const uint32_t*>(r0) : 0u;
  af[1] = g + 8 < rows ? *reinterpret_cast<const uint32_t*>(r1) : 0u;
  af[2] = g < rows ? *reinterpret_cast<const uint32_t*>(r0 + 8) : 0u;
  af[3] = g + 8 < rows ? *reinterpret_cast<const uint32_t*>(r1 + 8) : 0u;
}

// Tiles of `rows` rows (at most 16; the launcher picks the count that spreads the rows over one
// balanced wave of CTAs), tiles strided over the grid. WPR warps share a row (rows x WPR warps per
// CTA): warp w works on row w / WPR, and its lanes hold the row's groups of 4 columns
// gi = 32 (w % WPR) + lane + 32 WPR k (k < G).
template <typename T, int G, int WPR>
__global__ void __launch_bounds__(WPR == 1 ? 32 * RMS_MAXR : 1024) rms_fwd_kernel(RmsFwdArgs a, int rows) {
  pdl_enter();
  extern __shared__ __align__(16) uint8_t rms_smem[];
  __shared__ float sSS[32];
  const int H = a.H, ngroups = H / 4, ld = H + RMS_PAD, NW = rows * WPR;
  T* sY = reinterpret_cast<T*>(rms_smem);  // [2][rows][ld] dropped rows (q, v) of the tile
  float* sRed = reinterpret_cast<float*>(sY + 2 * rows * ld);  // [NW][16 rows][16]
  const bool lora_q = a.drop.drop_q && a.Aq != nullptr, lora_v = a.drop.drop_v && a.Av != nullptr;
  const int nad = (int)lora_q + (int)lora_v;  // adapters with a LoRA-A product
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rrow = warp / WPR, part = warp % WPR;
  const int ntiles = (a.n + rows - 1) / rows;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int row = tile * rows + rrow;
    const bool live = row < a.n;
    const int64_t base = (int64_t)row * H;
    // the row stays in registers between the passes for up to 16 columns per lane; wider rows
    // read it again (from L1)
    constexpr bool kKeepX = G <= 4 || WPR == 1;
    float4 xv[kKeepX ? G : 1];
    float ss = 0.f;
    if (live) {
#pragma unroll
      for (int k = 0; k < G; ++k) {
        const int gi = 32 * part + lane + 32 * WPR * k;
        if (gi < ngroups) {
          float4 x = *reinterpret_cast<const float4*>(a.x + base + 4 * gi);
          if (a.delta != nullptr) {
            const float4 d = load4<T>(reinterpret_cast<const T*>(a.delta) + base + 4 * gi);
            x = make_float4(x.x + d.x, x.y + d.y, x.z + d.z, x.w + d.w);
            *reinterpret_cast<float4*>(a.xsum + base + 4 * gi) = x;
          }
          if constexpr (kKeepX) xv[k] = x;
          ss += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
        }
      }
    }
    ss = warp_sum(ss);
    if constexpr (WPR > 1) {  // the row's warps add their sums in a fixed order
      if (lane == 0) sSS[warp] = ss;
      __syncthreads();
      ss = 0.f;
#pragma unroll
      for (int p = 0; p < WPR; ++p) ss += sSS[rrow * WPR + p];
    }
    if (live) {
      const float rstd = 1.0f / sqrtf(ss / (float)H + a.eps);
      if (lane == 0 && part == 0) a.rstd[row] = rstd;
      const int64_t e_row = (a.drop.drop_q || a.drop.drop_v) ? a.drop.tok[row] * (int64_t)H : 0;
      const int64_t wrow = (int64_t)row * (H / 32);
#pragma unroll
      for (int k = 0; k < G; ++k) {
        const int gi = 32 * part + lane + 32 * WPR * k;
        uint32_t nq = 0, nv = 0;
        if (gi < ngroups) {
          const int c = 4 * gi;
          const float4 w = *reinterpret_cast<const float4*>(a.w + c);
          float4 x;
          if constexpr (kKeepX) x = xv[k];
          else x = *reinterpret_cast<const float4*>((a.delta != nullptr ? a.xsum : a.x) + base + c);
          const float4 y = make_float4(w.x * (x.x * rstd), w.y * (x.y * rstd),
                                       w.z * (x.z * rstd), w.w * (x.w * rstd));
          if (a.y != nullptr) store4<T>(reinterpret_cast<T*>(a.y) + base + c, y);
          if (a.drop.drop_q) {
            nq = keep4(e_row + c, a.drop.ctr_q, a.drop);
            const float4 yq = masked4(y, nq, a.drop.keep_scale);
            if (a.yq != nullptr) store4<T>(reinterpret_cast<T*>(a.yq) + base + c, yq);
            if (lora_q) store4<T>(sY + rrow * ld + c, yq);
          }
          if (a.drop.drop_v) {
            nv = keep4(e_row + c, a.drop.ctr_v, a.drop);
            const float4 yv = masked4(y, nv, a.drop.keep_scale);
            if (a.yv != nullptr) store4<T>(reinterpret_cast<T*>(a.yv) + base + c, yv);
            if (lora_v) store4<T>(sY + (rows + rrow) * ld + c, yv);
          }
        }
        if (a.keep_q != nullptr) {
          const uint32_t wq = gather_bits(nq);
          if ((lane & 7) == 0 && gi < ngroups) a.keep_q[wrow + gi / 8] = wq;
        }
        if (a.keep_v != nullptr) {
          const uint32_t wv = gather_bits(nv);
          if ((lane & 7) == 0 && gi < ngroups) a.keep_v[wrow + gi / 8] = wv;
        }
      }
    }
    if (nad > 0) {
      // x_lo[rows][16] = drop(y)[rows][H] . A^T on the tensor cores, as nad x S work items
      // (adapter, K slice), S = max(1, NW / nad) slices per adapter; item i = adapter i / S, slice
      // i % S takes the 16-column K steps slice, slice + S, ... and goes to warp i % NW (a CTA of
      // one warp does both adapters). The tile's rows are rows 0 .. rows-1 of the A fragment.
      __syncthreads();
      const int S = NW / nad > 0 ? NW / nad : 1;
      const int g = lane >> 2, t = lane & 3;
      for (int item = warp; item < nad * S; item += NW) {
        const int adi = item / S, slice = item % S;
        const int ad = (nad == 2) ? adi : (lora_q ? 0 : 1);
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        const T* A = reinterpret_cast<const T*>(ad == 0 ? a.Aq : a.Av);
        const T* Y = sY + ad * rows * ld;
#pragma unroll 2
        for (int k0 = 16 * slice; k0 < H; k0 += 16 * S) {
          uint32_t af[4];
          frag_rows<T>(af, Y, ld, g, t, rows, k0);
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const unsigned int* Ab =
                reinterpret_cast<const unsigned int*>(A + (int64_t)(nt * 8 + g) * H + k0 + 2 * t);
            mma16816<T>(acc[nt], af, __ldg(Ab), __ldg(Ab + 4));
          }
        }
        // rows g and g + 8 of columns nt * 8 + 2t, 2t + 1
        float* red = sRed + (item * RMS_MAXR + g) * 16 + 2 * t;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          red[nt * 8] = acc[nt][0];
          red[nt * 8 + 1] = acc[nt][1];
          red[8 * 16 + nt * 8] = acc[nt][2];
          red[8 * 16 + nt * 8 + 1] = acc[nt][3];
        }
      }
      __syncthreads();
      // thread -> (adapter, row, r): the adapter's slices added in a fixed order
      for (int idx = threadIdx.x; idx < nad * rows * LORA_R; idx += blockDim.x) {
        const int oad = idx / (rows * LORA_R), rr = (idx / LORA_R) % rows, r = idx % LORA_R;
        const int orow = tile * rows + rr;
        if (orow < a.n) {
          float sum = 0.f;
          for (int sl = 0; sl < S; ++sl) sum += sRed[((oad * S + sl) * RMS_MAXR + rr) * 16 + r];
          const int dst = (nad == 2) ? oad : (lora_q ? 0 : 1);
          reinterpret_cast<T*>(dst == 0 ? a.xq : a.xv)[(int64_t)orow * LORA_R + r] = from_f<T>(sum);
        }
      }
    }
    __syncthreads();  // shared buffers are refilled by the next tile
  }
}

template <typename T, int G, int WPR>
__global__ void __launch_bounds__(WPR == 1 ? 32 * RMS_MAXR : 1024) rms_bwd_kernel(RmsBwdArgs a, int rows) {
  pdl_enter();
  extern __shared__ __align__(16) uint8_t rms_smem[];
  __shared__ float sDot[32];
  const int H = a.H, ngroups = H / 4, ld = H + RMS_PAD, NW = rows * WPR;
  T* sT = reinterpret_cast<T*>(rms_smem);  // [2][rows][ld] tq, tv of the tile (formed in-kernel)
  const bool fq = a.drop.drop_q && a.tq == nullptr, fv = a.drop.drop_v && a.tv == nullptr;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rrow = warp / WPR, part = warp % WPR;
  const int ntiles = (a.n + rows - 1) / rows;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    if (fq || fv) {
      // t[rows][H] = round16(dx_lo)[rows][16] . A[16][H] on the tensor cores, 8-column tiles
      // strided over the warps; the tile's rows are rows 0 .. rows-1 of the A fragment.
      const int g = lane >> 2, t = lane & 3;
#pragma unroll
      for (int ad = 0; ad < 2; ++ad) {
        if (!(ad == 0 ? fq : fv)) continue;
        const float* lo = ad == 0 ? a.dxlo_q : a.dxlo_v;
        const int r0 = tile * rows + g, r1 = r0 + 8;
        uint32_t af[4] = {0u, 0u, 0u, 0u};
        if (g < rows && r0 < a.n) {
          const float2 p0 = *reinterpret_cast<const float2*>(lo + (int64_t)r0 * LORA_R + 2 * t);
          const float2 p1 = *reinterpret_cast<const float2*>(lo + (int64_t)r0 * LORA_R + 8 + 2 * t);
          af[0] = pack_t2<T>(p0.x, p0.y);
          af[2] = pack_t2<T>(p1.x, p1.y);
        }
        if (g + 8 < rows && r1 < a.n) {
          const float2 p0 = *reinterpret_cast<const float2*>(lo + (int64_t)r1 * LORA_R + 2 * t);
          const float2 p1 = *reinterpret_cast<const float2*>(lo + (int64_t)r1 * LORA_R + 8 + 2 * t);
          af[1] = pack_t2<T>(p0.x, p0.y);
          af[3] = pack_t2<T>(p1.x, p1.y);
        }
        const unsigned short* Ab =
            reinterpret_cast<const unsigned short*>(ad == 0 ? a.Aq : a.Av) + g;
        T* dst0 = sT + (ad * rows + g) * ld + 2 * t;
        T* dst1 = sT + (ad * rows + g + 8) * ld + 2 * t;
        // 8-column groups n0 = 8 (warp + NW j), RB at a time: the groups' B fragments (strided
        // 16-bit reads of A's rows, from L2) are all requested before the first multiply
        constexpr int RB = 2;
        for (int j0 = 0; warp * 8 + j0 * 8 * NW < H; j0 += RB) {
          uint32_t b0[RB], b1[RB];
#pragma unroll
          for (int j = 0; j < RB; ++j) {
            const int n0 = warp * 8 + (j0 + j) * 8 * NW;
            b0[j] = b1[j] = 0u;
            if (n0 < H) {
              const unsigned short* col = Ab + n0;
              b0[j] = (uint32_t)__ldg(col + (2 * t) * H) | ((uint32_t)__ldg(col + (2 * t + 1) * H) << 16);
              b1[j] = (uint32_t)__ldg(col + (2 * t + 8) * H) | ((uint32_t)__ldg(col + (2 * t + 9) * H) << 16);
            }
          }
#pragma unroll
          for (int j = 0; j < RB; ++j) {
            const int n0 = warp * 8 + (j0 + j) * 8 * NW;
            if (n0 >= H) break;
            float c[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816<T>(c, af, b0[j], b1[j]);
            if (g < rows) *reinterpret_cast<uint32_t*>(dst0 + n0) = pack_t2<T>(c[0], c[1]);
            if (g + 8 < rows) *reinterpret_cast<uint32_t*>(dst1 + n0) = pack_t2<T>(c[2], c[3]);
          }
        }
      }
      __syncthreads();
    }
    const int row = tile * rows + rrow;
    const bool live = row < a.n;
    const int64_t base = (int64_t)row * H;
    float rstd = 0.f;
    // x * rstd stays in registers between the passes for up to 16 columns per lane; wider rows
    // read x again (from L1)
    constexpr bool kKeepX = G <= 4 || WPR == 1;
    float4 gv[G], xh[kKeepX ? G : 1];
    float dot = 0.f;
    if (live) {
      rstd = a.rstd[row];
      const int64_t e_row = (a.drop.drop_q || a.drop.drop_v) ? a.drop.tok[row] * (int64_t)H : 0;
      const int64_t wrow = (int64_t)row * (H / 32);
#pragma unroll
      for (int k = 0; k < G; ++k) {
        const int gi = 32 * part + lane + 32 * WPR * k;
        if (gi < ngroups) {
          const int c = 4 * gi;
          float4 dy = load4<T>(reinterpret_cast<const T*>(a.dy) + (int64_t)row * a.ld_dy + c);
#pragma unroll
          for (int which = 0; which < 2; ++which) {
            const bool on = which == 0 ? a.drop.drop_q : a.drop.drop_v;
            if (!on) continue;
            const void* tex = which == 0 ? a.tq : a.tv;
            const float4 t = tex != nullptr
                                 ? load4<T>(reinterpret_cast<const T*>(tex) + base + c)
                                 : load4<T>(sT + (which * rows + rrow) * ld + c);
            const uint32_t* bits = which == 0 ? a.keep_q : a.keep_v;
            const uint32_t keep = bits != nullptr
                                      ? (bits[wrow + c / 32] >> (c & 31)) & 15u
                                      : keep4(e_row + c, which == 0 ? a.drop.ctr_q : a.drop.ctr_v, a.drop);
            const float4 m = masked4(t, keep, a.drop.keep_scale);
            dy = make_float4(dy.x + m.x, dy.y + m.y, dy.z + m.z, dy.w + m.w);
          }
          const float4 w = *reinterpret_cast<const float4*>(a.w + c);
          const float4 x = *reinterpret_cast<const float4*>(a.x + base + c);
          const float4 g = make_float4(dy.x * w.x, dy.y * w.y, dy.z * w.z, dy.w * w.w);
          const float4 h = make_float4(x.x * rstd, x.y * rstd, x.z * rstd, x.w * rstd);
          gv[k] = g;
          if constexpr (kKeepX) xh[k] = h;
          dot += g.x * h.x + g.y * h.y + g.z * h.z + g.w * h.w;
        }
      }
    }
    dot = warp_sum(dot);
    if constexpr (WPR > 1) {
      if (lane == 0) sDot[warp] = dot;
      __syncthreads();
      dot = 0.f;
#pragma unroll
      for (int p = 0; p < WPR; ++p) dot += sDot[rrow * WPR + p];
    }
    if (live) {
      const float mean = dot / (float)H;
#pragma unroll
      for (int k = 0; k < G; ++k) {
        const int gi = 32 * part + lane + 32 * WPR * k;
        if (gi < ngroups) {
          const int c = 4 * gi;
          float4 h;
          if constexpr (kKeepX) {
            h = xh[k];
          } else {
            const float4 x = *reinterpret_cast<const float4*>(a.x + base + c);
            h = make_float4(x.x * rstd, x.y * rstd, x.z * rstd, x.w * rstd);
          }
          const float4 g = gv[k];
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
    __syncthreads();  // shared buffers are refilled by the next tile
  }
}

// Launch shape of both kernels for n rows of H columns: warps per row (wpr), rows per tile and
// grid, one CTA of up to 32 warps per SM. As many warps per row as still let the rows spread over
// one wave (4 for up to 8 rows per SM, 3 or 2 for up to 10 or 16, with G <= 4 / 8 groups per
// lane); past that, several waves of 8-row tiles with 4 warps per row. The row count per tile is
// then balanced so the tiles fill whole waves: ceil(n / (SMs x waves)). (Two CTAs of up to 16
// warps per SM measured slower: 16.8 / 19.5 us against 15.5 / 16.9 us for the forward / backward
// at 1,160 x 1,536.)
struct RmsShape {
  int wpr, rows, grid, G;
};

static RmsShape rms_shape(int64_t n, int H) {
  const int sms = sm_count();
  const int groups = H / 4;
  RmsShape r{1, RMS_MAXR, 0, 0};
  if (H >= 1024 && H <= 4096 && H % 128 == 0) {
    r.wpr = 4;
    r.rows = 8;
    if (n > (int64_t)sms * 8) {
      if (cdiv(groups, 96) <= 4 && n <= (int64_t)sms * 10) {
        r.wpr = 3;
        r.rows = 10;
      } else if (cdiv(groups, 64) <= 8 && n <= (int64_t)sms * 16) {
        r.wpr = 2;
        r.rows = 16;
      }
    }
  }
  const int64_t waves = cdiv(n, (int64_t)sms * r.rows);
  r.rows = (int)cdiv(n, (int64_t)sms * waves);
  if (r.wpr == 4 && n > (int64_t)sms * 16 && cdiv(groups, 64) <= 8) {
    // several waves: 8-row tiles of two warps per row (512 threads), two CTAs resident per SM,
    // so one tile's loads and stores overlap the other's arithmetic
    r.wpr = 2;
    r.rows = 8;
  }
  r.grid = (int)cdiv(n, r.rows);
  r.G = (int)cdiv(groups, 32 * r.wpr);
  return r;
}

// Opts a kernel into more than 48 KB of dynamic shared memory, once per kernel (and size).
template <typename K>
static void set_smem(K kern, int bytes) {
  if (bytes > 48 * 1024) smem_optin(reinterpret_cast<const void*>(kern), bytes);
}

// Instantiates kernel K<T, G, WPR> for the launch shape's (wpr, G) and launches it.
#define QL_RMS_DISPATCH(K, TT)                                                         \
  do {                                                                                 \
    if (sh.wpr == 4 && sh.G <= 4) QL_RMS_LAUNCH(K, TT, 4, 4);                          \
    else if (sh.wpr == 4) QL_RMS_LAUNCH(K, TT, 8, 4);                                  \
    else if (sh.wpr == 3) QL_RMS_LAUNCH(K, TT, 4, 3);                                  \
    else if (sh.wpr == 2) QL_RMS_LAUNCH(K, TT, 8, 2);                                  \
    else if (sh.G <= 4) QL_RMS_LAUNCH(K, TT, 4, 1);                                    \
    else if (sh.G <= 12) QL_RMS_LAUNCH(K, TT, 12, 1);                                  \
    else QL_RMS_LAUNCH(K, TT, 32, 1);                                                  \
  } while (0)
#define QL_RMS_LAUNCH(K, TT, GG, WW)                                                   \
  do {                                                                                 \
    set_smem(K<TT, GG, WW>, smem);                                                     \
    launch_k(K<TT, GG, WW>, dim3(sh.grid), dim3(32 * WW * sh.rows), smem, s, a, sh.rows); \
  } while (0)

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
                           c.p_keep, c.keep_scale, c.vec, c.drop_q, c.drop_v, FastDiv{}},
               c.drop_q ? c.keep_q : nullptr, c.drop_v ? c.keep_v : nullptr};
  if (c.vec != 4 && c.vec != 8) return QL_STATUS_BAD_ARG;
  if (!prepare_dropout(a.drop)) return QL_STATUS_BAD_ARG;
  const bool lora = (c.drop_q && c.Aq != nullptr) || (c.drop_v && c.Av != nullptr);
  if ((a.keep_q != nullptr || a.keep_v != nullptr) && c.H % 32 != 0) return QL_STATUS_BAD_ARG;
  if (lora && c.H % 16 != 0) return QL_STATUS_UNSUPPORTED;  // 16-column tensor-core K steps
  const RmsShape sh = rms_shape(c.n, c.H);
  // the dropped rows, then one [16 rows][16] partial per (adapter, K slice) work item: at most
  // max(warps, 2) items
  const int items = sh.rows * sh.wpr > 2 ? sh.rows * sh.wpr : 2;
  const int smem = lora ? 2 * sh.rows * (c.H + RMS_PAD) * 2 + items * RMS_MAXR * LORA_R * 4 : 0;
  if (c.dtype == QL_F16) QL_RMS_DISPATCH(rms_fwd_kernel, __half);
  else if (c.dtype == QL_BF16) QL_RMS_DISPATCH(rms_fwd_kernel, __nv_bfloat16);
  else return QL_STATUS_BAD_ARG;
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
                           c.p_keep, c.keep_scale, c.vec, c.drop_q, c.drop_v, FastDiv{}},
               c.keep_q, c.keep_v};
  if ((c.keep_q != nullptr || c.keep_v != nullptr) && c.H % 32 != 0) return QL_STATUS_BAD_ARG;
  if (!prepare_dropout(a.drop)) return QL_STATUS_BAD_ARG;
  const bool lora = (c.drop_q && c.tq == nullptr) || (c.drop_v && c.tv == nullptr);
  if (lora && c.H % 8 != 0) return QL_STATUS_UNSUPPORTED;  // 8-column tensor-core tiles
  const RmsShape sh = rms_shape(c.n, c.H);
  const int smem = lora ? 2 * sh.rows * (c.H + RMS_PAD) * 2 : 0;
  if (c.dtype == QL_F16) QL_RMS_DISPATCH(rms_bwd_kernel, __half);
  else if (c.dtype == QL_BF16) QL_RMS_DISPATCH(rms_bwd_kernel, __nv_bfloat16);
  else return QL_STATUS_BAD_ARG;
  return launched(1);
}
#undef QL_RMS_LAUNCH
#undef QL_RMS_DISPATCH

}  // namespace ql

namespace ql {

__global__ void dropout_keep_kernel(int8_t* out, int64_t nelem, DropoutArgs d) {
  pdl_enter();
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
