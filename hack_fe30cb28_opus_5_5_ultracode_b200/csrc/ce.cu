// Cross-entropy, entropy and argmax over a 151,936-word vocabulary without fp32 logits.
//
// ce_rows (reference lm_head_ce_kernel, solution/kernels.py:344-388): one CTA per row of 16-bit
// logits. One online pass keeps (max, sum exp, sum exp * x, best, argmax) per thread — merged
// across the CTA, first maximum wins — giving lse, entropy = lse - sum(p x), the loss lse - x_t
// and accuracy; a second pass writes softmax - onehot over the row in place (unscaled), or zeros
// for a row without a target when asked. The target logit is read before any thread writes.
//
// ce_piece / ce_finish (reference lm_head_piece_kernel / lm_head_finish_kernel,
// solution/kernels.py:401-479): the same statistics carried across vocabulary pieces in a
// [rows, 4] state (max, sum exp, sum exp * x, best) plus the argmax; rows with a target get
// exp(x - running max) written over their logits for the gradient GEMM and the rescale factor
// alpha = exp(old max - new max); the target's weight row is copied out when it falls in the
// piece; optionally the fp32 gradient accumulator is moved to the new max in the same pass,
// acc = alpha (acc + part), folding in the previous piece's product `part` (so the product GEMM
// never reads its output and keeps its split-K); finish forms loss, entropy, accuracy and
// dh = (acc + part) / s - W_target.
#include <math_constants.h>

#include "common.cuh"
#include "profile.h"
#include "ops.h"

namespace ql {

constexpr int CE_THREADS = 512;

struct OnlineStat {
  float m, s, t, best;
  int64_t arg;
};

__device__ __forceinline__ void stat_merge(OnlineStat& a, const OnlineStat& b) {
  const float m = fmaxf(a.m, b.m);
  const float fa = a.m == -CUDART_INF_F ? 0.f : __expf(a.m - m);
  const float fb = b.m == -CUDART_INF_F ? 0.f : __expf(b.m - m);
  a.s = a.s * fa + b.s * fb;
  a.t = a.t * fa + b.t * fb;
  a.m = m;
  if (b.best > a.best || (b.best == a.best && b.arg < a.arg)) {
    a.best = b.best;
    a.arg = b.arg;
  }
}

__device__ __forceinline__ void stat_add(OnlineStat& st, float x, int64_t col) {
  if (x > st.best) {  // columns arrive in increasing order per thread: first max wins
    st.best = x;
    st.arg = col;
  }
  if (x > st.m) {
    const float f = st.m == -CUDART_INF_F ? 0.f : __expf(st.m - x);
    st.s *= f;
    st.t *= f;
    st.m = x;
  }
  const float e = __expf(x - st.m);
  st.s += e;
  st.t += e * x;
}

__device__ OnlineStat block_merge(OnlineStat st, OnlineStat* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    OnlineStat b;
    b.m = __shfl_xor_sync(0xffffffffu, st.m, o);
    b.s = __shfl_xor_sync(0xffffffffu, st.s, o);
    b.t = __shfl_xor_sync(0xffffffffu, st.t, o);
    b.best = __shfl_xor_sync(0xffffffffu, st.best, o);
    b.arg = __shfl_xor_sync(0xffffffffu, st.arg, o);
    stat_merge(st, b);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) sh[warp] = st;
  __syncthreads();
  OnlineStat r = sh[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) stat_merge(r, sh[w]);
  return r;
}

// Online statistics of row [0, width) of src, columns offset by v0 for the argmax.
template <typename T>
__device__ __forceinline__ OnlineStat row_stats(const T* src, int64_t width, int64_t v0) {
  OnlineStat st{-CUDART_INF_F, 0.f, 0.f, -CUDART_INF_F, 0};
  const bool vec = (reinterpret_cast<uintptr_t>(src) % 16 == 0);
  if (vec) {
    const int64_t nvec = width / 8;
    for (int64_t i = threadIdx.x; i < nvec; i += blockDim.x) {
      const uint4 u = *reinterpret_cast<const uint4*>(src + i * 8);
      const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) stat_add(st, to_f<T>(h[j]), v0 + i * 8 + j);
    }
    for (int64_t c = nvec * 8 + threadIdx.x; c < width; c += blockDim.x) stat_add(st, to_f<T>(src[c]), v0 + c);
  } else {
    for (int64_t c = threadIdx.x; c < width; c += blockDim.x) stat_add(st, to_f<T>(src[c]), v0 + c);
  }
  return st;
}

template <typename T>
__global__ void __launch_bounds__(CE_THREADS) ce_rows_kernel(CeRowsC a) {
  pdl_enter();
  __shared__ OnlineStat sh[CE_THREADS / 32];
  __shared__ float xt_sh;
  const int64_t row = blockIdx.x;
  T* src = reinterpret_cast<T*>(a.logits) + row * a.ld;
  const int64_t target = a.target[row];
  const bool valid = target >= 0 && target < a.V;
  if (threadIdx.x == 0) xt_sh = valid ? to_f<T>(src[target]) : 0.f;
  OnlineStat st = row_stats<T>(src, a.V, 0);
  st = block_merge(st, sh);  // (its __syncthreads also publish xt_sh)
  const float lse = st.m + logf(st.s);
  if (threadIdx.x == 0) {
    a.entropy[row] = lse - st.t / st.s;
    a.loss[row] = valid ? lse - xt_sh : 0.f;
    a.correct[row] = (valid && st.arg == target) ? 1 : 0;
  }
  if (valid && a.write_grad) {
    for (int64_t c = threadIdx.x; c < a.V; c += blockDim.x) {
      const float x = to_f<T>(src[c]);
      src[c] = from_f<T>(__expf(x - lse) - (c == target ? 1.f : 0.f));
    }
  } else if (!valid && a.zero_unsupervised) {
    for (int64_t c = threadIdx.x; c < a.V; c += blockDim.x) src[c] = from_f<T>(0.f);
  }
}

// Adds 8 consecutive logits (columns col0 .. col0+7, in increasing order) to a running state:
// one rescale for the group's maximum, then the exponentials against it; the first maximum
// keeps the argmax.
__device__ __forceinline__ void stat_add8(OnlineStat& st, const float* v, int64_t col0) {
  float m8 = v[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) m8 = fmaxf(m8, v[j]);
  if (m8 > st.m) {
    const float f = st.m == -CUDART_INF_F ? 0.f : __expf(st.m - m8);
    st.s *= f;
    st.t *= f;
    st.m = m8;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (v[j] > st.best) {
      st.best = v[j];
      st.arg = col0 + j;
    }
    const float e = __expf(v[j] - st.m);
    st.s += e;
    st.t += e * v[j];
  }
}

__device__ __forceinline__ OnlineStat warp_merge(OnlineStat st) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    OnlineStat b;
    b.m = __shfl_xor_sync(0xffffffffu, st.m, o);
    b.s = __shfl_xor_sync(0xffffffffu, st.s, o);
    b.t = __shfl_xor_sync(0xffffffffu, st.t, o);
    b.best = __shfl_xor_sync(0xffffffffu, st.best, o);
    b.arg = __shfl_xor_sync(0xffffffffu, st.arg, o);
    stat_merge(st, b);
  }
  return st;
}

constexpr int CE_PIECE_THREADS = 128;  // per row: a CTA of 4 warps (~8 CTAs, 32 warps per SM)
constexpr int CE_PIECE_UNROLL = 4;     // 16-byte vectors each thread has in flight

// One CTA of 4 warps per row of a vocabulary piece: each thread walks the row in 8-column vectors
// (16-byte loads, four in flight) with its own running state; the states are merged across the
// warp, the CTA and into the row's state from the earlier pieces. Then, for rows with a target,
// exp(x - new max) over the row in place, and the fp32 gradient accumulator moved to the new max
// (acc = alpha (acc + part)).
template <typename T>
__global__ void __launch_bounds__(CE_PIECE_THREADS) ce_piece_kernel(CePieceC a) {
  pdl_enter();
  __shared__ OnlineStat sh[CE_PIECE_THREADS / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row = blockIdx.x;
  T* src = reinterpret_cast<T*>(a.logits) + row * a.ld;
  const int64_t target = a.target[row];
  const int64_t local = target - a.v0;
  const bool here = target >= 0 && local >= 0 && local < a.width;
  const float xt = here ? to_f<T>(src[local]) : 0.f;  // read before the row is overwritten
  OnlineStat st{-CUDART_INF_F, 0.f, 0.f, -CUDART_INF_F, 0};
  const bool vec = (reinterpret_cast<uintptr_t>(src) % 16 == 0);
  const int64_t nvec = vec ? a.width / 8 : 0;
  constexpr int STEP = CE_PIECE_THREADS * CE_PIECE_UNROLL;
  for (int64_t i0 = threadIdx.x; i0 < nvec; i0 += STEP) {
    uint4 u[CE_PIECE_UNROLL];
#pragma unroll
    for (int k = 0; k < CE_PIECE_UNROLL; ++k) {
      const int64_t i = i0 + (int64_t)k * CE_PIECE_THREADS;
      if (i < nvec) u[k] = *reinterpret_cast<const uint4*>(src + i * 8);
    }
#pragma unroll
    for (int k = 0; k < CE_PIECE_UNROLL; ++k) {
      const int64_t i = i0 + (int64_t)k * CE_PIECE_THREADS;
      if (i < nvec) {
        const T* h = reinterpret_cast<const T*>(&u[k]);
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = to_f<T>(h[j]);
        stat_add8(st, v, a.v0 + i * 8);
      }
    }
  }
  for (int64_t c = nvec * 8 + threadIdx.x; c < a.width; c += CE_PIECE_THREADS)
    stat_add(st, to_f<T>(src[c]), a.v0 + c);
  st = warp_merge(st);
  if (lane == 0) sh[warp] = st;
  __syncthreads();
  st = sh[0];
#pragma unroll
  for (int w = 1; w < CE_PIECE_THREADS / 32; ++w) stat_merge(st, sh[w]);
  OnlineStat prev{a.state[row * 4], a.state[row * 4 + 1], a.state[row * 4 + 2],
                  a.state[row * 4 + 3], a.best_idx[row]};
  const float m_old = prev.m;
  // earlier pieces hold smaller columns, so on a tie the earlier maximum stays (stat_merge)
  stat_merge(prev, st);
  st = prev;
  __syncthreads();  // every thread has read the row state before thread 0 rewrites it
  if (threadIdx.x == 0) {
    a.state[row * 4] = st.m;
    a.state[row * 4 + 1] = st.s;
    a.state[row * 4 + 2] = st.t;
    a.state[row * 4 + 3] = st.best;
    a.best_idx[row] = st.arg;
    if (here) a.xt[row] = xt;
    if (row < a.n_sup) a.alpha[row] = m_old == -CUDART_INF_F ? 0.f : __expf(m_old - st.m);
  }
  if (here && a.wt != nullptr) {
    const T* w = reinterpret_cast<const T*>(a.w) + local * a.H;
    T* dst = reinterpret_cast<T*>(a.wt) + row * a.H;
    for (int c = threadIdx.x; c < a.H; c += CE_PIECE_THREADS) dst[c] = w[c];
  }
  if (row < a.n_sup) {
    const float m = st.m;
    for (int64_t i0 = threadIdx.x; i0 < nvec; i0 += STEP) {
      uint4 u[CE_PIECE_UNROLL];
#pragma unroll
      for (int k = 0; k < CE_PIECE_UNROLL; ++k) {
        const int64_t i = i0 + (int64_t)k * CE_PIECE_THREADS;
        if (i < nvec) u[k] = *reinterpret_cast<const uint4*>(src + i * 8);
      }
#pragma unroll
      for (int k = 0; k < CE_PIECE_UNROLL; ++k) {
        const int64_t i = i0 + (int64_t)k * CE_PIECE_THREADS;
        if (i < nvec) {
          T* h = reinterpret_cast<T*>(&u[k]);
#pragma unroll
          for (int j = 0; j < 8; ++j) h[j] = from_f<T>(__expf(to_f<T>(h[j]) - m));
          *reinterpret_cast<uint4*>(src + i * 8) = u[k];
        }
      }
    }
    for (int64_t c = nvec * 8 + threadIdx.x; c < a.width; c += CE_PIECE_THREADS)
      src[c] = from_f<T>(__expf(to_f<T>(src[c]) - m));
    if (a.acc != nullptr) {
      // the gradient accumulator, moved to this piece's running max: acc = alpha (acc + part),
      // part being the previous piece's product (when part_valid); zero before the first piece
      float* acc = a.acc + row * a.H;
      const float* part = a.part_valid ? a.part + row * a.H : nullptr;
      const float alpha = m_old == -CUDART_INF_F ? 0.f : __expf(m_old - m);
      for (int c = threadIdx.x; c < a.H; c += CE_PIECE_THREADS) {
        if (m_old == -CUDART_INF_F) acc[c] = 0.f;
        else acc[c] = alpha * (acc[c] + (part != nullptr ? part[c] : 0.f));
      }
    }
  }
}

template <typename T>
__global__ void ce_finish_kernel(CeFinishC a) {
  pdl_enter();
  const int64_t row = blockIdx.x;
  const float m = a.state[row * 4], s = a.state[row * 4 + 1], t = a.state[row * 4 + 2];
  const float lse = m + logf(s);
  const int64_t target = a.target[row];
  const bool valid = target >= 0;
  if (threadIdx.x == 0) {
    a.entropy[row] = lse - t / s;
    a.loss[row] = valid ? lse - a.xt[row] : 0.f;
    a.correct[row] = (valid && a.best_idx[row] == target) ? 1 : 0;
  }
  if (row < a.n_sup) {
    const float* acc = a.acc + row * a.H;
    const float* part = a.part != nullptr ? a.part + row * a.H : nullptr;
    const T* wt = reinterpret_cast<const T*>(a.wt) + row * a.H;
    T* dh = reinterpret_cast<T*>(a.dh) + row * a.H;
    for (int c = threadIdx.x; c < a.H; c += blockDim.x)
      dh[c] = from_f<T>((acc[c] + (part != nullptr ? part[c] : 0.f)) / s - to_f<T>(wt[c]));
  }
}

int ce_rows(const CeRowsC& a, cudaStream_t s) {
  if (a.rows < 0 || a.V <= 0 || a.ld < a.V) return QL_STATUS_BAD_ARG;
  if (a.rows == 0) return QL_STATUS_OK;
  ProfScope prof(PK_CE, 0, (double)a.rows * a.V * 2 * (a.write_grad ? 3 : 1), s);
  if (a.dtype == QL_F16) ce_rows_kernel<__half><<<a.rows, CE_THREADS, 0, s>>>(a);
  else if (a.dtype == QL_BF16) ce_rows_kernel<__nv_bfloat16><<<a.rows, CE_THREADS, 0, s>>>(a);
  else return QL_STATUS_BAD_ARG;
  return launched(1);
}

int ce_piece(const CePieceC& a, cudaStream_t s) {
  if (a.rows < 0 || a.width <= 0 || a.ld < a.width || a.H <= 0) return QL_STATUS_BAD_ARG;
  if (a.part_valid && (a.acc == nullptr || a.part == nullptr)) return QL_STATUS_BAD_ARG;
  if (a.rows == 0) return QL_STATUS_OK;
  ProfScope prof(PK_CE, 0, (double)a.rows * a.width * 2 + (double)a.n_sup * a.width * 2 +
                               (a.acc != nullptr ? (double)a.n_sup * a.H * (a.part_valid ? 12 : 4) : 0),
                 s);
  const unsigned grid = (unsigned)a.rows;
  if (a.dtype == QL_F16) launch_k(ce_piece_kernel<__half>, dim3(grid), dim3(CE_PIECE_THREADS), 0, s, a);
  else if (a.dtype == QL_BF16) launch_k(ce_piece_kernel<__nv_bfloat16>, dim3(grid), dim3(CE_PIECE_THREADS), 0, s, a);
  else return QL_STATUS_BAD_ARG;
  return launched(1);
}

int ce_finish(const CeFinishC& a, cudaStream_t s) {
  if (a.rows < 0 || a.H <= 0) return QL_STATUS_BAD_ARG;
  if (a.rows == 0) return QL_STATUS_OK;
  ProfScope prof(PK_CE, 0, (double)a.n_sup * a.H * (4 + (a.part != nullptr ? 4 : 0) + 2 + 2), s);
  if (a.dtype == QL_F16) ce_finish_kernel<__half><<<a.rows, 256, 0, s>>>(a);
  else if (a.dtype == QL_BF16) ce_finish_kernel<__nv_bfloat16><<<a.rows, 256, 0, s>>>(a);
  else return QL_STATUS_BAD_ARG;
  return launched(1);
}

}  // namespace ql
