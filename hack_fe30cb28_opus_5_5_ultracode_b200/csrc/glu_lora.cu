// SwiGLU over the fused [gate | up] GEMM output, the LoRA weight-gradient reductions, and the
// embedding gather.
//
// glu_fwd (reference glu_fwd_kernel, solution/kernels.py:312-321): m = silu(g) * u in fp32.
// glu_bwd (reference glu_bwd_kernel, solution/kernels.py:324-336): in place,
//   [g | u] <- [dm * u * sig * (1 + g * (1 - sig)) | dm * g * sig].
// Both stream 16-byte vectors: HBM-bound (fwd reads 4 B and writes 2 B per element of m, bwd
// reads 6 B and writes 4 B).
//
// lora_colsum: out[i, r] (or out[r, i]) = scale * sum_t X[t, i] * Y[t, r], the LoRA weight
// gradients dB = s g^T x_lo and dA = dx_lo^T drop(a) (solution/engine.py:1322-1328), as a
// deterministic two-stage column reduction over the tokens (per-split partials in a caller
// workspace, then a fixed-order sum).
#include "common.cuh"
#include "profile.h"
#include "ops.h"

namespace ql {

template <typename T>
__global__ void glu_fwd_kernel(const T* __restrict__ gu, T* __restrict__ m, int64_t n, int I) {
  const int64_t per_row = I / 8;
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= n * per_row) return;
  const int64_t row = idx / per_row, c = (idx % per_row) * 8;
  const uint4 gv = *reinterpret_cast<const uint4*>(gu + row * 2 * I + c);
  const uint4 uv = *reinterpret_cast<const uint4*>(gu + row * 2 * I + I + c);
  const T* g = reinterpret_cast<const T*>(&gv);
  const T* u = reinterpret_cast<const T*>(&uv);
  T o[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float gf = to_f<T>(g[j]);
    o[j] = from_f<T>(gf / (1.0f + __expf(-gf)) * to_f<T>(u[j]));
  }
  *reinterpret_cast<uint4*>(m + row * I + c) = *reinterpret_cast<const uint4*>(o);
}

template <typename T>
__global__ void glu_bwd_kernel(const T* __restrict__ dm, T* __restrict__ gu, int64_t n, int I) {
  const int64_t per_row = I / 8;
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= n * per_row) return;
  const int64_t row = idx / per_row, c = (idx % per_row) * 8;
  T* gp = gu + row * 2 * I + c;
  T* up = gp + I;
  const uint4 gv = *reinterpret_cast<const uint4*>(gp);
  const uint4 uv = *reinterpret_cast<const uint4*>(up);
  const uint4 dv = *reinterpret_cast<const uint4*>(dm + row * I + c);
  const T* g = reinterpret_cast<const T*>(&gv);
  const T* u = reinterpret_cast<const T*>(&uv);
  const T* d = reinterpret_cast<const T*>(&dv);
  T og[8], ou[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float gf = to_f<T>(g[j]), uf = to_f<T>(u[j]), df = to_f<T>(d[j]);
    const float sig = 1.0f / (1.0f + __expf(-gf));
    og[j] = from_f<T>(df * uf * sig * (1.0f + gf * (1.0f - sig)));
    ou[j] = from_f<T>(df * gf * sig);
  }
  *reinterpret_cast<uint4*>(gp) = *reinterpret_cast<const uint4*>(og);
  *reinterpret_cast<uint4*>(up) = *reinterpret_cast<const uint4*>(ou);
}

int glu_fwd(const void* gu, void* m, int64_t n, int I, int dtype, cudaStream_t s) {
  if (n < 0 || I <= 0 || I % 8 != 0) return QL_STATUS_BAD_ARG;
  if (n == 0) return QL_STATUS_OK;
  ProfScope prof(PK_GLU_FWD, 0, (double)n * I * 6, s);
  const int64_t work = n * (I / 8);
  const unsigned grid = (unsigned)cdiv(work, 256);
  if (dtype == QL_F16)
    glu_fwd_kernel<__half><<<grid, 256, 0, s>>>((const __half*)gu, (__half*)m, n, I);
  else if (dtype == QL_BF16)
    glu_fwd_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)gu, (__nv_bfloat16*)m, n, I);
  else return QL_STATUS_BAD_ARG;
  return launched(1);
}

int glu_bwd(const void* dm, void* gu, int64_t n, int I, int dtype, cudaStream_t s) {
  if (n < 0 || I <= 0 || I % 8 != 0) return QL_STATUS_BAD_ARG;
  if (n == 0) return QL_STATUS_OK;
  ProfScope prof(PK_GLU_BWD, 0, (double)n * I * 10, s);
  const int64_t work = n * (I / 8);
  const unsigned grid = (unsigned)cdiv(work, 256);
  if (dtype == QL_F16)
    glu_bwd_kernel<__half><<<grid, 256, 0, s>>>((const __half*)dm, (__half*)gu, n, I);
  else if (dtype == QL_BF16)
    glu_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)dm, (__nv_bfloat16*)gu, n, I);
  else return QL_STATUS_BAD_ARG;
  return launched(1);
}

// ---------------------------------------------------------------------------------------------
// LoRA weight gradients
// ---------------------------------------------------------------------------------------------
constexpr int CS_COLS = 64, CS_TOK = 32, CS_R = 16, CS_THREADS = 256;

__device__ __forceinline__ void cs_cp16(void* smem, const void* gmem, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(pred ? 16 : 0)
               : "memory");
}

// Stage 1: split blockIdx.y of the tokens, columns [blockIdx.x * 64, +64): partial[sp][i][r].
// Tiles of 32 tokens x 64 columns of X and 32 x 16 of Y are staged by cp.async (double buffered,
// every load of a tile in flight at once); thread t accumulates column t % 64 for 4 of the 16 r.
template <typename TX, typename TY>
__global__ void __launch_bounds__(CS_THREADS) colsum_kernel(const TX* __restrict__ X, int64_t ldx,
                                                             const TY* __restrict__ Y, int64_t n,
                                                             int ncols, int64_t tok_per_split,
                                                             float* __restrict__ partial) {
  __shared__ __align__(16) TX xs[2][CS_TOK][CS_COLS];
  __shared__ __align__(16) TY ys[2][CS_TOK][CS_R];
  const int c0 = blockIdx.x * CS_COLS;
  const int64_t t0 = blockIdx.y * tok_per_split;
  const int64_t t1 = min(n, t0 + tok_per_split);
  const int c = threadIdx.x % CS_COLS, rg = threadIdx.x / CS_COLS;  // rg: r = 4 rg .. 4 rg + 3
  constexpr int XCH = CS_TOK * CS_COLS * sizeof(TX) / 16;  // 16-byte chunks of an X tile
  constexpr int YCH = CS_TOK * CS_R * sizeof(TY) / 16;
  constexpr int XPR = CS_COLS * sizeof(TX) / 16;           // chunks per X row
  constexpr int YPR = CS_R * sizeof(TY) / 16;
  auto load = [&](int buf, int64_t tb) {
    for (int i = threadIdx.x; i < XCH; i += CS_THREADS) {
      const int tt = i / XPR, ch = i % XPR;
      const int col = c0 + ch * (16 / (int)sizeof(TX));
      const bool ok = tb + tt < t1 && col < ncols;
      cs_cp16(&xs[buf][tt][ch * (16 / sizeof(TX))], ok ? X + (tb + tt) * ldx + col : X, ok);
    }
    for (int i = threadIdx.x; i < YCH; i += CS_THREADS) {
      const int tt = i / YPR, ch = i % YPR;
      const bool ok = tb + tt < t1;
      cs_cp16(&ys[buf][tt][ch * (16 / sizeof(TY))], ok ? Y + (tb + tt) * CS_R + ch * (16 / sizeof(TY)) : Y, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  int buf = 0;
  if (t0 < t1) load(0, t0);
  for (int64_t tb = t0; tb < t1; tb += CS_TOK) {
    if (tb + CS_TOK < t1) {
      load(buf ^ 1, tb + CS_TOK);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
#pragma unroll 8
    for (int tt = 0; tt < CS_TOK; ++tt) {
      const float x = to_f<TX>(xs[buf][tt][c]);
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] += x * to_f<TY>(ys[buf][tt][4 * rg + j]);
    }
    __syncthreads();  // the buffer is refilled next iteration
    buf ^= 1;
  }
  if (c0 + c < ncols) {
    float* p = partial + ((int64_t)blockIdx.y * ncols + c0 + c) * CS_R + 4 * rg;
    *reinterpret_cast<float4*>(p) = make_float4(acc[0], acc[1], acc[2], acc[3]);
  }
}

// Stage 2: out = scale * sum over splits (fixed order), as [ncols, R] or transposed [R, ncols].
__global__ void colsum_reduce_kernel(const float* __restrict__ partial, int splits, int ncols,
                                     float scale, int transpose, float* __restrict__ out) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= (int64_t)ncols * CS_R) return;
  float s = 0.f;
  for (int sp = 0; sp < splits; ++sp) s += partial[(int64_t)sp * ncols * CS_R + idx];
  const int i = (int)(idx / CS_R), r = (int)(idx % CS_R);
  if (transpose) out[(int64_t)r * ncols + i] = s * scale;
  else out[idx] = s * scale;
}

int lora_colsum_splits(int64_t n, int ncols) {
  // about 4 CTAs per SM of 148, at least 32 tokens per split, at most 64 splits
  const int64_t colblocks = cdiv(ncols, CS_COLS);
  int64_t s = cdiv(592, colblocks);
  const int64_t by_tokens = cdiv(n, CS_TOK);
  if (s > by_tokens) s = by_tokens;
  if (s > 64) s = 64;
  return (int)(s < 1 ? 1 : s);
}

int lora_colsum(const void* X, int64_t ldx, int x_dtype, const void* Y, int y_dtype, int64_t n,
                int ncols, int rank, float scale, int transpose, float* out, float* workspace,
                int64_t workspace_floats, cudaStream_t s) {
  if (rank != CS_R) return QL_STATUS_UNSUPPORTED;
  if (n < 0 || ncols <= 0) return QL_STATUS_BAD_ARG;
  // 16-byte staging: aligned bases and row strides, whole 8-column groups
  if (reinterpret_cast<uintptr_t>(X) % 16 != 0 || reinterpret_cast<uintptr_t>(Y) % 16 != 0 ||
      ldx % 8 != 0 || ncols % 8 != 0)
    return QL_STATUS_BAD_ARG;
  const int splits = lora_colsum_splits(n, ncols);
  if (workspace_floats < (int64_t)splits * ncols * CS_R) return QL_STATUS_BAD_ARG;
  ProfScope prof(PK_COLSUM, 2.0 * n * ncols * CS_R, (double)n * ncols * 2, s);
  const int64_t per = cdiv(cdiv(n > 0 ? n : 1, splits), CS_TOK) * CS_TOK;
  dim3 grid((unsigned)cdiv(ncols, CS_COLS), (unsigned)splits);
#define QL_COLSUM(TX, TY) \
  colsum_kernel<TX, TY><<<grid, CS_THREADS, 0, s>>>((const TX*)X, ldx, (const TY*)Y, n, ncols, per, workspace)
  if (x_dtype == QL_F16 && y_dtype == QL_F16) QL_COLSUM(__half, __half);
  else if (x_dtype == QL_F16 && y_dtype == QL_F32) QL_COLSUM(__half, float);
  else if (x_dtype == QL_BF16 && y_dtype == QL_BF16) QL_COLSUM(__nv_bfloat16, __nv_bfloat16);
  else if (x_dtype == QL_BF16 && y_dtype == QL_F32) QL_COLSUM(__nv_bfloat16, float);
  else return QL_STATUS_BAD_ARG;
#undef QL_COLSUM
  const int64_t total = (int64_t)ncols * CS_R;
  colsum_reduce_kernel<<<(unsigned)cdiv(total, 256), 256, 0, s>>>(workspace, splits, ncols, scale,
                                                                  transpose, out);
  return launched(2);
}

// ---------------------------------------------------------------------------------------------
// embedding gather: h[t, :] = float(W[ids[t], :])
// ---------------------------------------------------------------------------------------------
template <typename T>
__global__ void embed_kernel(const int64_t* __restrict__ ids, const T* __restrict__ W,
                             float* __restrict__ h, int64_t n, int H, int64_t vocab, int* err) {
  const int64_t t = blockIdx.x;
  const int64_t id = ids[t];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) raise_status(err, QL_STATUS_BAD_ARG);
    for (int c = threadIdx.x; c < H; c += blockDim.x) h[t * H + c] = 0.f;
    return;
  }
  for (int c = threadIdx.x; c < H; c += blockDim.x) h[t * H + c] = to_f<T>(W[id * H + c]);
}

int embed(const int64_t* ids, const void* W, float* h, int64_t n, int H, int64_t vocab,
          int dtype, int* err, cudaStream_t s) {
  if (n < 0 || H <= 0) return QL_STATUS_BAD_ARG;
  if (n == 0) return QL_STATUS_OK;
  if (dtype == QL_F16) embed_kernel<__half><<<n, 256, 0, s>>>(ids, (const __half*)W, h, n, H, vocab, err);
  else if (dtype == QL_BF16)
    embed_kernel<__nv_bfloat16><<<n, 256, 0, s>>>(ids, (const __nv_bfloat16*)W, h, n, H, vocab, err);
  else return QL_STATUS_BAD_ARG;
  return launched(1);
}

}  // namespace ql

namespace ql {

// ---------------------------------------------------------------------------------------------
// row permutations of the head (rows with a target first, solution/engine.py:731, 1364-1398)
// ---------------------------------------------------------------------------------------------
__global__ void gather_rows_kernel(const float* __restrict__ src, const int64_t* __restrict__ idx,
                                   float* __restrict__ dst, int H) {
  const int64_t r = blockIdx.x;
  const float4* s = reinterpret_cast<const float4*>(src + idx[r] * H);
  float4* d = reinterpret_cast<float4*>(dst + r * H);
  for (int c = threadIdx.x; c < H / 4; c += blockDim.x) d[c] = s[c];
}

template <typename T>
__global__ void scatter_rows_kernel(const float* __restrict__ src, const int64_t* __restrict__ idx,
                                    const float* __restrict__ scale, float* __restrict__ dst,
                                    T* __restrict__ dst16, int H) {
  const int64_t r = blockIdx.x;
  const float s = scale != nullptr ? *scale : 1.f;
  const int64_t o = idx[r] * H;
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    const float v = src[r * H + c] * s;
    dst[o + c] = v;
    if (dst16 != nullptr) dst16[o + c] = from_f<T>(v);
  }
}

int gather_rows(const float* src, const int64_t* idx, float* dst, int64_t n, int H, cudaStream_t s) {
  if (n < 0 || H <= 0 || H % 4 != 0) return QL_STATUS_BAD_ARG;
  if (n == 0) return QL_STATUS_OK;
  gather_rows_kernel<<<n, 128, 0, s>>>(src, idx, dst, H);
  return launched(1);
}

int scatter_rows(const float* src, const int64_t* idx, const float* scale, float* dst, void* dst16,
                 int64_t n, int H, int dtype, cudaStream_t s) {
  if (n < 0 || H <= 0) return QL_STATUS_BAD_ARG;
  if (n == 0) return QL_STATUS_OK;
  if (dtype == QL_F16) scatter_rows_kernel<__half><<<n, 128, 0, s>>>(src, idx, scale, dst, (__half*)dst16, H);
  else if (dtype == QL_BF16)
    scatter_rows_kernel<__nv_bfloat16><<<n, 128, 0, s>>>(src, idx, scale, dst, (__nv_bfloat16*)dst16, H);
  else return QL_STATUS_BAD_ARG;
  return launched(1);
}

}  // namespace ql
