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
  const int64_t work = n * (I / 8);
  const unsigned grid = (unsigned)cdiv(work, 256);
  if (dtype == QL_F16)
    glu_fwd_kernel<__half><<<grid, 256, 0, s>>>((const __half*)gu, (__half*)m, n, I);
  else if (dtype == QL_BF16)
    glu_fwd_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)gu, (__nv_bfloat16*)m, n, I);
  else return QL_STATUS_BAD_ARG;
  return cudaPeekAtLastError() == cudaSuccess ? QL_STATUS_OK : QL_STATUS_CUDA;
}

int glu_bwd(const void* dm, void* gu, int64_t n, int I, int dtype, cudaStream_t s) {
  if (n < 0 || I <= 0 || I % 8 != 0) return QL_STATUS_BAD_ARG;
  if (n == 0) return QL_STATUS_OK;
  const int64_t work = n * (I / 8);
  const unsigned grid = (unsigned)cdiv(work, 256);
  if (dtype == QL_F16)
    glu_bwd_kernel<__half><<<grid, 256, 0, s>>>((const __half*)dm, (__half*)gu, n, I);
  else if (dtype == QL_BF16)
    glu_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)dm, (__nv_bfloat16*)gu, n, I);
  else return QL_STATUS_BAD_ARG;
  return cudaPeekAtLastError() == cudaSuccess ? QL_STATUS_OK : QL_STATUS_CUDA;
}

// ---------------------------------------------------------------------------------------------
// LoRA weight gradients
// ---------------------------------------------------------------------------------------------
constexpr int CS_COLS = 128, CS_TOK = 64, CS_R = 16;

// Stage 1: split `sp` of the tokens, columns [blockIdx.x * 128, +128): partial[sp][i][r].
template <typename TX, typename TY>
__global__ void __launch_bounds__(CS_COLS) colsum_kernel(const TX* __restrict__ X, int64_t ldx,
                                                          const TY* __restrict__ Y, int64_t n,
                                                          int ncols, int64_t tok_per_split,
                                                          float* __restrict__ partial) {
  __shared__ float ys[CS_TOK][CS_R];
  const int i = blockIdx.x * CS_COLS + threadIdx.x;
  const int64_t t0 = blockIdx.y * tok_per_split;
  const int64_t t1 = min(n, t0 + tok_per_split);
  float acc[CS_R];
#pragma unroll
  for (int r = 0; r < CS_R; ++r) acc[r] = 0.f;
  for (int64_t tb = t0; tb < t1; tb += CS_TOK) {
    const int cnt = (int)min((int64_t)CS_TOK, t1 - tb);
    __syncthreads();
    for (int j = threadIdx.x; j < CS_TOK * CS_R; j += CS_COLS) {
      const int tt = j / CS_R, r = j % CS_R;
      ys[tt][r] = tt < cnt ? to_f<TY>(Y[(tb + tt) * CS_R + r]) : 0.f;
    }
    __syncthreads();
    if (i < ncols) {
      for (int tt = 0; tt < cnt; ++tt) {
        const float x = to_f<TX>(X[(tb + tt) * ldx + i]);
#pragma unroll
        for (int r = 0; r < CS_R; ++r) acc[r] += x * ys[tt][r];
      }
    }
  }
  if (i < ncols) {
    float* p = partial + ((int64_t)blockIdx.y * ncols + i) * CS_R;
#pragma unroll
    for (int r = 0; r < CS_R; ++r) p[r] = acc[r];
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

int lora_colsum_splits(int64_t n) {
  const int64_t s = cdiv(n, 128);
  return (int)(s < 1 ? 1 : (s > 64 ? 64 : s));
}

int lora_colsum(const void* X, int64_t ldx, int x_dtype, const void* Y, int y_dtype, int64_t n,
                int ncols, int rank, float scale, int transpose, float* out, float* workspace,
                int64_t workspace_floats, cudaStream_t s) {
  if (rank != CS_R) return QL_STATUS_UNSUPPORTED;
  if (n < 0 || ncols <= 0) return QL_STATUS_BAD_ARG;
  const int splits = lora_colsum_splits(n);
  if (workspace_floats < (int64_t)splits * ncols * CS_R) return QL_STATUS_BAD_ARG;
  const int64_t per = cdiv(n > 0 ? n : 1, splits);
  dim3 grid((unsigned)cdiv(ncols, CS_COLS), (unsigned)splits);
#define QL_COLSUM(TX, TY) \
  colsum_kernel<TX, TY><<<grid, CS_COLS, 0, s>>>((const TX*)X, ldx, (const TY*)Y, n, ncols, per, workspace)
  if (x_dtype == QL_F16 && y_dtype == QL_F16) QL_COLSUM(__half, __half);
  else if (x_dtype == QL_F16 && y_dtype == QL_F32) QL_COLSUM(__half, float);
  else if (x_dtype == QL_BF16 && y_dtype == QL_BF16) QL_COLSUM(__nv_bfloat16, __nv_bfloat16);
  else if (x_dtype == QL_BF16 && y_dtype == QL_F32) QL_COLSUM(__nv_bfloat16, float);
  else return QL_STATUS_BAD_ARG;
#undef QL_COLSUM
  const int64_t total = (int64_t)ncols * CS_R;
  colsum_reduce_kernel<<<(unsigned)cdiv(total, 256), 256, 0, s>>>(workspace, splits, ncols, scale,
                                                                  transpose, out);
  return cudaPeekAtLastError() == cudaSuccess ? QL_STATUS_OK : QL_STATUS_CUDA;
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
  return cudaPeekAtLastError() == cudaSuccess ? QL_STATUS_OK : QL_STATUS_CUDA;
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
  return cudaPeekAtLastError() == cudaSuccess ? QL_STATUS_OK : QL_STATUS_CUDA;
}

int scatter_rows(const float* src, const int64_t* idx, const float* scale, float* dst, void* dst16,
                 int64_t n, int H, int dtype, cudaStream_t s) {
  if (n < 0 || H <= 0) return QL_STATUS_BAD_ARG;
  if (n == 0) return QL_STATUS_OK;
  if (dtype == QL_F16) scatter_rows_kernel<__half><<<n, 128, 0, s>>>(src, idx, scale, dst, (__half*)dst16, H);
  else if (dtype == QL_BF16)
    scatter_rows_kernel<__nv_bfloat16><<<n, 128, 0, s>>>(src, idx, scale, dst, (__nv_bfloat16*)dst16, H);
  else return QL_STATUS_BAD_ARG;
  return cudaPeekAtLastError() == cudaSuccess ? QL_STATUS_OK : QL_STATUS_CUDA;
}

}  // namespace ql
