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
  pdl_enter();
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
  pdl_enter();
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
    launch_k(glu_fwd_kernel<__half>, dim3(grid), dim3(256), 0, s, (const __half*)gu, (__half*)m, n, I);
  else if (dtype == QL_BF16)
    launch_k(glu_fwd_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, s, (const __nv_bfloat16*)gu, (__nv_bfloat16*)m, n, I);
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
    launch_k(glu_bwd_kernel<__half>, dim3(grid), dim3(256), 0, s, (const __half*)dm, (__half*)gu, n, I);
  else if (dtype == QL_BF16)
    launch_k(glu_bwd_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, s, (const __nv_bfloat16*)dm, (__nv_bfloat16*)gu, n, I);
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
  pdl_enter();
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
  pdl_enter();
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
// the LoRA weight gradients of a layer, all four products in one launch
// ---------------------------------------------------------------------------------------------
constexpr int LG_COLS = 64, LG_THREADS = 256, LG_MAXJOBS = 4, LG_MAXSPLITS = 16;
constexpr int LG_MAXTOK = 256;  // tokens staged in shared memory at once
constexpr int64_t LG_COUNTER_BYTES = 2048;

struct LgJob {
  const void* X;
  int64_t ldx;
  const void* Y;
  float* out;
  float* part;  // [S][nblk * 64][16]
  int ncols, y_f32, transpose, blk0;
  float scale;
};
struct LgArgs {
  LgJob job[LG_MAXJOBS];
  int njobs, splits;
  int64_t n, tok_per_split;
  int* counters;  // one per 64-column block of all jobs
};

// CTA (column block b, split sp): out^T-partial[64 cols][16] = X[toks][64]^T . Y[toks][16] on
// the tensor cores (mma.sync m16n8k16, fp32 accumulation). Rounds of up to 256 tokens of X
// (16-byte chunks XOR-swizzled by token: conflict-free ldmatrix) and Y (fp32 rounded to the
// 16-bit type on the way in: the reference's fp16 dx_lo) are staged in shared memory; warp w
// takes column tile w % 4 (16 columns) and the 16-token steps of parity w / 4, both operands
// read with ldmatrix.trans. The two parities meet in shared memory (fixed order), the split's
// partial goes to the workspace, and the last split of the block (counter) adds all splits in
// split order.
template <typename TX>
__global__ void __launch_bounds__(LG_THREADS) lora_grads_kernel(LgArgs a) {
  pdl_enter();
  extern __shared__ __align__(16) uint8_t lg_smem[];
  __shared__ float sp2[2][LG_COLS * 16];
  __shared__ int last;
  int j = 0;
#pragma unroll
  for (int q = 1; q < LG_MAXJOBS; ++q)
    if (q < a.njobs && (int)blockIdx.x >= a.job[q].blk0) j = q;
  const LgJob& J = a.job[j];
  const int blk = blockIdx.x - J.blk0, c0 = blk * LG_COLS;
  const int64_t t0 = blockIdx.y * a.tok_per_split;
  const int64_t t1 = min(a.n, t0 + a.tok_per_split);
  const int stage_tok = (int)min(a.tok_per_split, (int64_t)LG_MAXTOK);  // a multiple of 16
  TX* sX = reinterpret_cast<TX*>(lg_smem);   // [stage_tok][64], chunk c of token t at c ^ (t & 7)
  TX* sY = sX + stage_tok * LG_COLS;          // [stage_tok][16]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = warp & 3, par = warp >> 2;
  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  for (int64_t tb = t0; tb < t1; tb += stage_tok) {  // rounds of up to 256 tokens
    const int nt = (int)min((int64_t)stage_tok, t1 - tb);
    const int nt16 = (nt + 15) & ~15;  // rows past nt are zero
    const TX* X = reinterpret_cast<const TX*>(J.X) + c0;
    for (int i = threadIdx.x; i < nt16 * 8; i += LG_THREADS) {  // 8 chunks of 16 B per row
      const int tt = i >> 3, ch = i & 7;
      const bool ok = tt < nt && c0 + ch * 8 < J.ncols;
      cs_cp16(sX + tt * LG_COLS + ((ch ^ (tt & 7)) << 3), ok ? X + (tb + tt) * J.ldx + ch * 8 : J.X, ok);
    }
    if (J.y_f32) {
      const float* Y = reinterpret_cast<const float*>(J.Y) + tb * 16;
      for (int i = threadIdx.x; i < nt16 * 4; i += LG_THREADS) {  // 4 values per thread
        const int tt = i >> 2;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (tt < nt) v = __ldg(reinterpret_cast<const float4*>(Y) + i);
        TX h[4] = {from_f<TX>(v.x), from_f<TX>(v.y), from_f<TX>(v.z), from_f<TX>(v.w)};
        *reinterpret_cast<uint2*>(sY + i * 4) = *reinterpret_cast<const uint2*>(h);
      }
    } else {
      const TX* Y = reinterpret_cast<const TX*>(J.Y) + tb * 16;
      for (int i = threadIdx.x; i < nt16 * 2; i += LG_THREADS)
        cs_cp16(sY + i * 8, (i >> 1) < nt ? Y + i * 8 : J.Y, (i >> 1) < nt);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    const int mi = lane >> 3, ri = lane & 7;  // ldmatrix: matrix, row of this lane's address
    for (int k0 = par * 16; k0 < nt16; k0 += 32) {
      // A = X^T (16 columns x 16 tokens): matrices (cols +0/+8) x (tokens +0/+8)
      const int ta = k0 + ((mi >> 1) << 3) + ri;
      const int cha = mt * 2 + (mi & 1);
      uint32_t af[4];
      ldsm_x4_t(sX + ta * LG_COLS + ((cha ^ (ta & 7)) << 3), af[0], af[1], af[2], af[3]);
      // B = Y (16 tokens x 16 ranks): matrices (tokens +0/+8) x (ranks +0/+8)
      const int tb2 = k0 + ((mi & 1) << 3) + ri;
      uint32_t b00, b01, b10, b11;
      ldsm_x4_t(sY + tb2 * 16 + ((mi >> 1) << 3), b00, b01, b10, b11);
      mma16816<TX>(acc[0], af, b00, b01);
      mma16816<TX>(acc[1], af, b10, b11);
    }
    __syncthreads();  // the staging buffers are refilled by the next round
  }
  // C fragments: column mt*16 + g (+8), ranks nt*8 + 2t (+1)
  {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int n8 = 0; n8 < 2; ++n8) {
      float* d0 = &sp2[par][(mt * 16 + g) * 16 + n8 * 8 + 2 * t];
      float* d1 = &sp2[par][(mt * 16 + g + 8) * 16 + n8 * 8 + 2 * t];
      d0[0] = acc[n8][0];
      d0[1] = acc[n8][1];
      d1[0] = acc[n8][2];
      d1[1] = acc[n8][3];
    }
  }
  __syncthreads();
  const int64_t padc = (int64_t)((J.ncols + LG_COLS - 1) / LG_COLS) * LG_COLS;  // columns per split
  float* part = J.part + ((int64_t)blockIdx.y * padc + c0) * 16;
#pragma unroll
  for (int e = threadIdx.x; e < LG_COLS * 16; e += LG_THREADS) __stcg(part + e, sp2[0][e] + sp2[1][e]);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int old = atomicAdd(a.counters + blockIdx.x, 1);
    last = old == a.splits - 1;
    if (last) a.counters[blockIdx.x] = 0;  // ready for the next launch
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  const int64_t stride = padc * 16;
  const float* base = J.part + (int64_t)c0 * 16;
#pragma unroll
  for (int e = threadIdx.x; e < LG_COLS * 16; e += LG_THREADS) {
    const int c = c0 + e / 16, r = e % 16;
    float v[LG_MAXSPLITS];
#pragma unroll
    for (int q = 0; q < LG_MAXSPLITS; ++q) v[q] = q < a.splits ? __ldcg(base + q * stride + e) : 0.f;
    float sum = 0.f;
#pragma unroll
    for (int q = 0; q < LG_MAXSPLITS; ++q)
      if (q < a.splits) sum += v[q];  // split order
    if (c < J.ncols) {
      if (J.transpose) J.out[(int64_t)r * J.ncols + c] = sum * J.scale;
      else J.out[(int64_t)c * 16 + r] = sum * J.scale;
    }
  }
}

static int lora_grads_splits(int64_t n, int64_t blocks) {
  const int sms = sm_count();
  int64_t s = cdiv(4LL * sms, blocks > 0 ? blocks : 1);  // about 4 CTAs per SM
  const int64_t by_tokens = cdiv(n, 32);                  // at least 32 tokens per split
  if (s > by_tokens) s = by_tokens;
  if (s > LG_MAXSPLITS) s = LG_MAXSPLITS;
  return (int)(s < 1 ? 1 : s);
}

int64_t lora_grads_workspace(int64_t n, const int32_t* ncols, int njobs) {
  if (njobs < 0 || njobs > LG_MAXJOBS || (njobs > 0 && ncols == nullptr)) return -1;
  int64_t blocks = 0, cols = 0;
  for (int q = 0; q < njobs; ++q) {
    blocks += cdiv(ncols[q], LG_COLS);
    cols += cdiv(ncols[q], LG_COLS) * LG_COLS;
  }
  const int s = lora_grads_splits(n, blocks);
  return LG_COUNTER_BYTES + ((s * cols * 16 * 4 + 255) / 256) * 256 + 256 * LG_MAXJOBS;
}

int lora_grads(const ql_lora_grad_job* jobs, int njobs, int64_t n, int x_dtype, void* workspace,
               int64_t workspace_bytes, cudaStream_t s) {
  if (njobs <= 0 || njobs > LG_MAXJOBS || jobs == nullptr || n < 0) return QL_STATUS_BAD_ARG;
  if (x_dtype != QL_F16 && x_dtype != QL_BF16) return QL_STATUS_BAD_ARG;
  if (workspace == nullptr || reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return QL_STATUS_BAD_ARG;
  LgArgs a{};
  a.njobs = njobs;
  a.n = n;
  int32_t nc[LG_MAXJOBS];
  int64_t blocks = 0;
  for (int q = 0; q < njobs; ++q) {
    const ql_lora_grad_job& J = jobs[q];
    if (J.ncols <= 0 || J.ncols % 8 != 0 || J.ldx % 8 != 0 || J.X == nullptr || J.Y == nullptr ||
        J.out == nullptr || reinterpret_cast<uintptr_t>(J.X) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(J.Y) % 16 != 0)
      return QL_STATUS_BAD_ARG;
    if (J.y_dtype != QL_F32 && J.y_dtype != x_dtype) return QL_STATUS_BAD_ARG;
    nc[q] = J.ncols;
    a.job[q] = LgJob{J.X, J.ldx, J.Y, J.out, nullptr, J.ncols, J.y_dtype == QL_F32 ? 1 : 0,
                     J.transpose, (int)blocks, J.scale};
    blocks += cdiv(J.ncols, LG_COLS);
  }
  if (blocks * 4 > LG_COUNTER_BYTES) return QL_STATUS_UNSUPPORTED;
  if (workspace_bytes < lora_grads_workspace(n, nc, njobs)) return QL_STATUS_BAD_ARG;
  a.splits = lora_grads_splits(n, blocks);
  a.tok_per_split = cdiv(cdiv(n > 0 ? n : 1, a.splits), 16) * 16;  // whole 16-token steps
  a.splits = (int)cdiv(n > 0 ? n : 1, a.tok_per_split);
  a.counters = static_cast<int*>(workspace);
  float* p = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + LG_COUNTER_BYTES);
  for (int q = 0; q < njobs; ++q) {
    a.job[q].part = p;
    p += (int64_t)a.splits * cdiv(nc[q], LG_COLS) * LG_COLS * 16;
  }
  double flops = 0, bytes = 0;
  for (int q = 0; q < njobs; ++q) {
    flops += 2.0 * n * nc[q] * 16;
    bytes += (double)n * nc[q] * 2;
  }
  ProfScope prof(PK_COLSUM, flops, bytes, s);
  dim3 grid((unsigned)blocks, (unsigned)a.splits);
  const int smem = (int)(min(a.tok_per_split, (int64_t)LG_MAXTOK) * (LG_COLS + 16) * 2);
  if (x_dtype == QL_F16) {
    smem_optin(reinterpret_cast<const void*>(lora_grads_kernel<__half>), smem);
    launch_k(lora_grads_kernel<__half>, grid, dim3(LG_THREADS), smem, s, a);
  } else {
    smem_optin(reinterpret_cast<const void*>(lora_grads_kernel<__nv_bfloat16>), smem);
    launch_k(lora_grads_kernel<__nv_bfloat16>, grid, dim3(LG_THREADS), smem, s, a);
  }
  return launched(1);
}

// ---------------------------------------------------------------------------------------------
// embedding gather: h[t, :] = float(W[ids[t], :])
// ---------------------------------------------------------------------------------------------
template <typename T>
__global__ void embed_kernel(const int64_t* __restrict__ ids, const T* __restrict__ W,
                             float* __restrict__ h, int64_t n, int H, int64_t vocab, int* err) {
  pdl_enter();
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
  pdl_enter();
  const int64_t r = blockIdx.x;
  const float4* s = reinterpret_cast<const float4*>(src + idx[r] * H);
  float4* d = reinterpret_cast<float4*>(dst + r * H);
  for (int c = threadIdx.x; c < H / 4; c += blockDim.x) d[c] = s[c];
}

template <typename T>
__global__ void scatter_rows_kernel(const float* __restrict__ src, const int64_t* __restrict__ idx,
                                    const float* __restrict__ scale, float* __restrict__ dst,
                                    T* __restrict__ dst16, int H) {
  pdl_enter();
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

// embedding gather from a table in page-locked host memory, read by the kernel over the host
// link (zero-copy): one CTA per token, 16-byte loads when the row allows. The loads are plain
// ld.global (the read-only data path is not used on host memory).
__device__ __forceinline__ uint4 ld_plain_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ unsigned short ld_plain_u16(const void* p) {
  unsigned short v;
  asm volatile("ld.global.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

template <typename T>
__global__ void embed_host_kernel(const int64_t* __restrict__ ids, const T* W, float* __restrict__ h,
                                  int64_t n, int H, int64_t vocab, int vec, int* err) {
  pdl_enter();
  const int64_t t = blockIdx.x;
  const int64_t id = ids[t];
  float* out = h + t * H;
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) raise_status(err, QL_STATUS_BAD_ARG);
    for (int c = threadIdx.x; c < H; c += blockDim.x) out[c] = 0.f;
    return;
  }
  const T* row = W + id * H;
  if (vec) {
    for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
      const uint4 v = ld_plain_v4(row + c * 8);
      const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
      for (int j = 0; j < 8; ++j) out[c * 8 + j] = to_f<T>(e[j]);
    }
  } else {
    for (int c = threadIdx.x; c < H; c += blockDim.x) {
      const unsigned short b = ld_plain_u16(row + c);
      out[c] = to_f<T>(*reinterpret_cast<const T*>(&b));
    }
  }
}

int embed_host(const int64_t* ids, const void* W_dev, float* h, int64_t n, int H, int64_t vocab,
               int dtype, int* err, cudaStream_t s) {
  if (n < 0 || H <= 0) return QL_STATUS_BAD_ARG;
  if (n == 0) return QL_STATUS_OK;
  const int vec = ((uintptr_t)W_dev % 16 == 0 && (H * 2) % 16 == 0) ? 1 : 0;
  if (dtype == QL_F16)
    embed_host_kernel<__half><<<n, 128, 0, s>>>(ids, (const __half*)W_dev, h, n, H, vocab, vec, err);
  else if (dtype == QL_BF16)
    embed_host_kernel<__nv_bfloat16><<<n, 128, 0, s>>>(ids, (const __nv_bfloat16*)W_dev, h, n, H,
                                                       vocab, vec, err);
  else return QL_STATUS_BAD_ARG;
  return launched(1);
}

}  // namespace ql
