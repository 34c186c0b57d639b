// NF4 -> fp16 / bf16 dequantisation of bitsandbytes-layout weights (blocksize 64).
//
// Bit-exact restatement of the reference's nf4_dequant_kernel (solution/kernels.py:68-105),
// which itself matches bitsandbytes' dequantize_4bit: value = level[nibble] * scale in fp32,
// rounded once to the output type; the nested scale is code2[q] * absmax2 rounded, then + offset
// (two roundings, no fused multiply-add: solution/kernels.py:85-92).
//
// Two layouts: the weight as stored ([rows, cols], HBM-bound streaming, one thread per half
// block), and its transpose ([cols, rows], through a 64 x 64 shared-memory tile) for the
// data-gradient GEMMs, whose B operand is the weight's transpose in K-major order.
#include "common.cuh"
#include "profile.h"

namespace ql {

struct Nf4Args {
  const uint8_t* packed;
  const void* absmax;
  const float* code2;
  const float* absmax2;
  const float* offsets;
  const float* code;
  int64_t n_blocks;
  int bs2;
  int64_t seg1, seg2;
};

template <bool NESTED>
__device__ __forceinline__ float nf4_scale(const Nf4Args& a, int64_t blk) {
  if constexpr (NESTED) {
    const uint8_t q = reinterpret_cast<const uint8_t*>(a.absmax)[blk];
    const float s = __fmul_rn(__ldg(a.code2 + q), __ldg(a.absmax2 + blk / a.bs2));
    const int seg = (blk >= a.seg1) + (blk >= a.seg2);
    return __fadd_rn(s, __ldg(a.offsets + seg));
  } else {
    return __ldg(reinterpret_cast<const float*>(a.absmax) + blk);
  }
}

template <typename OutT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  OutT l = from_f<OutT>(lo), h = from_f<OutT>(hi);
  return (uint32_t)(*reinterpret_cast<uint16_t*>(&l)) | ((uint32_t)(*reinterpret_cast<uint16_t*>(&h)) << 16);
}

// One thread: 16 packed bytes = 32 values = half of a 64-value block.
template <typename OutT, bool NESTED>
__global__ void __launch_bounds__(256) nf4_dequant_kernel(Nf4Args a, OutT* __restrict__ out) {
  pdl_enter();
  __shared__ float lv[16];
  if (threadIdx.x < 16) lv[threadIdx.x] = a.code[threadIdx.x];
  __syncthreads();
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t blk = t >> 1;
  if (blk >= a.n_blocks) return;
  const float scale = nf4_scale<NESTED>(a, blk);
  const uint4 b = __ldg(reinterpret_cast<const uint4*>(a.packed) + t);
  const uint32_t words[4] = {b.x, b.y, b.z, b.w};
  uint32_t o[16];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t byte = (words[w] >> (8 * j)) & 0xFFu;
      // element 2j <- high nibble, 2j+1 <- low nibble
      o[w * 4 + j] = pack2<OutT>(__fmul_rn(lv[byte >> 4], scale), __fmul_rn(lv[byte & 15u], scale));
    }
  }
  uint4* dst = reinterpret_cast<uint4*>(out) + t * 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
}

// Transposed: W [rows, cols] -> out [cols, rows]. CTA tile: 64 rows x 64 cols (64 blocks),
// 128 threads; thread (r, h) decodes half a block of row r into smem column r, then each thread
// writes 32 consecutive values of one output row.
template <typename OutT, bool NESTED>
__global__ void __launch_bounds__(128) nf4_dequant_t_kernel(Nf4Args a, OutT* __restrict__ out,
                                                            int64_t rows, int64_t cols) {
  pdl_enter();
  __shared__ float lv[16];
  __shared__ uint16_t tile[64][64 + 2];
  if (threadIdx.x < 16) lv[threadIdx.x] = a.code[threadIdx.x];
  __syncthreads();
  const int64_t r0 = blockIdx.y * 64, c0 = blockIdx.x * 64;
  {
    const int r = threadIdx.x >> 1, h = threadIdx.x & 1;
    const int64_t elem = (r0 + r) * cols + c0 + h * 32;  // first of 32 values
    const int64_t blk = elem >> 6;
    const float scale = nf4_scale<NESTED>(a, blk);
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(a.packed + (elem >> 1)));
    const uint32_t words[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int w = 0; w < 4; ++w) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t byte = (words[w] >> (8 * j)) & 0xFFu;
        const int c = h * 32 + w * 8 + j * 2;
        OutT hi = from_f<OutT>(__fmul_rn(lv[byte >> 4], scale));
        OutT lo = from_f<OutT>(__fmul_rn(lv[byte & 15u], scale));
        tile[c][r] = *reinterpret_cast<uint16_t*>(&hi);
        tile[c + 1][r] = *reinterpret_cast<uint16_t*>(&lo);
      }
    }
  }
  __syncthreads();
  {
    const int c = threadIdx.x >> 1, h = threadIdx.x & 1;
    uint32_t o[16];
#pragma unroll
    for (int i = 0; i < 16; ++i)
      o[i] = (uint32_t)tile[c][h * 32 + 2 * i] | ((uint32_t)tile[c][h * 32 + 2 * i + 1] << 16);
    uint4* dst = reinterpret_cast<uint4*>(out + (c0 + c) * rows + r0 + h * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
  }
}

template <typename OutT>
static int launch_nf4(const Nf4Args& a, void* out, int64_t rows, int64_t cols, bool nested,
                      bool transpose, cudaStream_t s) {
  OutT* o = reinterpret_cast<OutT*>(out);
  if (transpose) {
    dim3 grid((unsigned)(cols / 64), (unsigned)(rows / 64));
    if (nested) launch_k(nf4_dequant_t_kernel<OutT, true>, grid, dim3(128), 0, s, a, o, rows, cols);
    else launch_k(nf4_dequant_t_kernel<OutT, false>, grid, dim3(128), 0, s, a, o, rows, cols);
  } else {
    const int64_t threads = a.n_blocks * 2;
    const unsigned grid = (unsigned)cdiv(threads, 256);
    if (nested) launch_k(nf4_dequant_kernel<OutT, true>, dim3(grid), dim3(256), 0, s, a, o);
    else launch_k(nf4_dequant_kernel<OutT, false>, dim3(grid), dim3(256), 0, s, a, o);
  }
  return launched(1);
}

int nf4_dequant(const uint8_t* packed, const void* absmax, const float* code2,
                const float* absmax2, const float* offsets, const float* code, void* out,
                int64_t rows, int64_t cols, int nested, int bs2, int64_t seg1, int64_t seg2,
                int out_dtype, int transpose, cudaStream_t stream) {
  if (rows < 0 || cols < 0) return QL_STATUS_BAD_ARG;
  const int64_t numel = rows * cols;
  if (numel == 0) return QL_STATUS_OK;
  if (numel % 64 != 0) return QL_STATUS_BAD_ARG;
  if (transpose && (rows % 64 != 0 || cols % 64 != 0)) return QL_STATUS_BAD_ARG;
  if (nested && (bs2 <= 0 || code2 == nullptr || absmax2 == nullptr || offsets == nullptr))
    return QL_STATUS_BAD_ARG;
  if (reinterpret_cast<uintptr_t>(packed) % 16 != 0 || reinterpret_cast<uintptr_t>(out) % 16 != 0)
    return QL_STATUS_BAD_ARG;
  Nf4Args a{packed, absmax, code2, absmax2, offsets, code, numel / 64, bs2 > 0 ? bs2 : 1,
            seg1, seg2};
  ProfScope prof(PK_DEQUANT, 0, numel * (0.5 + (nested ? 1.0 : 4.0) / 64 + 2.0), stream);
  if (out_dtype == QL_F16) return launch_nf4<__half>(a, out, rows, cols, nested, transpose, stream);
  if (out_dtype == QL_BF16)
    return launch_nf4<__nv_bfloat16>(a, out, rows, cols, nested, transpose, stream);
  return QL_STATUS_BAD_ARG;
}

// ---------------------------------------------------------------------------------------------
// Many weights in one launch (every group of every layer at the start of a step): one thread per
// half block as above; the item of a thread is found by binary search over the items' first
// threads (kernel parameters, up to NF4_BATCH items per launch).
// ---------------------------------------------------------------------------------------------
constexpr int NF4_BATCH = 28;

struct Nf4Item {
  const uint8_t* packed;
  const void* absmax;
  const float* code2;
  const float* absmax2;
  const float* offsets;
  const float* code;
  void* out;
  int64_t first;     // first thread (half block) of this item in the launch
  int64_t seg1, seg2;
  int32_t bs2, nested;
};
struct Nf4Batch {
  Nf4Item item[NF4_BATCH];
  int count;
  int64_t total;     // threads of the launch
};

template <typename OutT>
__global__ void __launch_bounds__(256) nf4_dequant_batch_kernel(const __grid_constant__ Nf4Batch b) {
  pdl_enter();
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= b.total) return;
  int lo = 0, hi = b.count - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (t >= b.item[mid].first) lo = mid; else hi = mid - 1;
  }
  const Nf4Item& it = b.item[lo];
  const int64_t lt = t - it.first, blk = lt >> 1;
  float scale;
  if (it.nested) {
    const uint8_t q = reinterpret_cast<const uint8_t*>(it.absmax)[blk];
    const float s = __fmul_rn(__ldg(it.code2 + q), __ldg(it.absmax2 + blk / it.bs2));
    const int seg = (blk >= it.seg1) + (blk >= it.seg2);
    scale = __fadd_rn(s, __ldg(it.offsets + seg));
  } else {
    scale = __ldg(reinterpret_cast<const float*>(it.absmax) + blk);
  }
  const uint4 w = __ldg(reinterpret_cast<const uint4*>(it.packed) + lt);
  const uint32_t words[4] = {w.x, w.y, w.z, w.w};
  uint32_t o[16];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t byte = (words[k] >> (8 * j)) & 0xFFu;
      o[k * 4 + j] = pack2<OutT>(__fmul_rn(__ldg(it.code + (byte >> 4)), scale),
                                 __fmul_rn(__ldg(it.code + (byte & 15u)), scale));
    }
  }
  uint4* dst = reinterpret_cast<uint4*>(it.out) + lt * 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
}

int nf4_dequant_batch(const ql_nf4_weight* w, void* const* outs, int count, int out_dtype,
                      cudaStream_t s) {
  if (count < 0 || (count > 0 && (w == nullptr || outs == nullptr))) return QL_STATUS_BAD_ARG;
  if (out_dtype != QL_F16 && out_dtype != QL_BF16) return QL_STATUS_BAD_ARG;
  double bytes = 0;
  for (int i = 0; i < count; ++i) {
    const ql_nf4_weight& g = w[i];
    const int64_t numel = g.rows * g.cols;
    if (g.rows < 0 || g.cols < 0 || numel % 64 != 0 || g.packed == nullptr || g.absmax == nullptr ||
        g.code == nullptr || outs[i] == nullptr ||
        reinterpret_cast<uintptr_t>(g.packed) % 16 != 0 || reinterpret_cast<uintptr_t>(outs[i]) % 16 != 0)
      return QL_STATUS_BAD_ARG;
    if (g.nested && (g.bs2 <= 0 || g.code2 == nullptr || g.absmax2 == nullptr || g.offsets == nullptr))
      return QL_STATUS_BAD_ARG;
    bytes += numel * (0.5 + (g.nested ? 1.0 : 4.0) / 64 + 2.0);
  }
  ProfScope prof(PK_DEQUANT, 0, bytes, s);
  int launches = 0;
  for (int i0 = 0; i0 < count; i0 += NF4_BATCH) {
    Nf4Batch b{};
    b.count = count - i0 < NF4_BATCH ? count - i0 : NF4_BATCH;
    int64_t first = 0;
    for (int k = 0; k < b.count; ++k) {
      const ql_nf4_weight& g = w[i0 + k];
      b.item[k] = Nf4Item{g.packed, g.absmax, g.code2, g.absmax2, g.offsets, g.code, outs[i0 + k],
                          first, g.seg1, g.seg2, g.bs2 > 0 ? g.bs2 : 1, g.nested};
      first += g.rows * g.cols / 32;  // half blocks
    }
    b.total = first;
    if (first == 0) continue;
    const dim3 grid((unsigned)cdiv(first, 256));
    cudaError_t e = out_dtype == QL_F16
                        ? launch_k(nf4_dequant_batch_kernel<__half>, grid, dim3(256), 0, s, b)
                        : launch_k(nf4_dequant_batch_kernel<__nv_bfloat16>, grid, dim3(256), 0, s, b);
    if (e != cudaSuccess) return QL_STATUS_CUDA;
    ++launches;
  }
  return launches ? launched(launches) : QL_STATUS_OK;
}

}  // namespace ql
