// Shared pieces of the tcgen05 GEMM kernels (dense and NF4-fused): arguments, tile
// configuration, epilogue stores and the host-side tensor-map helpers.
#pragma once

#include <cstring>
#include <unordered_map>

#include "common.cuh"

namespace ql {

struct GemmArgs {
  int M, N, K;
  void* C;
  int64_t ldc;
  const void* bias;  // [N] of the input type, or null
  int out_dtype;     // QL_F16 / QL_BF16 / QL_F32
  int accumulate;    // C += result (fp32 output only)
  const float* residual;  // fp32 [M, ldc] or null: C = residual + (result rounded to the input type)
  int* err;
  // split-K: each output tile's K range is cut into `splits` parts computed by different work
  // units; every unit writes its fp32 partial to ws, the last one of a tile (counters) adds them
  // in split order and runs the epilogue. counters: one int per tile, zero between launches.
  int splits, kb_per_split;
  float* ws;
  int* counters;
  int tma_c;  // 16-bit C written by TMA tensor stores from per-warp shared-memory staging
  int b3d;    // MN-major B with one-chunk stages: the stage's 64-column boxes in one 3-D copy
};

// Epilogue staging for TMA stores of a 16-bit C: per epilogue warp two 32 x 32 buffers of 2 KB.
constexpr int EPI_BYTES = 4 * 2 * 2048;

// KC: 64-element K chunks per pipeline stage (1: one 2-D copy per 64-wide box; 2: one 3-D copy
// of two chunks per operand, see tma_load_3d).
template <int BN, bool kEpi = false, int KC = 1>
struct GemmCfg {
  static constexpr int BM = 128, BK = 64 * KC;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI = kEpi ? EPI_BYTES : 0;  // TMA-store staging (16-bit outputs)
  // as many ring slots as fit in 225 KB (at most 8)
  static constexpr int STAGES_FIT = (225 * 1024 - 1280 - EPI) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  // two accumulators of BN fp32 columns; the allocation is a power of two >= 32 columns
  static constexpr int TMEM_COLS = 2 * BN <= 256 ? 256 : 512;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "UMMA N (M = 128) and 32-column epilogue");
  static_assert(B_BYTES % 1024 == 0, "128-byte swizzle atoms of 8 rows");
};

template <typename OutT>
__device__ __forceinline__ void store_row32(OutT* dst, const float* v, int ncols) {
  if (ncols >= 32 && (reinterpret_cast<uintptr_t>(dst) % 16) == 0) {
    if constexpr (sizeof(OutT) == 2) {
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        OutT lo = from_f<OutT>(v[2 * i]), hi = from_f<OutT>(v[2 * i + 1]);
        w[i] = (uint32_t)(*reinterpret_cast<uint16_t*>(&lo)) |
               ((uint32_t)(*reinterpret_cast<uint16_t*>(&hi)) << 16);
      }
      uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int i = 0; i < 4; ++i) d[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    } else {
      float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
      for (int i = 0; i < 8; ++i) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < ncols) dst[i] = from_f<OutT>(v[i]);
  }
}

// One 32-row x 32-column chunk of a 16-bit C from this warp, through shared memory and a TMA
// tensor store: rows staged as 64-byte segments with the 64-byte swizzle (16-byte unit u of row
// r at u ^ ((r >> 1) & 3): conflict-free), two buffers per warp, lane 0 issuing the store. The
// tensor map clips rows and columns past C's edge.
template <typename OutT>
__device__ __forceinline__ void epi_tma_chunk(const CUtensorMap* map, uint8_t* stage, int& buf,
                                              const float* v, int x, int y) {
  const int lane = threadIdx.x & 31;
  uint8_t* stg = stage + buf * 2048;
  if (lane == 0) bulk_wait_read<1>();  // the store issued from this buffer two chunks ago
  __syncwarp();
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const uint4 w = make_uint4(pack_t2<OutT>(v[8 * u], v[8 * u + 1]), pack_t2<OutT>(v[8 * u + 2], v[8 * u + 3]),
                               pack_t2<OutT>(v[8 * u + 4], v[8 * u + 5]), pack_t2<OutT>(v[8 * u + 6], v[8 * u + 7]));
    *reinterpret_cast<uint4*>(stg + lane * 64 + ((u ^ ((lane >> 1) & 3)) << 4)) = w;
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(map, stg, x, y);
    bulk_commit();
  }
  buf ^= 1;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// Tensor maps already encoded, per host thread: a map is a pure function of its encode
// arguments, and the step asks for the same ones again and again (the static weights every step,
// the layer workspaces' buffers in every layer), while an encode costs a driver call. Keyed by
// every argument; cleared when it grows past a few thousand entries.
struct MapKey {
  uintptr_t ptr;
  int64_t rows, cols, ld;
  int box_rows, kind;  // kind: 0 / 1 K-major fp16 / bf16, 2 / 3 store maps, 4 + 2 chunks + bf16: 3-D
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && ld == o.ld &&
           box_rows == o.box_rows && kind == o.kind;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    uint64_t h = k.ptr * 0x9E3779B97F4A7C15ull;
    for (uint64_t v : {(uint64_t)k.rows, (uint64_t)k.cols, (uint64_t)k.ld,
                       (uint64_t)(k.box_rows * 8 + k.kind)})
      h = (h ^ v) * 0x100000001B3ull;
    return (size_t)h;
  }
};
static inline std::unordered_map<MapKey, CUtensorMap, MapKeyHash>& map_cache() {
  thread_local std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  if (cache.size() > 4096) cache.clear();
  return cache;
}

// A row-major [rows, cols] 16-bit matrix with row stride ld (elements), boxes of box_rows x 64.
static inline int encode_kmajor_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols,
                                    int64_t ld, int box_rows, bool bf16) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return QL_STATUS_CUDA;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QL_STATUS_OK : QL_STATUS_CUDA;
}

static inline int make_kmajor_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols,
                                  int64_t ld, int box_rows, bool bf16) {
  const MapKey key{reinterpret_cast<uintptr_t>(ptr), rows, cols, ld, box_rows, bf16 ? 1 : 0};
  auto& cache = map_cache();
  auto it = cache.find(key);
  if (it != cache.end()) {
    *map = it->second;
    return QL_STATUS_OK;
  }
  const int rc = encode_kmajor_map(map, ptr, rows, cols, ld, box_rows, bf16);
  if (rc == QL_STATUS_OK) cache.emplace(key, *map);
  return rc;
}

// The 3-D view of a row-major [rows, cols] 16-bit matrix (row stride ld elements, cols a multiple
// of 64): {64 columns, rows, cols / 64 chunks}, chunk stride 128 B, 128-byte swizzle, boxes of
// {64, box_rows, box_chunks}. K-major operands take box_chunks 2 (two K chunks of box_rows rows);
// an MN-major operand [K, N] takes box_rows K rows of box_chunks 64-column N chunks.
static inline int encode_chunked_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols,
                                     int64_t ld, int box_rows, int box_chunks, bool bf16) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr || cols % 64 != 0) return QL_STATUS_CUDA;
  cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(cols / 64)};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), 128};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, (cuuint32_t)box_chunks};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QL_STATUS_OK : QL_STATUS_CUDA;
}

static inline int make_chunked_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols,
                                   int64_t ld, int box_rows, int box_chunks, bool bf16) {
  const MapKey key{reinterpret_cast<uintptr_t>(ptr), rows, cols, ld, box_rows,
                   4 + 2 * box_chunks + (bf16 ? 1 : 0)};
  auto& cache = map_cache();
  auto it = cache.find(key);
  if (it != cache.end()) {
    *map = it->second;
    return QL_STATUS_OK;
  }
  const int rc = encode_chunked_map(map, ptr, rows, cols, ld, box_rows, box_chunks, bf16);
  if (rc == QL_STATUS_OK) cache.emplace(key, *map);
  return rc;
}

// A row-major [rows, cols] 16-bit C with row stride ld (elements), boxes of 32 x 32 staged with
// the 64-byte swizzle (rows of 64 bytes).
static inline int encode_store_map(CUtensorMap* map, void* ptr, int64_t rows, int64_t cols,
                                   int64_t ld, bool bf16) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return QL_STATUS_CUDA;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QL_STATUS_OK : QL_STATUS_CUDA;
}

static inline int make_store_map(CUtensorMap* map, void* ptr, int64_t rows, int64_t cols,
                                 int64_t ld, bool bf16) {
  const MapKey key{reinterpret_cast<uintptr_t>(ptr), rows, cols, ld, 32, bf16 ? 3 : 2};
  auto& cache = map_cache();
  auto it = cache.find(key);
  if (it != cache.end()) {
    *map = it->second;
    return QL_STATUS_OK;
  }
  const int rc = encode_store_map(map, ptr, rows, cols, ld, bf16);
  if (rc == QL_STATUS_OK) cache.emplace(key, *map);
  return rc;
}

static inline int num_sms() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

}  // namespace ql
