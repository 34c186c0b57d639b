// extern "C" entry points of libqlora_sm100a.so (declared in include/qlora_sm100.h): argument
// checks, the per-thread error message, the device status word, and dispatch to the kernels.
#include <atomic>
#include <cstdio>
#include <mutex>
#include <unordered_map>
#include <cstring>
#include <string>

#include "common.cuh"
#include "ops.h"
#include "philox.cuh"

namespace {
__device__ int g_status_word = 0;  // QL_STATUS_TIMEOUT etc., recorded by kernels
thread_local std::string g_last_error;
std::atomic<long long> g_launches{0};  // kernels launched by this library (all host threads)

int fail(int code, const char* where) {
  const cudaError_t e = cudaGetLastError();
  char buf[512];
  std::snprintf(buf, sizeof(buf), "%s: %s%s%s", where,
                code == QL_STATUS_BAD_ARG     ? "invalid argument"
                : code == QL_STATUS_UNSUPPORTED ? "unsupported request"
                : code == QL_STATUS_TIMEOUT   ? "timeout"
                                              : "CUDA error",
                e != cudaSuccess ? " / " : "", e != cudaSuccess ? cudaGetErrorString(e) : "");
  g_last_error = buf;
  return code;
}

int done(int code, const char* where) {
  if (code == QL_STATUS_OK) return QL_STATUS_OK;
  return fail(code, where);
}
}  // namespace

namespace ql {
int launched(int kernels) {
  if (cudaPeekAtLastError() != cudaSuccess) return QL_STATUS_CUDA;
  g_launches.fetch_add(kernels, std::memory_order_relaxed);
  return QL_STATUS_OK;
}

void smem_optin(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::unordered_map<const void*, int> done;  // per kernel: the limit already set
  std::lock_guard<std::mutex> lk(mu);
  int& have = done[kernel];
  if (have >= bytes) return;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) ==
      cudaSuccess)
    have = bytes;
}

int sm_count() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

static std::atomic<bool> g_pdl{true};
bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed); }
void set_pdl(bool on) { g_pdl.store(on, std::memory_order_relaxed); }

int* status_word() {
  // one address per device, looked up once (host threads may race to fill an entry: both store
  // the same address)
  static std::atomic<int*> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  int* p = cache[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_status_word) != cudaSuccess) return nullptr;
    p = static_cast<int*>(addr);
    cache[dev].store(p, std::memory_order_release);
  }
  return p;
}

// The bounded-wait probe (ql_wait_probe): one CTA, two roles. Warp 0 waits on an mbarrier that
// nothing arrives on, under limit_ns, so its wait runs out and records QL_STATUS_TIMEOUT; warp 1
// waits on another such barrier under the full limit and gives up as soon as it sees the status
// recorded (what every other role of a kernel does when one role times out). Each role adds 1 to
// *returned when it has left its wait.
__global__ void wait_probe_kernel(int* err, unsigned long long limit_ns, int* returned) {
  __shared__ __align__(8) uint64_t bars[2];
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0 && warp < 2) {
    mbar_wait(&bars[warp], 0, err, warp == 0 ? limit_ns : QL_WAIT_NS);
    atomicAdd(returned, 1);
  }
}
}  // namespace ql

extern "C" {

const char* ql_version(void) { return "qlora_sm100a 0.1 (sm_100a, tcgen05)"; }

const char* ql_last_error(void) { return g_last_error.c_str(); }

long long ql_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int* ql_device_status_ptr(void) { return ql::status_word(); }

int ql_device_status(int* status_out, int clear) {
  int* p = ql::status_word();
  if (p == nullptr || status_out == nullptr) return fail(QL_STATUS_CUDA, "ql_device_status");
  if (cudaMemcpy(status_out, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return fail(QL_STATUS_CUDA, "ql_device_status");
  if (clear && cudaMemset(p, 0, sizeof(int)) != cudaSuccess)
    return fail(QL_STATUS_CUDA, "ql_device_status");
  return QL_STATUS_OK;
}

int ql_nf4_dequant(const uint8_t* packed, const void* absmax, const float* code2,
                   const float* absmax2, const float* offsets, const float* code, void* out,
                   int64_t rows, int64_t cols, int nested, int bs2, int64_t seg1, int64_t seg2,
                   int out_dtype, int transpose, cudaStream_t stream) {
  return done(ql::nf4_dequant(packed, absmax, code2, absmax2, offsets, code, out, rows, cols,
                              nested, bs2, seg1, seg2, out_dtype, transpose, stream),
              "ql_nf4_dequant");
}

int ql_gemm_tn(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
               const void* bias, int M, int N, int K, int in_dtype, int out_dtype, int accumulate,
               const float* residual, void* workspace, int64_t workspace_bytes,
               cudaStream_t stream) {
  return done(ql::gemm_tn(A, lda, B, ldb, C, ldc, bias, M, N, K, in_dtype, out_dtype, accumulate,
                          residual, ql::status_word(), stream, workspace, workspace_bytes),
              "ql_gemm_tn");
}

int ql_gemm_nn(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
               const void* bias, int M, int N, int K, int in_dtype, int out_dtype, int accumulate,
               const float* residual, void* workspace, int64_t workspace_bytes,
               cudaStream_t stream) {
  return done(ql::gemm_nn(A, lda, B, ldb, C, ldc, bias, M, N, K, in_dtype, out_dtype, accumulate,
                          residual, ql::status_word(), stream, workspace, workspace_bytes),
              "ql_gemm_nn");
}

int ql_nf4_dequant_batch(const ql_nf4_weight* weights, void* const* outs, int count, int out_dtype,
                         cudaStream_t stream) {
  return done(ql::nf4_dequant_batch(weights, outs, count, out_dtype, stream), "ql_nf4_dequant_batch");
}

int64_t ql_gemm_workspace_bytes(int M, int N, int K) { return ql::gemm_workspace_bytes(M, N, K); }

int ql_gemm_nf4(const void* A, int64_t lda, const ql_nf4_weight* W, int layout, void* C,
                int64_t ldc, const void* bias, int M, int in_dtype, int out_dtype, int accumulate,
                const float* residual, cudaStream_t stream) {
  if (W == nullptr) return done(QL_STATUS_BAD_ARG, "ql_gemm_nf4");
  return done(ql::gemm_nf4(A, lda, *W, layout, C, ldc, bias, M, in_dtype, out_dtype, accumulate,
                           residual, ql::status_word(), stream),
              "ql_gemm_nf4");
}

int ql_wait_probe(int64_t limit_ns, int* returned, cudaStream_t stream) {
  if (returned == nullptr || limit_ns < 1000000 || limit_ns > (int64_t)ql::QL_WAIT_NS)
    return done(QL_STATUS_BAD_ARG, "ql_wait_probe");
  int* err = ql::status_word();
  if (err == nullptr) return fail(QL_STATUS_CUDA, "ql_wait_probe");
  ql::wait_probe_kernel<<<1, 64, 0, stream>>>(err, (unsigned long long)limit_ns, returned);
  return done(ql::launched(1), "ql_wait_probe");
}

uint32_t ql_dropout_keep_threshold(float p_keep) {
  ql::DropoutArgs d{};
  d.threads = 1;
  d.p_keep = p_keep;
  ql::prepare_dropout(d);
  return d.keep_below;
}

int ql_set_pdl(int on) {
  if (on != 0 && on != 1) return done(QL_STATUS_BAD_ARG, "ql_set_pdl");
  ql::set_pdl(on != 0);
  return QL_STATUS_OK;
}

int ql_gemm_set_mode(int mode) {
  if (mode < 0 || mode > 6 || (mode & 3) == 3) return done(QL_STATUS_BAD_ARG, "ql_gemm_set_mode");
  ql::gemm_set_mode(mode);
  return QL_STATUS_OK;
}

}  // extern "C"

extern "C" {

int ql_rms_fwd(const ql_rms_fwd_args* args, cudaStream_t stream) {
  if (args == nullptr) return fail(QL_STATUS_BAD_ARG, "ql_rms_fwd");
  return done(ql::rms_fwd(*args, stream), "ql_rms_fwd");
}

int ql_rms_bwd(const ql_rms_bwd_args* args, cudaStream_t stream) {
  if (args == nullptr) return fail(QL_STATUS_BAD_ARG, "ql_rms_bwd");
  return done(ql::rms_bwd(*args, stream), "ql_rms_bwd");
}

int ql_dropout_keep(int8_t* out, int64_t nelem, int64_t seed, int64_t ctr, int64_t threads,
                    float p_keep, int vec, cudaStream_t stream) {
  return done(ql::dropout_keep(out, nelem, seed, ctr, threads, p_keep, vec, stream),
              "ql_dropout_keep");
}

}  // extern "C"

extern "C" {

int ql_rope_fwd(const ql_rope_fwd_args* args, cudaStream_t stream) {
  if (args == nullptr) return fail(QL_STATUS_BAD_ARG, "ql_rope_fwd");
  return done(ql::rope_fwd(*args, stream), "ql_rope_fwd");
}

int ql_rope_bwd(const ql_rope_bwd_args* args, cudaStream_t stream) {
  if (args == nullptr) return fail(QL_STATUS_BAD_ARG, "ql_rope_bwd");
  return done(ql::rope_bwd(*args, stream), "ql_rope_bwd");
}

int ql_glu_fwd(const void* gu, void* m, int64_t n, int I, int dtype, cudaStream_t stream) {
  return done(ql::glu_fwd(gu, m, n, I, dtype, stream), "ql_glu_fwd");
}

int ql_glu_bwd(const void* dm, void* gu, int64_t n, int I, int dtype, cudaStream_t stream) {
  return done(ql::glu_bwd(dm, gu, n, I, dtype, stream), "ql_glu_bwd");
}

int64_t ql_lora_colsum_workspace(int64_t n, int ncols, int rank) {
  return (int64_t)ql::lora_colsum_splits(n, ncols) * ncols * rank;
}

int ql_lora_colsum(const void* X, int64_t ldx, int x_dtype, const void* Y, int y_dtype, int64_t n,
                   int ncols, int rank, float scale, int transpose, float* out, float* workspace,
                   int64_t workspace_floats, cudaStream_t stream) {
  return done(ql::lora_colsum(X, ldx, x_dtype, Y, y_dtype, n, ncols, rank, scale, transpose, out,
                              workspace, workspace_floats, stream),
              "ql_lora_colsum");
}

// LoRA column sums whose per-split partials live in a scratch array compiled into the library,
// for callers that cannot hand in a workspace: a plain C or ctypes host with no device allocator
// of its own (a cudaMalloc there would synchronise the whole device in the middle of a step), or
// a runtime whose device memory is planned once at start-up and must not grow while a step runs.
// The scratch is one per device: calls that overlap on a device race on it. Nothing in it has to
// start at zero (every call writes each partial it later reads).
namespace {
__device__ __align__(256) float g_colsum_scratch[QL_COLSUM_STATIC_FLOATS];
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
float* g_scratch_ptr[kMaxDevices] = {};

// The scratch's address on the current device, looked up once per device (the lookup can load
// the module on that device, so it is done by the first call, never per launch).
int colsum_scratch(float** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(QL_STATUS_CUDA, "ql_lora_colsum_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) {
    g_last_error = "ql_lora_colsum_noalloc: device ordinal " + std::to_string(dev) +
                   " is beyond the " + std::to_string(kMaxDevices) + " devices it keeps scratch for";
    return QL_STATUS_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_colsum_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(QL_STATUS_CUDA, "ql_lora_colsum_noalloc: cudaGetSymbolAddress of the scratch");
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return QL_STATUS_OK;
}
}  // namespace

int ql_lora_colsum_noalloc(const void* X, int64_t ldx, int x_dtype, const void* Y, int y_dtype,
                           int64_t n, int ncols, int rank, float scale, int transpose, float* out,
                           cudaStream_t stream) {
  if (rank != 16) {
    g_last_error = "ql_lora_colsum_noalloc: rank " + std::to_string(rank) +
                   " is not supported (rank 16 only)";
    return QL_STATUS_UNSUPPORTED;
  }
  if (n < 0 || ncols <= 0) return done(QL_STATUS_BAD_ARG, "ql_lora_colsum_noalloc");
  const int64_t need = (int64_t)ql::lora_colsum_splits(n, ncols) * (int64_t)ncols * 16;
  if (need > QL_COLSUM_STATIC_FLOATS) {
    g_last_error = "ql_lora_colsum_noalloc: this shape needs " + std::to_string(need) +
                   " floats of scratch, the static scratch holds " +
                   std::to_string((long long)QL_COLSUM_STATIC_FLOATS) +
                   " (4 MiB); use ql_lora_colsum with a workspace";
    return QL_STATUS_BAD_ARG;
  }
  float* scratch = nullptr;
  const int rc = colsum_scratch(&scratch);
  if (rc != QL_STATUS_OK) return rc;
  return done(ql::lora_colsum(X, ldx, x_dtype, Y, y_dtype, n, ncols, rank, scale, transpose, out,
                              scratch, QL_COLSUM_STATIC_FLOATS, stream),
              "ql_lora_colsum_noalloc");
}

int64_t ql_lora_grads_workspace(int64_t n, const int32_t* ncols, int njobs) {
  return ql::lora_grads_workspace(n, ncols, njobs);
}

int ql_lora_grads(const ql_lora_grad_job* jobs, int njobs, int64_t n, int x_dtype, void* workspace,
                  int64_t workspace_bytes, cudaStream_t stream) {
  return done(ql::lora_grads(jobs, njobs, n, x_dtype, workspace, workspace_bytes, stream),
              "ql_lora_grads");
}

int ql_embed(const int64_t* ids, const void* W, float* h, int64_t n, int H, int64_t vocab,
             int dtype, cudaStream_t stream) {
  return done(ql::embed(ids, W, h, n, H, vocab, dtype, ql::status_word(), stream), "ql_embed");
}

int ql_embed_host(const int64_t* ids, const void* W, float* h, int64_t n, int H, int64_t vocab,
                  int dtype, cudaStream_t stream) {
  if (W == nullptr || n < 0 || H <= 0 || vocab <= 0 || (dtype != QL_F16 && dtype != QL_BF16))
    return fail(QL_STATUS_BAD_ARG, "ql_embed_host");
  // The table must be page-locked host memory mapped for this device, over its whole extent:
  // its device address (the same pointer under unified addressing) from the runtime, for the
  // first and the last byte; anything else is refused before a kernel could touch it.
  const char* first = static_cast<const char*>(W);
  const char* last = first + vocab * (int64_t)H * 2 - 1;
  cudaPointerAttributes a0{}, a1{};
  const bool ok0 = cudaPointerGetAttributes(&a0, first) == cudaSuccess;
  const bool ok1 = ok0 && cudaPointerGetAttributes(&a1, last) == cudaSuccess;
  cudaGetLastError();
  if (!ok1 || a0.type != cudaMemoryTypeHost || a1.type != cudaMemoryTypeHost ||
      a0.devicePointer == nullptr ||
      static_cast<const char*>(a1.devicePointer) !=
          static_cast<const char*>(a0.devicePointer) + (last - first)) {
    g_last_error = "ql_embed_host: the table is not page-locked host memory this device can read";
    return QL_STATUS_BAD_ARG;
  }
  return done(ql::embed_host(ids, a0.devicePointer, h, n, H, vocab, dtype, ql::status_word(),
                             stream),
              "ql_embed_host");
}

int ql_ce_rows(const ql_ce_rows_args* args, cudaStream_t stream) {
  if (args == nullptr) return fail(QL_STATUS_BAD_ARG, "ql_ce_rows");
  return done(ql::ce_rows(*args, stream), "ql_ce_rows");
}

int ql_ce_piece(const ql_ce_piece_args* args, cudaStream_t stream) {
  if (args == nullptr) return fail(QL_STATUS_BAD_ARG, "ql_ce_piece");
  return done(ql::ce_piece(*args, stream), "ql_ce_piece");
}

int ql_ce_finish(const ql_ce_finish_args* args, cudaStream_t stream) {
  if (args == nullptr) return fail(QL_STATUS_BAD_ARG, "ql_ce_finish");
  return done(ql::ce_finish(*args, stream), "ql_ce_finish");
}

}  // extern "C"

extern "C" {

int ql_attn_fwd(const ql_attn_fwd_args* args, cudaStream_t stream) {
  if (args == nullptr) return fail(QL_STATUS_BAD_ARG, "ql_attn_fwd");
  return done(ql::attn_fwd(*args, stream), "ql_attn_fwd");
}

int ql_attn_bwd(const ql_attn_bwd_args* args, cudaStream_t stream) {
  if (args == nullptr) return fail(QL_STATUS_BAD_ARG, "ql_attn_bwd");
  return done(ql::attn_bwd(*args, stream), "ql_attn_bwd");
}

int ql_exp2_fma_eval(const float* x, float* y, int64_t n, cudaStream_t stream) {
  return done(ql::exp2_fma_eval(x, y, n, stream), "ql_exp2_fma_eval");
}

int64_t ql_attn_bwd_partials_floats(int32_t n, int32_t max_len, int32_t HQ, int32_t HKV) {
  if (n <= 0 || max_len <= 0 || HKV <= 0 || HQ % HKV != 0) return 0;
  ql_attn_bwd_args a{};
  a.n = n; a.max_len = max_len; a.HQ = HQ; a.HKV = HKV;
  return ql::attn_part_q_floats(a) + 2 * ql::attn_part_kv_floats(a);
}

int ql_attn_set_deterministic(int on) {
  if (on != 0 && on != 1) return done(QL_STATUS_BAD_ARG, "ql_attn_set_deterministic");
  ql::attn_set_deterministic(on != 0);
  return QL_STATUS_OK;
}

int ql_attn_set_impl(int impl) {
  if (impl < 0 || impl > 2) return done(QL_STATUS_BAD_ARG, "ql_attn_set_impl");
  ql::attn_set_impl(impl);
  return QL_STATUS_OK;
}

}  // extern "C"

extern "C" {

int ql_gather_rows(const float* src, const int64_t* idx, float* dst, int64_t n, int H,
                   cudaStream_t stream) {
  return done(ql::gather_rows(src, idx, dst, n, H, stream), "ql_gather_rows");
}

int ql_scatter_rows(const float* src, const int64_t* idx, const float* scale, float* dst,
                    void* dst16, int64_t n, int H, int dtype, cudaStream_t stream) {
  return done(ql::scatter_rows(src, idx, scale, dst, dst16, n, H, dtype, stream),
              "ql_scatter_rows");
}

}  // extern "C"

extern "C" {

int64_t ql_layer_weight_elems(const ql_layer_desc* layer) {
  return layer == nullptr ? -1 : ql::layer_weight_elems(*layer);
}

int64_t ql_layer_workspace_bytes(const ql_layer_desc* layer, int backward) {
  return layer == nullptr ? -1 : ql::layer_workspace_bytes(*layer, backward);
}

int ql_layer_forward(const ql_layer_desc* layer, const ql_layer_saved* saved, float* h_out,
                     void* workspace, int64_t workspace_bytes, cudaStream_t stream) {
  if (layer == nullptr || saved == nullptr) return fail(QL_STATUS_BAD_ARG, "ql_layer_forward");
  return done(ql::layer_forward(*layer, *saved, h_out, workspace, workspace_bytes,
                                ql::status_word(), stream),
              "ql_layer_forward");
}

int ql_layer_backward(const ql_layer_desc* layer, const ql_layer_saved* saved, const float* dh3,
                      const void* dh3_16, float* grads, float* dh_out, void* dh16_out,
                      void* workspace, int64_t workspace_bytes, cudaStream_t stream) {
  if (layer == nullptr || saved == nullptr) return fail(QL_STATUS_BAD_ARG, "ql_layer_backward");
  return done(ql::layer_backward(*layer, *saved, dh3, dh3_16, grads, dh_out, dh16_out, workspace,
                                 workspace_bytes, ql::status_word(), stream),
              "ql_layer_backward");
}

int ql_layers_set_step(ql_layer_desc* descs, int count, const ql_layer_desc* step,
                       const int64_t* ctr_q, const int64_t* ctr_v) {
  if (descs == nullptr || step == nullptr || count < 0) return fail(QL_STATUS_BAD_ARG, "ql_layers_set_step");
  for (int i = 0; i < count; ++i) {
    ql_layer_desc& d = descs[i];
    d.cos = step->cos; d.sin = step->sin; d.pos = step->pos; d.cu_seqlens = step->cu_seqlens;
    d.tok = step->tok; d.seed = step->seed; d.threads = step->threads;
    d.ctr_q = ctr_q != nullptr ? ctr_q[i] : 0;
    d.ctr_v = ctr_v != nullptr ? ctr_v[i] : 0;
    d.p_keep = step->p_keep; d.keep_scale = step->keep_scale; d.vec = step->vec;
    d.drop_q = step->drop_q; d.drop_v = step->drop_v;
    d.n = step->n; d.B = step->B; d.max_len = step->max_len;
  }
  return QL_STATUS_OK;
}

int ql_layers_forward(const ql_layer_desc* descs, const ql_layer_saved* saved, int count,
                      float* const* h_out, void* workspace, int64_t workspace_bytes,
                      cudaStream_t stream) {
  if (descs == nullptr || saved == nullptr || h_out == nullptr || count < 0)
    return fail(QL_STATUS_BAD_ARG, "ql_layers_forward");
  return done(ql::layers_forward(descs, saved, count, h_out, workspace, workspace_bytes,
                                 ql::status_word(), stream),
              "ql_layers_forward");
}

int ql_layers_backward(const ql_layer_desc* descs, const ql_layer_saved* saved, int count,
                       float* dh, void* dh16, float* dh_alt, void* dh16_alt, float* grads,
                       const int64_t* grad_offsets, int skip_first_input_grad, void* workspace,
                       int64_t workspace_bytes, cudaStream_t stream) {
  if (descs == nullptr || saved == nullptr || grads == nullptr || grad_offsets == nullptr ||
      count < 0)
    return fail(QL_STATUS_BAD_ARG, "ql_layers_backward");
  int* err = ql::status_word();
  float* cur[2] = {dh, dh_alt};
  void* cur16[2] = {dh16, dh16_alt};
  int c = 0;
  for (int i = count - 1; i >= 0; --i) {
    const bool need = !(i == 0 && skip_first_input_grad);
    const int rc = ql::layer_backward(descs[i], saved[i], cur[c], cur16[c], grads + grad_offsets[i],
                                      need ? cur[1 - c] : nullptr, need ? cur16[1 - c] : nullptr,
                                      workspace, workspace_bytes, err, stream);
    if (rc != QL_STATUS_OK) return done(rc, "ql_layers_backward");
    c = 1 - c;
  }
  return QL_STATUS_OK;
}

}  // extern "C"

extern "C" {

int ql_profile_start(int capacity) { return done(ql::profile_start(capacity), "ql_profile_start"); }
int ql_profile_stop(void) { return done(ql::profile_stop(), "ql_profile_stop"); }
int ql_profile_read(double* count, double* ms, double* flops, double* bytes) {
  return done(ql::profile_read(count, ms, flops, bytes), "ql_profile_read");
}

}  // extern "C"
