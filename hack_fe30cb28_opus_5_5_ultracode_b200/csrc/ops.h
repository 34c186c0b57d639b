// Internal C++ entry points of the kernels (namespace ql); capi.cu wraps them as extern "C".
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/qlora_sm100.h"

namespace ql {

int* status_word();

int nf4_dequant_batch(const ql_nf4_weight* w, void* const* outs, int count, int out_dtype,
                      cudaStream_t s);
int nf4_dequant(const uint8_t* packed, const void* absmax, const float* code2,
                const float* absmax2, const float* offsets, const float* code, void* out,
                int64_t rows, int64_t cols, int nested, int bs2, int64_t seg1, int64_t seg2,
                int out_dtype, int transpose, cudaStream_t stream);

int gemm_tn(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
            const void* bias, int M, int N, int K, int in_dtype, int out_dtype, int accumulate,
            const float* residual, int* err, cudaStream_t stream, void* workspace = nullptr,
            int64_t workspace_bytes = 0);
int gemm_nn(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
            const void* bias, int M, int N, int K, int in_dtype, int out_dtype, int accumulate,
            const float* residual, int* err, cudaStream_t stream, void* workspace = nullptr,
            int64_t workspace_bytes = 0);
int64_t gemm_workspace_bytes(int M, int N, int K);
void gemm_set_mode(int mode);

typedef ql_rms_fwd_args RmsFwdC;
typedef ql_rms_bwd_args RmsBwdC;
int rms_fwd(const RmsFwdC& c, cudaStream_t s);
int rms_bwd(const RmsBwdC& c, cudaStream_t s);
int dropout_keep(int8_t* out, int64_t nelem, int64_t seed, int64_t ctr, int64_t threads,
                 float p_keep, int vec, cudaStream_t s);

}  // namespace ql

namespace ql {
typedef ql_rope_fwd_args RopeFwdC;
typedef ql_rope_bwd_args RopeBwdC;
typedef ql_ce_rows_args CeRowsC;
typedef ql_ce_piece_args CePieceC;
typedef ql_ce_finish_args CeFinishC;
int rope_fwd(const RopeFwdC& a, cudaStream_t s);
int rope_bwd(const RopeBwdC& a, cudaStream_t s);
int glu_fwd(const void* gu, void* m, int64_t n, int I, int dtype, cudaStream_t s);
int glu_bwd(const void* dm, void* gu, int64_t n, int I, int dtype, cudaStream_t s);
int lora_colsum_splits(int64_t n, int ncols);
int64_t lora_grads_workspace(int64_t n, const int32_t* ncols, int njobs);
int lora_grads(const ql_lora_grad_job* jobs, int njobs, int64_t n, int x_dtype, void* workspace,
               int64_t workspace_bytes, cudaStream_t s);
int lora_colsum(const void* X, int64_t ldx, int x_dtype, const void* Y, int y_dtype, int64_t n,
                int ncols, int rank, float scale, int transpose, float* out, float* workspace,
                int64_t workspace_floats, cudaStream_t s);
int embed_host(const int64_t* ids, const void* W_dev, float* h, int64_t n, int H, int64_t vocab,
               int dtype, int* err, cudaStream_t s);
int embed(const int64_t* ids, const void* W, float* h, int64_t n, int H, int64_t vocab,
          int dtype, int* err, cudaStream_t s);
int ce_rows(const CeRowsC& a, cudaStream_t s);
int ce_piece(const CePieceC& a, cudaStream_t s);
int ce_finish(const CeFinishC& a, cudaStream_t s);
}  // namespace ql

namespace ql {
typedef ql_attn_fwd_args AttnFwdC;
typedef ql_attn_bwd_args AttnBwdC;
// Queries per CTA of the tcgen05 attention backward (a chunk of a key block's queries, from its
// diagonal on): 256 for sequences of up to 2,048 tokens, so the longest key block's walk is four
// 64-query blocks and the work spreads over the SMs instead of waiting on one long chain; 1,024
// for longer ones, where every chain is long enough to keep the tensor cores busy.
__host__ __device__ inline int attn_bwd_qch(int max_len) { return max_len <= 2048 ? 256 : 1024; }
// The deterministic attention backward's partials (D = 128): the dq contributions of each
// 128-key block, [ceil(max_len / 128)][n][HQ][128]; then the dk, and the dv, contributions of
// each (query head of the GQA group, query chunk), [HQ / HKV][ceil(max_len / qch)][n][HKV][128]
// each.
__host__ __device__ inline int64_t attn_part_q_floats(const AttnBwdC& a) {
  return (int64_t)((a.max_len + 127) / 128) * a.n * a.HQ * 128;
}
__host__ __device__ inline int64_t attn_part_kv_floats(const AttnBwdC& a) {
  const int qch = attn_bwd_qch(a.max_len);
  return (int64_t)(a.HQ / a.HKV) * ((a.max_len + qch - 1) / qch) * a.n * a.HKV * 128;
}
void attn_set_deterministic(bool on);
bool attn_deterministic();
int attn_fwd(const AttnFwdC& a, cudaStream_t s);
int attn_fwd_tc(const AttnFwdC& a, cudaStream_t s);  // D = 128 on tcgen05 (launch only)
int attn_bwd_tc(const AttnBwdC& a, cudaStream_t s);  // D = 128 on tcgen05 (main kernel only)
void attn_set_impl(int impl);
int exp2_fma_eval(const float* x, float* y, int64_t n, cudaStream_t s);
int attn_bwd(const AttnBwdC& a, cudaStream_t s);
}  // namespace ql

namespace ql {
int gather_rows(const float* src, const int64_t* idx, float* dst, int64_t n, int H, cudaStream_t s);
int scatter_rows(const float* src, const int64_t* idx, const float* scale, float* dst, void* dst16,
                 int64_t n, int H, int dtype, cudaStream_t s);
}  // namespace ql

namespace ql {
int gemm_nf4(const void* A, int64_t lda, const ql_nf4_weight& W, int layout, void* C, int64_t ldc,
             const void* bias, int M, int in_dtype, int out_dtype, int accumulate,
             const float* residual, int* err, cudaStream_t stream);
int64_t layer_workspace_bytes(const ql_layer_desc& L, int backward);
int64_t layer_weight_elems(const ql_layer_desc& L);
int layer_forward(const ql_layer_desc& L, const ql_layer_saved& S, float* h_out, void* ws,
                  int64_t ws_bytes, int* err, cudaStream_t s, const float* x_base = nullptr,
                  const void* d_in = nullptr, void* d_out = nullptr);
int layers_forward(const ql_layer_desc* descs, const ql_layer_saved* saved, int count,
                   float* const* h_out, void* ws, int64_t ws_bytes, int* err, cudaStream_t s);
int layer_backward(const ql_layer_desc& L, const ql_layer_saved& S, const float* dh3,
                   const void* dh3_16, float* grads, float* dh_out, void* dh16_out, void* ws,
                   int64_t ws_bytes, int* err, cudaStream_t s);
}  // namespace ql

namespace ql {
int profile_start(int capacity);
int profile_stop();
int profile_read(double* count, double* ms, double* flops, double* bytes);
}  // namespace ql
