/* C ABI of the B200 (sm_100a) fused QLoRA training step: Qwen2 + NF4 + LoRA.
 *
 * Every entry point takes caller-owned device pointers, explicit sizes, and a cudaStream_t; it
 * allocates nothing, never synchronizes the host, and returns an int status (QL_STATUS_OK = 0).
 * A launch error or an invalid argument is reported through the return value and a message
 * readable with ql_last_error(). A kernel that gives up a bounded wait records
 * QL_STATUS_TIMEOUT in the library's device status word (ql_device_status()).
 *
 * Each entry point names the reference interface it replaces (file:line inside the reference
 * project Magurin/hack-fe30cb28-opus-5-5-ultracode); the reference launches Triton kernels and
 * cuBLAS / PyTorch attention from Python, so these are the operations its launch wrappers define.
 */
#ifndef QLORA_SM100_H
#define QLORA_SM100_H

#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  QL_STATUS_OK = 0,
  QL_STATUS_BAD_ARG = 1,     /* a size, stride, alignment or dtype the kernel does not take */
  QL_STATUS_CUDA = 2,        /* a CUDA runtime / driver call failed */
  QL_STATUS_UNSUPPORTED = 3, /* a valid request this build has no kernel for */
  QL_STATUS_TIMEOUT = 4      /* a kernel gave up a bounded wait (device status word) */
};

enum { QL_F16 = 0, QL_BF16 = 1, QL_F32 = 2 };

/* ---- library ---------------------------------------------------------------------------- */
const char* ql_version(void);
/* Message of the last failed call on this host thread ("" if none). */
const char* ql_last_error(void);
/* Reads (and with clear != 0 resets) the device status word of the current device. Synchronous
 * (a device-to-host copy on the legacy stream): for tests and error paths, not the step. */
int ql_device_status(int* status_out, int clear);
/* Device address of the status word, which kernels are given to record a timeout in. */
int* ql_device_status_ptr(void);
/* Kernels launched through this library since it was loaded (all host threads). */
long long ql_launch_count(void);
/* Optional operation profiler: while started, every operation records a CUDA event before and
 * after its launches (a pool of 2 x capacity events); ql_profile_read synchronises on them and
 * returns per kind (gemm, dequant, rms_fwd, rms_bwd, rope_fwd, rope_bwd, attn_fwd, attn_bwd,
 * glu_fwd, glu_bwd, lora_colsum, ce, other: 13 entries per array) the operation count,
 * milliseconds, algorithmic FLOPs and bytes. */
int ql_profile_start(int capacity);
int ql_profile_stop(void);
int ql_profile_read(double* count, double* ms, double* flops, double* bytes);
/* Whether this library's launches carry the programmatic-dependent-launch attribute (1, the
 * default: each kernel's CTAs are scheduled while the previous kernel drains and wait for its
 * results in their first instruction) or not (0: plain stream order). A measurement switch with
 * no counterpart in the reference: per-operation event timings add up only with it off. */
int ql_set_pdl(int on);
/* Exercises the bounded waits' timeout path (a test entry point, no counterpart in the
 * reference): a one-CTA kernel whose first role waits on an mbarrier nothing arrives on, under
 * limit_ns (1 ms .. 2 s), and so records QL_STATUS_TIMEOUT in the device status word; its second
 * role gives up its own wait when it sees that status. Each role adds 1 to the device int
 * *returned when it has left its wait; ql_device_status then reports the timeout. */
int ql_wait_probe(int64_t limit_ns, int* returned, cudaStream_t stream);

/* ---- NF4 dequantisation ------------------------------------------------------------------
 * Replaces NF4Weight.dequant_into / NF4Group.dequant_into (solution/engine.py:103-109,
 * 148-157) and nf4_dequant_kernel (solution/kernels.py:68-105).
 * A [rows, cols] weight stored by bitsandbytes: element i in byte i/2 (high nibble for even i),
 * one absmax per block of bs1 = 64 consecutive elements. Non-nested: absmax is fp32 [blocks].
 * Nested (double quantisation): absmax is uint8 [blocks], the block scale is
 *   code2[absmax[b]] * absmax2[b / bs2] (rounded) + offsets[segment(b)]
 * with segment(b) = (b >= seg1) + (b >= seg2) (up to three weights stored back to back).
 * code: the 16 fp32 levels. out_dtype: QL_F16 or QL_BF16.
 * transpose = 0 writes out[rows, cols]; transpose = 1 writes out[cols, rows] (the weight's
 * transpose, the B operand of the data-gradient GEMM); it needs rows % 64 == cols % 64 == 0. */
int ql_nf4_dequant(const uint8_t* packed, const void* absmax, const float* code2,
                   const float* absmax2, const float* offsets, const float* code, void* out,
                   int64_t rows, int64_t cols, int nested, int bs2, int64_t seg1, int64_t seg2,
                   int out_dtype, int transpose, cudaStream_t stream);

/* ---- dense GEMM on tcgen05 ---------------------------------------------------------------
 * Replaces the cuBLAS torch.addmm / torch.mm calls of the step (solution/engine.py:1081-1082,
 * 1111-1112, 1132-1139, 1163-1165, 1178-1179, 1238-1301, 1386-1390).
 * C[M, N] (+)= A[M, K] . B[N, K]^T (+ bias[N]); A, B of in_dtype (QL_F16 / QL_BF16), row-major
 * with leading dimensions lda, ldb (elements, multiples of 8, 16-byte aligned bases), K % 8 == 0;
 * C of out_dtype with leading dimension ldc; accumulate (fp32 C only) adds to C; residual
 * (fp32 C only, [M, ldc] or NULL) writes C = residual + (the result rounded to in_dtype), the
 * reference's fp16 projection output added to the fp32 residual stream (solution/engine.py:
 * 1048-1051, 966 delta add).
 * workspace (256-byte aligned, or NULL): lets a GEMM with too few output tiles to fill the
 * GPU split K across SMs; partial sums are added in a fixed order (results do not depend on
 * scheduling). Its first 2048 bytes must be zero before the first call; calls leave them zero,
 * so one workspace serves every later call. ql_gemm_workspace_bytes(M, N, K) is the size a
 * shape can use (0: it never splits). */
int ql_gemm_tn(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
               const void* bias, int M, int N, int K, int in_dtype, int out_dtype, int accumulate,
               const float* residual, void* workspace, int64_t workspace_bytes,
               cudaStream_t stream);
/* C[M, N] (+)= A[M, K] . B[K, N] (+ bias[N]) with B row-major, N contiguous (ldb >= N, N % 8 ==
 * 0), read by the tensor cores as an MN-major operand: the data-gradient products dX = dY . W of
 * the reference's backward (solution/engine.py:1239, 1293, 1301, 1316) straight from the
 * forward-layout weight, with no transposed copy. Other arguments as ql_gemm_tn. */
int ql_gemm_nn(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
               const void* bias, int M, int N, int K, int in_dtype, int out_dtype, int accumulate,
               const float* residual, void* workspace, int64_t workspace_bytes,
               cudaStream_t stream);
int64_t ql_gemm_workspace_bytes(int M, int N, int K);
/* Tile kind of ql_gemm_tn / ql_gemm_nn for this process (a tuning and test switch, no counterpart
 * in the reference): mode & 3 = 0 chosen per shape by the cost model (default), 1 single-CTA
 * 128-row tiles only, 2 2-SM 256-row pair tiles (tcgen05 cta_group::2) for every shape they
 * support; mode & 4: pipeline stages of one 64-wide K chunk (one 2-D copy per 64-column box)
 * instead of two chunks in one 3-D copy per operand (the default for single-CTA tiles of up to
 * 128 columns where K is a multiple of 128). */
int ql_gemm_set_mode(int mode);

/* ---- RMSNorm with the LoRA dropout inputs --------------------------------------------------
 * Dropout fields (shared by both structs): the mask is PyTorch's CUDA dropout mask of the padded
 * [B, T, H] LoRA input, element tok[row] * H + col; seed = the CUDA generator's seed (its 64
 * bits as int64), ctr_q / ctr_v = Philox counters (generator offset / 4) of the q and v dropout
 * calls, threads = that call's grid * 256, vec = 16 / sizeof(LoRA input element), p_keep = 1-p,
 * keep_scale = 1/(1-p) (solution/engine.py:787-805, 919-927). dtype: the 16-bit compute type of
 * every void* tensor (QL_F16 / QL_BF16). rank: the LoRA rank (16 is supported). */
typedef struct {
  const float* x;       /* [n, H] fp32 residual */
  const void* delta;    /* [n, H] or NULL: x + delta is normalised and written to xsum */
  const float* w;       /* [H] norm weight (fp32) */
  float* xsum;          /* [n, H] or NULL */
  void* y;              /* [n, H] or NULL */
  void* yq;             /* [n, H] or NULL: dropped copy for the q LoRA */
  void* yv;             /* [n, H] or NULL */
  float* rstd;          /* [n] */
  const void* Aq;       /* [rank, H] or NULL: also writes xq = drop_q(y) . Aq^T */
  const void* Av;
  void* xq;             /* [n, rank] */
  void* xv;
  int32_t n, H, rank, dtype;
  float eps;
  float p_keep, keep_scale;
  int32_t vec, drop_q, drop_v;
  const int64_t* tok;   /* [n] */
  int64_t seed, ctr_q, ctr_v, threads;
  uint32_t* keep_q;     /* [n, H / 32] or NULL: the q / v dropout masks as bits (column c: bit */
  uint32_t* keep_v;     /* c % 32 of word c / 32), kept for the backward; H % 32 == 0 */
} ql_rms_fwd_args;

typedef struct {
  const void* dy;       /* [n, ld_dy] */
  int64_t ld_dy;
  const float* x;       /* [n, H] the forward's normalised input */
  const float* rstd;    /* [n] */
  const float* w;       /* [H] */
  const float* dres;    /* [n, H] or NULL: residual gradient added to dx */
  float* dx;            /* [n, H] */
  void* dx16;           /* [n, H] or NULL: dx also in the 16-bit type */
  const void* tq;       /* [n, H] or NULL: gradient w.r.t. the dropped q LoRA input */
  const void* tv;
  const float* dxlo_q;  /* [n, rank] or NULL: tq = dxlo_q . Aq formed in-kernel */
  const float* dxlo_v;
  const void* Aq;       /* [rank, H] */
  const void* Av;
  int32_t n, H, rank, dtype;
  float grad_scale;
  float p_keep, keep_scale;
  int32_t vec, drop_q, drop_v;
  const int64_t* tok;
  int64_t seed, ctr_q, ctr_v, threads;
  const uint32_t* keep_q;  /* [n, H / 32] or NULL: masks written by the forward (else the */
  const uint32_t* keep_v;  /* Philox draws are regenerated) */
} ql_rms_bwd_args;

/* Replaces _rms_fwd + rms_fwd_kernel (solution/engine.py:947-966, solution/kernels.py:145-175)
 * and the LoRA-A GEMMs xq = aq @ A^T (solution/engine.py:1088-1093). With Aq / Av, H % 64 == 0. */
int ql_rms_fwd(const ql_rms_fwd_args* args, cudaStream_t stream);
/* Replaces _rms_bwd + rms_bwd_kernel (solution/engine.py:969-981, solution/kernels.py:178-205)
 * and the tq = dx_lo @ A GEMMs (solution/engine.py:1326-1330): dx_lo is rounded to the 16-bit
 * type (the reference's fp16 dx_lo) and tq to the 16-bit type. */
int ql_rms_bwd(const ql_rms_bwd_args* args, cudaStream_t stream);
/* The keep mask (int8 0/1) of elements 0 .. nelem-1 of one dropout call; replaces
 * torch_dropout_keep_kernel (solution/kernels.py:129-135). */
int ql_dropout_keep(int8_t* out, int64_t nelem, int64_t seed, int64_t ctr, int64_t threads,
                    float p_keep, int vec, cudaStream_t stream);
/* The integer form of the keep test the kernels use: a Philox draw u is kept iff
 * u < ql_dropout_keep_threshold(p_keep), which equals the fp32 test u * 2^-32 + 2^-33 < p_keep of
 * solution/kernels.py:108-126 for every u (p_keep < 1; 0xFFFFFFFF for p_keep >= 1, where the
 * kernels keep everything without drawing). Host only. */
uint32_t ql_dropout_keep_threshold(float p_keep);

/* ---- qkv + LoRA + RoPE ---------------------------------------------------------------------
 * cos / sin: fp32 [positions, D/2] (the first half of the model's rotary table); pos: int32 [n].
 * All void* tensors are of dtype (16-bit). */
typedef struct {
  const void* qkv;      /* [n, (HQ + 2 HKV) D] biased qkv GEMM output */
  const void* lq;       /* [n, HQ D] or NULL: explicit LoRA-B output of q */
  const void* lv;       /* [n, HKV D] or NULL */
  const void* xq;       /* [n, rank] or NULL: lq = xq . Bq^T formed in-kernel */
  const void* xv;
  const void* Bq;       /* [HQ D, rank] */
  const void* Bv;       /* [HKV D, rank] */
  const float* cos;
  const float* sin;
  const int32_t* pos;
  void* q;              /* [n, HQ, D] */
  void* k;              /* [n, HKV, D] */
  void* v;              /* [n, HKV, D] */
  float lora_scale;
  int32_t n, HQ, HKV, D, rank, dtype;
} ql_rope_fwd_args;

typedef struct {
  const void* dq;       /* [n, HQ, D] of grad_dtype */
  const void* dk;       /* [n, kv_heads_in, D]: HKV, or HQ (summed over each GQA group) */
  const void* dv;
  const float* cos;
  const float* sin;
  const int32_t* pos;
  void* dqkv;           /* [n, (HQ + 2 HKV) D] of dtype: the pre-rotary gradient */
  const void* Bq;       /* [HQ D, rank] or NULL */
  const void* Bv;
  float* dxlo_q;        /* [n, rank] or NULL: s * (dqkv_q . Bq), the LoRA-A output gradient */
  float* dxlo_v;
  float lora_scale;
  int32_t n, HQ, HKV, D, kv_heads_in, rank, dtype, grad_dtype;
} ql_rope_bwd_args;

/* Replaces _rope_fwd + qkv_rope_fwd_kernel (solution/engine.py:984-997,
 * solution/kernels.py:212-264) and the LoRA-B GEMMs lq = xq @ B^T (solution/engine.py:1088-1093). */
int ql_rope_fwd(const ql_rope_fwd_args* args, cudaStream_t stream);
/* Replaces _rope_bwd + qkv_rope_bwd_kernel (solution/engine.py:1000-1009,
 * solution/kernels.py:267-306) and dx_lo = s * (g @ B) (solution/engine.py:1322-1326). */
int ql_rope_bwd(const ql_rope_bwd_args* args, cudaStream_t stream);

/* ---- SwiGLU ------------------------------------------------------------------------------ */
/* Replaces _glu_fwd + glu_fwd_kernel (solution/engine.py:1012-1017, solution/kernels.py:312-321):
 * m[n, I] = silu(gu[:, :I]) * gu[:, I:]. I % 8 == 0. */
int ql_glu_fwd(const void* gu, void* m, int64_t n, int I, int dtype, cudaStream_t stream);
/* Replaces _glu_bwd + glu_bwd_kernel (solution/engine.py:1020-1023, solution/kernels.py:324-336):
 * overwrites gu with [dL/dg | dL/du] given dm = dL/dm. */
int ql_glu_bwd(const void* dm, void* gu, int64_t n, int I, int dtype, cudaStream_t stream);

/* ---- LoRA weight gradients ---------------------------------------------------------------
 * Replaces db_w = (g^T @ x_lo) * s and da_w = dx_lo^T @ a_in (solution/engine.py:1322-1328):
 * out[i, r] (transpose = 0) or out[r, i] (transpose = 1) = scale * sum_t X[t, i] * Y[t, r],
 * X [n, ldx] (x_dtype 16-bit), Y [n, rank] (y_dtype 16-bit or QL_F32), out fp32. Deterministic:
 * per-split partials go to workspace (ql_lora_colsum_workspace floats), summed in fixed order. */
int64_t ql_lora_colsum_workspace(int64_t n, int ncols, int rank);
int ql_lora_colsum(const void* X, int64_t ldx, int x_dtype, const void* Y, int y_dtype, int64_t n,
                   int ncols, int rank, float scale, int transpose, float* out, float* workspace,
                   int64_t workspace_floats, cudaStream_t stream);

/* ---- the LoRA weight gradients of a layer in one launch -----------------------------------
 * Replaces the four LoRA weight-gradient GEMMs of _Layer.backward (solution/engine.py:1322-1328):
 * up to 4 products out_j = scale_j * X_j^T Y_j over the same n tokens. X_j: [n, ncols_j] 16-bit
 * (x_dtype) with row stride ldx_j (a column slice is fine; ncols_j, ldx_j multiples of 4, X_j
 * 8-byte aligned); Y_j: [n, rank = 16] of y_dtype_j (16-bit or QL_F32); out_j fp32 [ncols_j, 16],
 * or [16, ncols_j] with transpose_j. The tokens are split over CTAs; each 64-column block's last
 * split adds the splits' partials in split order (deterministic) and writes out_j. workspace:
 * ql_lora_grads_workspace(...) bytes, 256-byte aligned, its first 2048 bytes zero before the first
 * call (block counters; calls leave them zero). */
typedef struct {
  const void* X;
  int64_t ldx;
  const void* Y;
  float* out;
  int32_t ncols, y_dtype, transpose;
  float scale;
} ql_lora_grad_job;
int64_t ql_lora_grads_workspace(int64_t n, const int32_t* ncols, int njobs);
int ql_lora_grads(const ql_lora_grad_job* jobs, int njobs, int64_t n, int x_dtype, void* workspace,
                  int64_t workspace_bytes, cudaStream_t stream);

/* ---- LoRA column sums with the scratch built in (no counterpart in the reference) ---------
 * The same operation and results as ql_lora_colsum, but the per-split partial sums go to a
 * scratch array compiled into this library (static device memory, QL_COLSUM_STATIC_FLOATS floats
 * = 4 MiB per device) instead of a caller workspace. For callers that cannot allocate device
 * memory: a plain C or ctypes host with no device allocator of its own (cudaMalloc would stall the
 * whole device mid-step), or a runtime that plans all device memory at start-up.
 * Limit: shapes whose ql_lora_colsum_workspace(n, ncols, rank) exceeds QL_COLSUM_STATIC_FLOATS
 * (ncols above about 65,000 columns) return QL_STATUS_BAD_ARG, the sizes in ql_last_error().
 * Nothing in the scratch has to start at zero: each call writes every partial before reading it.
 * The first call on a device looks up the scratch's address there (cudaGetSymbolAddress, the
 * caller's current device) and keeps it; make that first call before any stream capture.
 * One scratch per device: calls that overlap on a device (other streams or host threads) race
 * on it and can return wrong sums; serialise them. */
enum { QL_COLSUM_STATIC_FLOATS = 1048576 };
int ql_lora_colsum_noalloc(const void* X, int64_t ldx, int x_dtype, const void* Y, int y_dtype,
                           int64_t n, int ncols, int rank, float scale, int transpose, float* out,
                           cudaStream_t stream);

/* ---- embedding ---------------------------------------------------------------------------
 * Replaces the embedding lookup of FusedQwen2.step (solution/engine.py:1904-1907):
 * h[t, :] = float(W[ids[t], :]). An id outside [0, vocab) records QL_STATUS_BAD_ARG in the
 * device status word and yields a zero row. */
int ql_embed(const int64_t* ids, const void* W, float* h, int64_t n, int H, int64_t vocab,
             int dtype, cudaStream_t stream);

/* The same lookup from a table in page-locked host memory, read by the kernel over the host link
 * (the reference keeps the embedding in host memory, solution/offload.py:55-111 and
 * solution/engine.py:1763-1771): W must be pinned and mapped for the current device over all of
 * its vocab * H 16-bit entries (checked with cudaPointerGetAttributes; otherwise
 * QL_STATUS_BAD_ARG and nothing is launched). */
int ql_embed_host(const int64_t* ids, const void* W, float* h, int64_t n, int H, int64_t vocab,
                  int dtype, cudaStream_t stream);

/* ---- cross-entropy head ------------------------------------------------------------------ */
typedef struct {
  void* logits;         /* [rows, ld] 16-bit, overwritten by the gradient */
  const int64_t* target;/* [rows], < 0: no target */
  float* loss;          /* [rows] */
  float* entropy;       /* [rows] */
  int32_t* correct;     /* [rows] */
  int64_t rows, V, ld;
  int32_t write_grad, zero_unsupervised, dtype;
} ql_ce_rows_args;

typedef struct {
  void* logits;         /* [rows, ld] logits of vocabulary [v0, v0 + width) */
  const void* w;        /* [width, H] the piece of the lm_head weight */
  const int64_t* target;
  float* state;         /* [rows, 4] (max, sum exp, sum exp * x, best); start -inf, 0, 0, -inf */
  int64_t* best_idx;    /* [rows] */
  float* xt;            /* [rows] target logit */
  float* alpha;         /* [n_sup] rescale of earlier pieces' accumulation */
  void* wt;             /* [n_sup, H] or NULL: the target's weight row */
  int64_t rows, v0, width, ld, n_sup;
  int32_t H, dtype;
  float* acc;           /* [n_sup, H] or NULL: fp32 gradient accumulator, moved to this piece's
                           running max in place: acc = alpha (acc + part); zeroed at the first
                           piece (state max -inf) */
  const float* part;    /* [n_sup, H]: the previous piece's product exp(x - max) . W_piece */
  int32_t part_valid;   /* whether `part` holds a product yet (0 before the first one) */
} ql_ce_piece_args;

typedef struct {
  const float* state;
  const int64_t* best_idx;
  const float* xt;
  const int64_t* target;
  float* loss;
  float* entropy;
  int32_t* correct;
  const float* acc;     /* [n_sup, H] sum_v exp(x_v - max) W_v */
  const void* wt;       /* [n_sup, H] */
  void* dh;             /* [n_sup, H] (acc + part) / s - W_target */
  int64_t rows, n_sup;
  int32_t H, dtype;
  const float* part;    /* [n_sup, H] or NULL: the last piece's product, not yet in acc */
} ql_ce_finish_args;

/* Replaces _ce + lm_head_ce_kernel (solution/engine.py:1026-1030, solution/kernels.py:344-388). */
int ql_ce_rows(const ql_ce_rows_args* args, cudaStream_t stream);
/* Replaces _ce_piece + lm_head_piece_kernel (solution/engine.py:1033-1038,
 * solution/kernels.py:401-450). */
int ql_ce_piece(const ql_ce_piece_args* args, cudaStream_t stream);
/* Replaces _ce_finish + lm_head_finish_kernel (solution/engine.py:1041-1045,
 * solution/kernels.py:458-479). */
int ql_ce_finish(const ql_ce_finish_args* args, cudaStream_t stream);

/* ---- varlen causal GQA attention ----------------------------------------------------------
 * Replaces _attn_fwd / _attn_bwd, PyTorch's memory-efficient attention over cu_seqlens
 * (solution/engine.py:857-869). q [n, HQ, D], k / v [n, HKV, D] (not expanded: each KV head
 * serves HQ / HKV query heads), cu_seqlens int32 [B + 1], causal, D = 128. */
typedef struct {
  const void* q;
  const void* k;
  const void* v;
  const int32_t* cu_seqlens;
  void* out;            /* [n, HQ, D] */
  float* lse;           /* [HQ, n] natural-log logsumexp of the scaled scores */
  float scale;
  int32_t n, B, max_len, HQ, HKV, D, dtype;
} ql_attn_fwd_args;

typedef struct {
  const void* q;
  const void* k;
  const void* v;
  const void* out;
  const void* dout;     /* [n, HQ, D] */
  const float* lse;
  const int32_t* cu_seqlens;
  float* dvec;          /* [HQ, n] workspace: rowsum(dout * out) */
  float* dq;            /* [n, HQ, D] fp32 (zeroed by the call) */
  float* dk;            /* [n, HKV, D] fp32, summed over each GQA group */
  float* dv;
  float scale;
  int32_t n, B, max_len, HQ, HKV, D, dtype;
  float* partials;      /* NULL, or ql_attn_bwd_partials_floats(...) floats: the deterministic
                           form (D = 128 tcgen05 kernels): each contribution to dq / dk / dv goes
                           to its own slot and one kernel sums the slots in a fixed order, instead
                           of fp32 reductions whose order varies from run to run */
} ql_attn_bwd_args;

int ql_attn_fwd(const ql_attn_fwd_args* args, cudaStream_t stream);
int ql_attn_bwd(const ql_attn_bwd_args* args, cudaStream_t stream);
/* Which kernels serve D = 128 (forward and backward): 0 (default) the tcgen05 kernels (TMEM
 * accumulators, TMA tiles), 1 the warp-level mma.sync kernels (always used for D = 64), 2 the
 * tcgen05 kernels.
 * No counterpart in the reference (one attention implementation there); tests and the
 * microbenchmark compare the two. */
int ql_attn_set_impl(int impl);
/* Size in floats of the deterministic attention backward's partials for a batch of n tokens
 * whose longest sequence has max_len tokens (D = 128). */
int64_t ql_attn_bwd_partials_floats(int32_t n, int32_t max_len, int32_t HQ, int32_t HKV);
/* Whether ql_layer_backward runs the attention backward in its deterministic form (1) or with
 * fp32 bulk reductions (0, the default: faster, not bit-reproducible run to run); the layer
 * workspace grows by the partials when on. A process-wide switch with no counterpart in the
 * reference, for reproducible gradients (the memory-plan and determinism tests). */
int ql_attn_set_deterministic(int on);
/* y[i] = 2^x[i] by the FMA-pipe polynomial the tcgen05 attention forward's softmax uses for half
 * of its off-diagonal exponentials (a check of its error bound against the GPU's exp2; no counterpart in
 * the reference). */
int ql_exp2_fma_eval(const float* x, float* y, int64_t n, cudaStream_t stream);

/* ---- head row order ----------------------------------------------------------------------
 * The head takes rows with a target first (solution/engine.py:731, 1364-1398):
 * gather: dst[i, :] = src[idx[i], :]; scatter: dst[idx[i], :] = src[i, :] * (*scale) (scale is a
 * device pointer, e.g. the loss's upstream gradient, or NULL for 1), also into the 16-bit dst16
 * when given. fp32 rows of H values (gather needs H % 4 == 0). */
int ql_gather_rows(const float* src, const int64_t* idx, float* dst, int64_t n, int H,
                   cudaStream_t stream);
int ql_scatter_rows(const float* src, const int64_t* idx, const float* scale, float* dst,
                    void* dst16, int64_t n, int H, int dtype, cudaStream_t stream);

/* ---- one decoder layer, forward and backward ----------------------------------------------
 * Replaces _Layer.forward / _Layer.backward (solution/engine.py:1184-1340) with keep-everything
 * semantics: the forward writes every intermediate the backward reads into caller-owned
 * buffers (ql_layer_saved), the backward reads them and recomputes nothing. Both launch the
 * kernels above in the reference's order on one stream; temporaries live in a caller-owned
 * workspace of ql_layer_workspace_bytes() bytes. */
typedef struct {
  const uint8_t* packed;   /* NF4 bytes of the group's weights back to back */
  const void* absmax;      /* fp32 [blocks] or (nested) uint8 [blocks] */
  const float* code;       /* [16] */
  const float* code2;      /* nested: [256] */
  const float* absmax2;    /* nested: [ceil(blocks / bs2)] over the whole group */
  const float* offsets;    /* nested: [members] */
  int64_t rows, cols, seg1, seg2;
  int32_t nested, bs2;
} ql_nf4_weight;

/* Many NF4 weights dequantised in as few launches as possible (one per 28 weights): out[i] gets
 * weights[i] [rows, cols] as ql_nf4_dequant with transpose = 0. Replaces the reference's
 * per-group dequant_into calls (solution/engine.py:103-109, 148-157) at the start of a step: all
 * layers' groups at once instead of four small launches per layer. */
int ql_nf4_dequant_batch(const ql_nf4_weight* weights, void* const* outs, int count, int out_dtype,
                         cudaStream_t stream);

/* GEMM with the NF4 weight dequantised inside the kernel (shared memory only, the 16-bit weight
 * never reaches HBM): replaces the reference's dequant_into + cuBLAS pairs (solution/engine.py:
 * 103-109 with 1081-1093, 1111-1112, 1132-1139, 1163-1165, 1178-1179, and 1239, 1293, 1301,
 * 1316 in the backward). layout 0: C[M, N] (+)= A[M, K] . W^T with W [N, K] (W.cols % 64 == 0);
 * layout 1: C[M, N] (+)= A[M, K] . W with W [K, N] (N % 64 == 0). Dequantisation is the
 * reference's (level x scale in fp32, rounded once to in_dtype; nested scales as ql_nf4_dequant),
 * so the result equals ql_nf4_dequant followed by ql_gemm_tn / ql_gemm_nn. Other arguments as
 * ql_gemm_tn (no workspace: no split-K). */
int ql_gemm_nf4(const void* A, int64_t lda, const ql_nf4_weight* W, int layout, void* C,
                int64_t ldc, const void* bias, int M, int in_dtype, int out_dtype, int accumulate,
                const float* residual, cudaStream_t stream);

typedef struct {
  ql_nf4_weight qkv, o, gu, down;   /* [C, H], [H, HQ D], [2 I, H] (gate rows, then up), [H, I] */
  const void* bias_qkv;             /* [C] */
  const float* ln1;                 /* [H] */
  const float* ln2;
  const void* Aq;                   /* LoRA in the 16-bit type: A [rank, H], B [out, rank] */
  const void* Bq;
  const void* Av;
  const void* Bv;
  const float* cos;                 /* [positions, D/2] */
  const float* sin;
  const int32_t* pos;               /* [n] */
  const int32_t* cu_seqlens;        /* [B + 1] */
  const int64_t* tok;               /* [n] padded-batch index of each token (dropout) */
  int64_t seed, ctr_q, ctr_v, threads;
  float p_keep, keep_scale, eps, scale, lora_scale;
  int32_t vec, drop_q, drop_v;
  int32_t n, B, max_len, H, HQ, HKV, D, I, rank, dtype;
} ql_layer_desc;

typedef struct {              /* what the forward keeps for the backward (all [n, ...]) */
  const float* h;             /* [n, H] fp32 layer input */
  float* rstd1;               /* [n] */
  void* yq;                   /* [n, H] dropped LoRA inputs */
  void* yv;
  void* xq;                   /* [n, rank] LoRA-A outputs */
  void* xv;
  void* q;                    /* [n, HQ, D] */
  void* k;                    /* [n, HKV, D] */
  void* v;
  void* out;                  /* [n, HQ, D] attention output */
  float* lse;                 /* [HQ, n] */
  float* h2;                  /* [n, H] residual after attention */
  float* rstd2;               /* [n] */
  void* gu;                   /* [n, 2 I] [gate | up] (overwritten by its gradient in backward) */
  uint32_t* keep_q;           /* [n, H / 32] dropout masks of the q / v LoRA inputs as bits */
  uint32_t* keep_v;
  void* w16;                  /* NULL, or ql_layer_weight_elems() 16-bit elements: the forward's
                                 dequantised weights [qkv | o | gate_up | down], read again by
                                 the backward instead of a second dequantisation */
  int32_t w16_ready;          /* 1: w16 already holds this step's dequantised weights (e.g. from
                                 one ql_nf4_dequant_batch over all layers): no dequant here */
} ql_layer_saved;

/* Elements of ql_layer_saved.w16 for a layer: (HQ + 2 HKV) D H + H HQ D + 3 I H. */
int64_t ql_layer_weight_elems(const ql_layer_desc* layer);

/* Workspace bytes of the forward (backward = 0) or backward (backward = 1) of a layer. Its first
 * 2048 bytes must be zero before the first call (GEMM tile counters); calls leave them zero. */
int64_t ql_layer_workspace_bytes(const ql_layer_desc* layer, int backward);
/* h_out [n, H] fp32: the layer's output (the next layer's input). */
int ql_layer_forward(const ql_layer_desc* layer, const ql_layer_saved* saved, float* h_out,
                     void* workspace, int64_t workspace_bytes, cudaStream_t stream);
/* dh3 / dh3_16: gradient of the layer's output (fp32 and 16-bit). Writes the LoRA gradients
 * into grads = [dAq (rank x H) | dBq (HQ D x rank) | dAv (rank x H) | dBv (HKV D x rank)] fp32,
 * and, when dh_out is not NULL, the gradient of the layer's input (dh_out fp32, dh16_out 16-bit). */
int ql_layer_backward(const ql_layer_desc* layer, const ql_layer_saved* saved, const float* dh3,
                      const void* dh3_16, float* grads, float* dh_out, void* dh16_out,
                      void* workspace, int64_t workspace_bytes, cudaStream_t stream);

/* ---- all layers of a step in one call -------------------------------------------------------
 * The same work as the per-layer calls above, looped over the layers in the library, for a host
 * that would otherwise pay its own per-call overhead 2 L times a step (no counterpart in the
 * reference, whose layer loop is Python: solution/engine.py:1904-1913). */
/* The step-dependent fields of every layer descriptor at once: cos .. max_len copied from `step`
 * into descs[0 .. count-1], and layer i's dropout counters from ctr_q[i] / ctr_v[i] (NULL: 0).
 * Host only, no launch. */
int ql_layers_set_step(ql_layer_desc* descs, int count, const ql_layer_desc* step,
                       const int64_t* ctr_q, const int64_t* ctr_v);
/* ql_layer_forward for layers 0 .. count-1 in order, h_out[i] = saved[i + 1].h for i < count - 1
 * (QL_STATUS_BAD_ARG otherwise). Between layers the residual stream goes through the norms: layer
 * i's down projection is handed on in the 16-bit type and layer i + 1's input RMSNorm writes
 * saved[i + 1].h = saved[i].h2 + d (the same fp32 addition of the rounded projection the
 * per-layer call does in its down GEMM); the last layer writes h_out[count - 1] itself. */
int ql_layers_forward(const ql_layer_desc* descs, const ql_layer_saved* saved, int count,
                      float* const* h_out, void* workspace, int64_t workspace_bytes,
                      cudaStream_t stream);
/* ql_layer_backward for layers count-1 .. 0. The top layer takes (dh, dh16), the gradient of its
 * output; each layer's input gradient goes to the other buffer pair, (dh_alt, dh16_alt) then
 * (dh, dh16) and so on, and feeds the layer below; layer 0's is not formed when
 * skip_first_input_grad (its input is the frozen embedding). grads: the flat fp32 LoRA gradients,
 * layer i's at grads + grad_offsets[i] floats. */
int ql_layers_backward(const ql_layer_desc* descs, const ql_layer_saved* saved, int count,
                       float* dh, void* dh16, float* dh_alt, void* dh16_alt, float* grads,
                       const int64_t* grad_offsets, int skip_first_input_grad, void* workspace,
                       int64_t workspace_bytes, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* QLORA_SM100_H */
