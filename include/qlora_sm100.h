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
 * C of out_dtype with leading dimension ldc; accumulate (fp32 C only) adds to C. */
int ql_gemm_tn(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
               const void* bias, int M, int N, int K, int in_dtype, int out_dtype, int accumulate,
               cudaStream_t stream);

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
} ql_rms_bwd_args;

/* Replaces _rms_fwd + rms_fwd_kernel (solution/engine.py:947-966, solution/kernels.py:145-175)
 * and the LoRA-A GEMMs xq = aq @ A^T (solution/engine.py:1088-1093). */
int ql_rms_fwd(const ql_rms_fwd_args* args, cudaStream_t stream);
/* Replaces _rms_bwd + rms_bwd_kernel (solution/engine.py:969-981, solution/kernels.py:178-205)
 * and the tq = dx_lo @ A GEMMs (solution/engine.py:1326-1330). */
int ql_rms_bwd(const ql_rms_bwd_args* args, cudaStream_t stream);
/* The keep mask (int8 0/1) of elements 0 .. nelem-1 of one dropout call; replaces
 * torch_dropout_keep_kernel (solution/kernels.py:129-135). */
int ql_dropout_keep(int8_t* out, int64_t nelem, int64_t seed, int64_t ctr, int64_t threads,
                    float p_keep, int vec, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* QLORA_SM100_H */
