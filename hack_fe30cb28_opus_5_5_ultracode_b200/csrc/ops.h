// Internal C++ entry points of the kernels (namespace ql); capi.cu wraps them as extern "C".
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/qlora_sm100.h"

namespace ql {

int* status_word();

int nf4_dequant(const uint8_t* packed, const void* absmax, const float* code2,
                const float* absmax2, const float* offsets, const float* code, void* out,
                int64_t rows, int64_t cols, int nested, int bs2, int64_t seg1, int64_t seg2,
                int out_dtype, int transpose, cudaStream_t stream);

int gemm_tn(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
            const void* bias, int M, int N, int K, int in_dtype, int out_dtype, int accumulate,
            int* err, cudaStream_t stream);

typedef ql_rms_fwd_args RmsFwdC;
typedef ql_rms_bwd_args RmsBwdC;
int rms_fwd(const RmsFwdC& c, cudaStream_t s);
int rms_bwd(const RmsBwdC& c, cudaStream_t s);
int dropout_keep(int8_t* out, int64_t nelem, int64_t seed, int64_t ctr, int64_t threads,
                 float p_keep, int vec, cudaStream_t s);

}  // namespace ql
