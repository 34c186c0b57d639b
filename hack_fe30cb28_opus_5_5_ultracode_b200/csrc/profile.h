// Optional per-operation timing inside the library: while enabled (ql_profile_start), every
// operation records a CUDA event before and after its launches on its stream, tagged with its
// kind and its algorithmic FLOPs and bytes. ql_profile_read sums them per kind. Off by default;
// an event pair costs a few microseconds of host time per operation.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ql {

enum ProfKind {
  PK_GEMM = 0, PK_DEQUANT, PK_RMS_FWD, PK_RMS_BWD, PK_ROPE_FWD, PK_ROPE_BWD, PK_ATTN_FWD,
  PK_ATTN_BWD, PK_GLU_FWD, PK_GLU_BWD, PK_COLSUM, PK_CE, PK_OTHER, PK_COUNT
};

bool profiling();
void profile_record(int kind, double flops, double bytes, cudaEvent_t start, cudaEvent_t end);
cudaEvent_t profile_event();

struct ProfScope {
  int kind;
  double flops, bytes;
  cudaStream_t stream;
  cudaEvent_t start = nullptr;
  ProfScope(int k, double f, double b, cudaStream_t s) : kind(k), flops(f), bytes(b), stream(s) {
    if (profiling()) {
      start = profile_event();
      if (start != nullptr) cudaEventRecord(start, stream);
    }
  }
  ~ProfScope() {
    if (start != nullptr) {
      cudaEvent_t end = profile_event();
      if (end != nullptr) {
        cudaEventRecord(end, stream);
        profile_record(kind, flops, bytes, start, end);
      }
    }
  }
};

}  // namespace ql
