// The library's optional operation profiler (see profile.h).
#include <mutex>
#include <vector>

#include "common.cuh"
#include "profile.h"

namespace ql {
namespace {
struct Rec {
  int kind;
  double flops, bytes;
  cudaEvent_t start, end;
};
std::mutex g_mu;
bool g_on = false;
std::vector<cudaEvent_t> g_pool;
size_t g_next = 0;
std::vector<Rec> g_recs;
}  // namespace

bool profiling() { return g_on; }

cudaEvent_t profile_event() {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_next >= g_pool.size()) return nullptr;  // pool exhausted: the op goes unrecorded
  return g_pool[g_next++];
}

void profile_record(int kind, double flops, double bytes, cudaEvent_t start, cudaEvent_t end) {
  std::lock_guard<std::mutex> lk(g_mu);
  g_recs.push_back(Rec{kind, flops, bytes, start, end});
}

int profile_start(int capacity) {
  std::lock_guard<std::mutex> lk(g_mu);
  while ((int)g_pool.size() < 2 * capacity) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return QL_STATUS_CUDA;
    g_pool.push_back(e);
  }
  g_next = 0;
  g_recs.clear();
  g_on = true;
  return QL_STATUS_OK;
}

int profile_stop() {
  std::lock_guard<std::mutex> lk(g_mu);
  g_on = false;
  return QL_STATUS_OK;
}

// per kind: launches, milliseconds, FLOPs, bytes (arrays of PK_COUNT doubles each)
int profile_read(double* count, double* ms, double* flops, double* bytes) {
  std::lock_guard<std::mutex> lk(g_mu);
  for (int k = 0; k < PK_COUNT; ++k) count[k] = ms[k] = flops[k] = bytes[k] = 0;
  for (const Rec& r : g_recs) {
    if (cudaEventSynchronize(r.end) != cudaSuccess) return QL_STATUS_CUDA;
    float t = 0.f;
    if (cudaEventElapsedTime(&t, r.start, r.end) != cudaSuccess) return QL_STATUS_CUDA;
    count[r.kind] += 1;
    ms[r.kind] += t;
    flops[r.kind] += r.flops;
    bytes[r.kind] += r.bytes;
  }
  return QL_STATUS_OK;
}

}  // namespace ql
