// PyTorch's CUDA dropout keep mask, bit for bit, as a pure function of the element index.
//
// Follows the reference's restatement (solution/kernels.py:108-126): element e of the contiguous
// [B, T, H] LoRA input is drawn by thread t = (e / VEC) % G of the dropout kernel's G threads, at
// Philox counter ctr + (e / VEC / G) * (VEC / 4) + (e % VEC) / 4, component e % 4, and is kept iff
// u * 2^-32 + 2^-33 < 1 - p (fp32). Philox4x32-10 (key = seed, counter = (c_lo, c_hi, t, 0)) is
// written from Salmon et al., "Parallel random numbers: as easy as 1, 2, 3" (SC'11).
#pragma once
#include <stdint.h>

namespace ql {

// Division of 32-bit unsigned integers by a divisor fixed at launch, by a multiply-high and a
// shift (Granlund & Montgomery, "Division by invariant integers using multiplication", 1994):
// for d >= 1, l = ceil(log2 d), m = floor(2^32 (2^l - d) / d) + 1,
// n / d = (t + ((n - t) >> 1)) >> (l - 1) with t = mulhi(m, n)   (l >= 1; d = 1 is n itself).
struct FastDiv {
  uint32_t d, m, l;
};

__host__ __device__ inline FastDiv make_fastdiv(uint32_t d) {
  FastDiv f{d, 0u, 0u};
  while (f.l < 32 && (1ull << f.l) < d) ++f.l;
  f.m = (uint32_t)(((1ull << 32) * ((1ull << f.l) - d)) / d + 1);
  return f;
}

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
  if (f.l == 0) return n;  // d == 1
  const uint32_t t = __umulhi(f.m, n);
  return (t + ((n - t) >> 1)) >> (f.l - 1);
}

struct DropoutArgs {
  const int64_t* tok;  // [n] each packed token's index in the padded [B, T] batch
  int64_t seed;        // the generator's seed, its 64 bits as an int64
  int64_t ctr_q, ctr_v;  // Philox counters (offset / 4) of the q and v masks
  int64_t threads;     // G = dropout grid * 256
  float p_keep, keep_scale;
  int vec;             // 16 / sizeof(LoRA input element): 4 for fp32
  int drop_q, drop_v;  // which masks exist
  FastDiv div_threads; // division by `threads`, set by the launcher (prepare_dropout)
  uint32_t keep_below; // a draw u is kept iff u < keep_below (set by prepare_dropout)
};

// Host: the keep test u * 2^-32 + 2^-33 < p_keep, evaluated in fp32 as the dropout kernel does
// (u rounded to fp32, an exact power-of-two product, one rounded add), is non-decreasing in u, so
// the kept draws are exactly u < U* for the least u whose value reaches p_keep; found by
// bisection over [0, 2^32) with the same fp32 operations (p_keep < 1: the largest u reaches 1).
inline float keep_value(uint32_t u) {
  volatile float f = static_cast<float>(u);  // round to nearest, as __uint2float_rn
  volatile float g = f * 2.3283064365386963e-10f;
  volatile float h = g + 1.1641532182693481e-10f;
  return h;
}

inline uint32_t keep_threshold(float p_keep) {
  uint64_t lo = 0, hi = 0xFFFFFFFFull;  // keep_value(hi) = 1 >= p_keep
  while (lo < hi) {
    const uint64_t mid = (lo + hi) >> 1;
    if (keep_value((uint32_t)mid) >= p_keep) hi = mid;
    else lo = mid + 1;
  }
  return (uint32_t)lo;
}

// Host: completes a DropoutArgs before launch. The element indices of a mask stay below 2^32
// (B T H < 4.3e9), so the per-element index math runs in 32 bits.
inline bool prepare_dropout(DropoutArgs& d) {
  if (d.threads <= 0 || d.threads > 0xFFFFFFFFll) return false;
  d.div_threads = make_fastdiv((uint32_t)d.threads);
  // the threshold of the last probability asked for (one per training run, normally)
  thread_local float last_p = -1.f;
  thread_local uint32_t last_t = 0;
  if (d.p_keep >= 1.0f) {
    d.keep_below = 0xFFFFFFFFu;
  } else {
    if (d.p_keep != last_p) {
      last_t = keep_threshold(d.p_keep);
      last_p = d.p_keep;
    }
    d.keep_below = last_t;
  }
  return true;
}

__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
    if (r < 9) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
  }
  return c;
}

__device__ __forceinline__ bool keep_from_u(uint32_t u, float p_keep) {
  // the product is exact (a power-of-two scale), so a contracted multiply-add rounds the same
  const float f = __fadd_rn(__fmul_rn(__uint2float_rn(u), 2.3283064365386963e-10f),
                            1.1641532182693481e-10f);
  return f < p_keep;
}

// Keep bits of the 4 consecutive elements e0 .. e0+3 (e0 % 4 == 0) of one dropout call: they
// share thread and counter when VEC is 4; for VEC 8 as well (the 4-group lies inside one VEC).
// Bit j of the result is element e0 + j.
__device__ __forceinline__ uint32_t keep4(int64_t e0, int64_t ctr, const DropoutArgs& d) {
  if (d.p_keep >= 1.0f) return 0xFu;  // no dropout: the LoRA input is used as is
  const uint32_t e = (uint32_t)e0;
  const uint32_t g = d.vec == 4 ? (e >> 2) : (e >> 3);       // e / VEC
  const uint32_t it = fdiv(g, d.div_threads);                 // g / threads
  const uint32_t thread = g - it * (uint32_t)d.threads;       // g % threads
  const uint64_t c = (uint64_t)ctr + (uint64_t)it * (uint32_t)(d.vec >> 2) +
                     (((e & (uint32_t)(d.vec - 1))) >> 2);    // + (e % VEC) / 4
  const uint4 r = philox4x32_10(make_uint4((uint32_t)c, (uint32_t)(c >> 32), thread, 0u),
                                (uint32_t)(uint64_t)d.seed, (uint32_t)((uint64_t)d.seed >> 32));
  const uint32_t t = d.keep_below;  // == keep_from_u(u, p_keep) for every u (prepare_dropout)
  return (r.x < t ? 1u : 0u) | (r.y < t ? 2u : 0u) | (r.z < t ? 4u : 0u) | (r.w < t ? 8u : 0u);
}

}  // namespace ql
