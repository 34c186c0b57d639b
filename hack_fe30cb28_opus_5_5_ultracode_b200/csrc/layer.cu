// Host-side orchestration of one decoder layer (forward and backward) in C++: the launch sequence
// of the reference's _layer_forward / _Layer.backward (solution/engine.py:1054-1340) over this
// library's kernels, on one stream, temporaries carved out of a caller-owned workspace. One call
// per layer pass replaces ~20 Python-level launches.
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "ops.h"

namespace ql {
namespace {

struct Bump {
  uint8_t* base;
  int64_t cap, off;
  void* take(int64_t bytes) {
    off = (off + 255) & ~int64_t(255);
    void* p = base != nullptr ? base + off : nullptr;
    off += bytes;
    return p;
  }
  bool ok() const { return base == nullptr || off <= cap; }
};

int64_t esz(int dtype) { return dtype == QL_F32 ? 4 : 2; }

int64_t max_weight_elems(const ql_layer_desc& L) {
  const int64_t C = (int64_t)(L.HQ + 2 * L.HKV) * L.D;
  int64_t m = C * L.H;
  m = m > (int64_t)L.H * L.HQ * L.D ? m : (int64_t)L.H * L.HQ * L.D;
  m = m > 2LL * L.I * L.H ? m : 2LL * L.I * L.H;
  return m;
}

// Offsets (elements) of the four dequantised groups [qkv | o | gate_up | down] in the forward's
// kept weights (ql_layer_saved.w16).
struct WeightSlots {
  int64_t qkv, o, gu, down, total;
};
WeightSlots weight_slots(const ql_layer_desc& L) {
  const int64_t C = (int64_t)(L.HQ + 2 * L.HKV) * L.D, QD = (int64_t)L.HQ * L.D;
  WeightSlots w;
  w.qkv = 0;
  w.o = w.qkv + C * L.H;
  w.gu = w.o + (int64_t)L.H * QD;
  w.down = w.gu + 2LL * L.I * L.H;
  w.total = w.down + (int64_t)L.H * L.I;
  return w;
}

int dequant(const ql_nf4_weight& w, void* out, int dtype, int transpose, cudaStream_t s) {
  return nf4_dequant(w.packed, w.absmax, w.code2, w.absmax2, w.offsets, w.code, out, w.rows,
                     w.cols, w.nested, w.bs2, w.seg1, w.seg2, dtype, transpose, s);
}

#define QL_TRY(x)                  \
  do {                             \
    const int _rc = (x);           \
    if (_rc != QL_STATUS_OK) return _rc; \
  } while (0)

// Per-shape memo of a pure function of a few ints (the host-side planning below runs for every
// layer of every pass; its result depends on the shapes only).
struct ShapeKey {
  int64_t v[6];
  bool operator==(const ShapeKey& o) const {
    for (int i = 0; i < 6; ++i)
      if (v[i] != o.v[i]) return false;
    return true;
  }
};
struct ShapeKeyHash {
  size_t operator()(const ShapeKey& k) const {
    uint64_t h = 0x9E3779B97F4A7C15ull;
    for (int64_t x : k.v) h = (h ^ (uint64_t)x) * 0x100000001B3ull;
    return (size_t)h;
  }
};
template <typename F>
int64_t memo(const ShapeKey& key, F compute) {
  thread_local std::unordered_map<ShapeKey, int64_t, ShapeKeyHash> cache;
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  if (cache.size() > 1024) cache.clear();
  const int64_t v = compute();
  cache.emplace(key, v);
  return v;
}

int64_t layer_gemm_ws_uncached(const ql_layer_desc& L);

// The split-K GEMM workspace sits at the start of the layer workspace (its first bytes are
// tile counters, zero between launches): the largest any GEMM of the layer asks for.
int64_t layer_gemm_ws(const ql_layer_desc& L) {
  return memo(ShapeKey{{L.n, L.H, L.HQ, L.HKV, L.D, L.I}}, [&] { return layer_gemm_ws_uncached(L); });
}

int64_t layer_gemm_ws_uncached(const ql_layer_desc& L) {
  const int64_t C = (int64_t)(L.HQ + 2 * L.HKV) * L.D;
  const int n = L.n, H = L.H, I = L.I, QD = L.HQ * L.D;
  const int64_t shapes[8][3] = {{n, C, H}, {n, H, QD}, {n, 2 * I, H}, {n, H, I},
                                {n, I, H}, {n, H, 2 * I}, {n, QD, H}, {n, H, C}};
  int64_t m = 0;
  for (const auto& sh : shapes) {
    const int64_t b = gemm_workspace_bytes((int)sh[0], (int)sh[1], (int)sh[2]);
    m = b > m ? b : m;
  }
  return m;
}

// The LoRA-gradient kernel's workspace follows at the same offset in both carves (its counters,
// zero between launches, must not be overwritten by the forward's temporaries).
int64_t layer_lora_ws(const ql_layer_desc& L) {
  return memo(ShapeKey{{L.n, L.H, L.HQ, L.HKV, L.D, -1}}, [&] {
    const int32_t nc[4] = {L.HQ * L.D, L.HKV * L.D, L.H, L.H};
    return lora_grads_workspace(L.n, nc, 4);
  });
}

struct FwdWs {
  void* gws;  // split-K GEMM workspace
  int64_t gws_bytes;
  void* lgw;  // LoRA-gradient workspace (unused by the forward, reserved)
  int64_t lgw_bytes;
  void* w;    // dequantised weight (largest of the four)
  void* a;    // [n, H] norm output (a, then b)
  void* qkv;  // [n, C]
  void* m;    // [n, I]
  void* o16;  // [n, H] the o projection, 16-bit (added to the residual by the second norm)
  void* d16[2];  // [n, H] down projections handed from layer to layer (layers_forward)
};

FwdWs carve_fwd(const ql_layer_desc& L, Bump& b) {
  const int64_t n = L.n, C = (int64_t)(L.HQ + 2 * L.HKV) * L.D, e = esz(L.dtype);
  FwdWs w;
  w.gws_bytes = layer_gemm_ws(L);
  w.gws = b.take(w.gws_bytes);
  w.lgw_bytes = layer_lora_ws(L);
  w.lgw = b.take(w.lgw_bytes);
  w.w = b.take(max_weight_elems(L) * e);
  w.a = b.take(n * L.H * e);
  w.qkv = b.take(n * C * e);
  w.m = b.take(n * L.I * e);
  w.o16 = b.take(n * L.H * e);
  w.d16[0] = b.take(n * L.H * e);
  w.d16[1] = b.take(n * L.H * e);
  return w;
}

struct BwdWs {
  void* gws;
  int64_t gws_bytes;
  void* lgw;
  int64_t lgw_bytes;
  void* w;
  void* dm;      // [n, I]
  void* db;      // [n, H]
  float* dh2;    // [n, H]
  void* dh2_16;  // [n, H]
  void* dout;    // [n, HQ D]
  float* dq;     // [n, HQ D]
  float* dk;     // [n, HKV D]
  float* dv;
  float* dvec;   // [HQ, n]
  void* dqkv;    // [n, C]
  float* dxq;    // [n, rank]
  float* dxv;
  void* da;      // [n, H]
  float* attn_part;  // the deterministic attention backward's partials, or null
};

BwdWs carve_bwd(const ql_layer_desc& L, Bump& b) {
  const int64_t n = L.n, C = (int64_t)(L.HQ + 2 * L.HKV) * L.D, e = esz(L.dtype);
  BwdWs w;
  w.gws_bytes = layer_gemm_ws(L);
  w.gws = b.take(w.gws_bytes);
  w.lgw_bytes = layer_lora_ws(L);
  w.lgw = b.take(w.lgw_bytes);
  w.w = b.take(max_weight_elems(L) * e);
  w.dm = b.take(n * L.I * e);
  w.db = b.take(n * L.H * e);
  w.dh2 = (float*)b.take(n * L.H * 4);
  w.dh2_16 = b.take(n * L.H * e);
  w.dout = b.take(n * L.HQ * L.D * e);
  w.dq = (float*)b.take(n * L.HQ * L.D * 4);
  w.dk = (float*)b.take(n * L.HKV * L.D * 4);
  w.dv = (float*)b.take(n * L.HKV * L.D * 4);
  w.dvec = (float*)b.take((int64_t)L.HQ * n * 4);
  w.dqkv = b.take(n * C * e);
  w.dxq = (float*)b.take(n * L.rank * 4);
  w.dxv = (float*)b.take(n * L.rank * 4);
  w.da = b.take(n * L.H * e);
  w.attn_part = nullptr;
  if (attn_deterministic() && L.D == 128) {
    const int64_t floats = ql_attn_bwd_partials_floats(L.n, L.max_len, L.HQ, L.HKV);
    if (floats > 0) w.attn_part = (float*)b.take(floats * 4);
  }
  return w;
}

void fill_drop(const ql_layer_desc& L, int64_t& seed, int64_t& cq, int64_t& cv, int64_t& thr,
               float& pk, float& ks, int32_t& vec, int32_t& dq, int32_t& dv) {
  seed = L.seed; cq = L.ctr_q; cv = L.ctr_v; thr = L.threads;
  pk = L.p_keep; ks = L.keep_scale; vec = L.vec; dq = L.drop_q; dv = L.drop_v;
}

int check(const ql_layer_desc& L) {
  if (L.n < 0 || L.H <= 0 || L.HQ <= 0 || L.HKV <= 0 || L.D <= 0 || L.I <= 0) return QL_STATUS_BAD_ARG;
  if (L.rank != 16) return QL_STATUS_UNSUPPORTED;
  if (L.dtype != QL_F16 && L.dtype != QL_BF16) return QL_STATUS_BAD_ARG;
  return QL_STATUS_OK;
}

// One side stream (and its fork / join events) per device for work of a layer pass that can run
// next to the main stream; created on first use.
struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};

SideStream& side_stream() {
  static std::mutex mu;
  static SideStream per_dev[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    static SideStream none;
    return none;
  }
  SideStream& ss = per_dev[dev];
  std::lock_guard<std::mutex> lock(mu);
  if (ss.s == nullptr) {
    cudaStream_t st = nullptr;
    cudaEvent_t a = nullptr, b = nullptr;
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) == cudaSuccess &&
        cudaEventCreateWithFlags(&a, cudaEventDisableTiming) == cudaSuccess &&
        cudaEventCreateWithFlags(&b, cudaEventDisableTiming) == cudaSuccess) {
      ss.fork = a;
      ss.join = b;
      ss.s = st;
    } else {
      cudaGetLastError();  // no side stream: the work runs on the main stream
    }
  }
  return ss;
}

int layer_backward_input(const ql_layer_desc& L, const ql_layer_saved& S, const BwdWs& w,
                         int64_t C, int dt, float* dh_out, void* dh16_out, int* err,
                         cudaStream_t s);

}  // namespace

int64_t layer_weight_elems(const ql_layer_desc& L) { return weight_slots(L).total; }

int64_t layer_workspace_bytes(const ql_layer_desc& L, int backward) {
  Bump b{nullptr, 0, 0};
  if (backward) carve_bwd(L, b); else carve_fwd(L, b);
  return b.off + 256;
}

// The residual stream goes through the norms: the o and down projections are written in the
// 16-bit type, and the RMSNorm that follows each adds it to the fp32 residual (h2 = h + o in the
// post-attention norm, the next layer's h = h2 + d in its input norm), writing the sum as its
// xsum - the same fp32 additions of the rounded projections as an add in the GEMM epilogue,
// done by a streaming kernel instead of a per-row epilogue behind the GEMM's last tile.
// x_base / d_in: this layer's input is x_base + d_in (the previous layer's h2 and down output),
// written to S.h by the input norm; both null: S.h is the input as it stands. d_out: the down
// projection goes there (16-bit) for the next layer; null: h_out = h2 + d (fp32) here.
int layer_forward(const ql_layer_desc& L, const ql_layer_saved& S, float* h_out, void* ws,
                  int64_t ws_bytes, int* err, cudaStream_t s, const float* x_base,
                  const void* d_in, void* d_out) {
  QL_TRY(check(L));
  if (L.n == 0) return QL_STATUS_OK;
  Bump bump{(uint8_t*)ws, ws_bytes, 0};
  const FwdWs w = carve_fwd(L, bump);
  if (!bump.ok()) return QL_STATUS_BAD_ARG;
  const int64_t n = L.n, C = (int64_t)(L.HQ + 2 * L.HKV) * L.D;
  const int dt = L.dtype;
  // each weight group dequantised once per step: into the kept copy when the caller gives one
  // (the backward then reads it), else into the workspace
  const WeightSlots slots = weight_slots(L);
  auto wbuf = [&](int64_t off) -> void* {
    return S.w16 != nullptr ? static_cast<uint8_t*>(S.w16) + off * esz(dt) : w.w;
  };
  void* const wqkv = wbuf(slots.qkv);
  void* const wo = wbuf(slots.o);
  void* const wgu = wbuf(slots.gu);
  void* const wdown = wbuf(slots.down);

  // input RMSNorm + the dropped LoRA inputs + LoRA-A products
  if ((d_in != nullptr) != (x_base != nullptr)) return QL_STATUS_BAD_ARG;
  RmsFwdC r1{};
  r1.x = d_in != nullptr ? x_base : S.h; r1.w = L.ln1; r1.y = w.a; r1.yq = S.yq; r1.yv = S.yv;
  r1.rstd = S.rstd1;
  if (d_in != nullptr) {  // the layer input h = h2 + d of the previous layer, kept as S.h
    r1.delta = d_in;
    r1.xsum = const_cast<float*>(S.h);
  }
  r1.Aq = L.Aq; r1.Av = L.Av; r1.xq = S.xq; r1.xv = S.xv; r1.keep_q = S.keep_q;
  r1.keep_v = S.keep_v;
  r1.n = L.n; r1.H = L.H; r1.rank = L.rank; r1.dtype = dt; r1.eps = L.eps; r1.tok = L.tok;
  fill_drop(L, r1.seed, r1.ctr_q, r1.ctr_v, r1.threads, r1.p_keep, r1.keep_scale, r1.vec,
            r1.drop_q, r1.drop_v);
  QL_TRY(rms_fwd(r1, s));
  // q, k, v in one GEMM (bias in the epilogue), then LoRA-B + RoPE
  const bool ready = S.w16 != nullptr && S.w16_ready;  // dequantised by the caller this step
  if (!ready) QL_TRY(dequant(L.qkv, wqkv, dt, 0, s));
  QL_TRY(gemm_tn(w.a, L.H, wqkv, L.H, w.qkv, C, L.bias_qkv, L.n, (int)C, L.H, dt, dt, 0, nullptr,
                 err, s, w.gws, w.gws_bytes));
  RopeFwdC rf{};
  rf.qkv = w.qkv; rf.xq = S.xq; rf.xv = S.xv; rf.Bq = L.Bq; rf.Bv = L.Bv; rf.cos = L.cos;
  rf.sin = L.sin; rf.pos = L.pos; rf.q = S.q; rf.k = S.k; rf.v = S.v;
  rf.lora_scale = L.lora_scale; rf.n = L.n; rf.HQ = L.HQ; rf.HKV = L.HKV; rf.D = L.D;
  rf.rank = L.rank; rf.dtype = dt;
  QL_TRY(rope_fwd(rf, s));
  AttnFwdC af{};
  af.q = S.q; af.k = S.k; af.v = S.v; af.cu_seqlens = L.cu_seqlens; af.out = S.out; af.lse = S.lse;
  af.scale = L.scale; af.n = L.n; af.B = L.B; af.max_len = L.max_len; af.HQ = L.HQ;
  af.HKV = L.HKV; af.D = L.D; af.dtype = dt;
  QL_TRY(attn_fwd(af, s));
  // o projection (16-bit), then the post-attention RMSNorm of h2 = h + o (kept as S.h2)
  if (!ready) QL_TRY(dequant(L.o, wo, dt, 0, s));
  QL_TRY(gemm_tn(S.out, (int64_t)L.HQ * L.D, wo, (int64_t)L.HQ * L.D, w.o16, L.H, nullptr, L.n,
                 L.H, L.HQ * L.D, dt, dt, 0, nullptr, err, s, w.gws, w.gws_bytes));
  RmsFwdC r2{};
  r2.x = S.h; r2.delta = w.o16; r2.xsum = S.h2;
  r2.w = L.ln2; r2.y = w.a; r2.rstd = S.rstd2; r2.n = L.n; r2.H = L.H;
  r2.rank = L.rank; r2.dtype = dt; r2.eps = L.eps; r2.vec = 4; r2.threads = 1; r2.p_keep = 1.f;
  r2.keep_scale = 1.f;
  QL_TRY(rms_fwd(r2, s));
  // [gate | up], SwiGLU, down with the residual add: h3 = h2 + d
  if (!ready) QL_TRY(dequant(L.gu, wgu, dt, 0, s));
  QL_TRY(gemm_tn(w.a, L.H, wgu, L.H, S.gu, 2LL * L.I, nullptr, L.n, 2 * L.I, L.H, dt, dt, 0,
                 nullptr, err, s, w.gws, w.gws_bytes));
  QL_TRY(glu_fwd(S.gu, w.m, n, L.I, dt, s));
  if (!ready) QL_TRY(dequant(L.down, wdown, dt, 0, s));
  if (d_out != nullptr)  // the next layer's input norm adds it to h2
    QL_TRY(gemm_tn(w.m, L.I, wdown, L.I, d_out, L.H, nullptr, L.n, L.H, L.I, dt, dt, 0, nullptr,
                   err, s, w.gws, w.gws_bytes));
  else
    QL_TRY(gemm_tn(w.m, L.I, wdown, L.I, h_out, L.H, nullptr, L.n, L.H, L.I, dt, QL_F32, 0,
                   S.h2, err, s, w.gws, w.gws_bytes));
  return QL_STATUS_OK;
}

// Every layer's forward in order (the keep-everything plan): layer i's down projection reaches
// layer i + 1 as a 16-bit delta through two alternating workspace buffers, and only the last
// layer writes its output h_out[count - 1] = h2 + d in fp32 (h_out[i] of the others is where the
// next layer's input norm writes that sum: saved[i + 1].h).
int layers_forward(const ql_layer_desc* descs, const ql_layer_saved* saved, int count,
                   float* const* h_out, void* ws, int64_t ws_bytes, int* err, cudaStream_t s) {
  for (int i = 0; i < count; ++i) {
    QL_TRY(check(descs[i]));
    if (i + 1 < count && h_out[i] != saved[i + 1].h) return QL_STATUS_BAD_ARG;
  }
  if (count == 0 || descs[0].n == 0) return QL_STATUS_OK;
  Bump bump{(uint8_t*)ws, ws_bytes, 0};
  const FwdWs w = carve_fwd(descs[0], bump);
  if (!bump.ok()) return QL_STATUS_BAD_ARG;
  for (int i = 0; i < count; ++i) {
    const bool last = i + 1 == count;
    QL_TRY(layer_forward(descs[i], saved[i], h_out[i], ws, ws_bytes, err, s,
                         i > 0 ? saved[i - 1].h2 : nullptr, i > 0 ? w.d16[(i - 1) & 1] : nullptr,
                         last ? nullptr : w.d16[i & 1]));
  }
  return QL_STATUS_OK;
}

int layer_backward(const ql_layer_desc& L, const ql_layer_saved& S, const float* dh3,
                   const void* dh3_16, float* grads, float* dh_out, void* dh16_out, void* ws,
                   int64_t ws_bytes, int* err, cudaStream_t s) {
  QL_TRY(check(L));
  if (L.n == 0) return QL_STATUS_OK;
  Bump bump{(uint8_t*)ws, ws_bytes, 0};
  const BwdWs w = carve_bwd(L, bump);
  if (!bump.ok()) return QL_STATUS_BAD_ARG;
  const int64_t n = L.n, C = (int64_t)(L.HQ + 2 * L.HKV) * L.D;
  const int dt = L.dtype;
  float* gAq = grads;
  float* gBq = gAq + (int64_t)L.rank * L.H;
  float* gAv = gBq + (int64_t)L.HQ * L.D * L.rank;
  float* gBv = gAv + (int64_t)L.rank * L.H;
  // the data-gradient products read each weight in its forward layout (MN-major operand): the
  // forward's kept copy, or a fresh dequantisation into the workspace
  const WeightSlots slots = weight_slots(L);
  auto weight = [&](const ql_nf4_weight& q, int64_t off, void** out) -> int {
    if (S.w16 != nullptr) {
      *out = static_cast<uint8_t*>(S.w16) + off * esz(dt);
      return QL_STATUS_OK;
    }
    *out = w.w;
    return dequant(q, w.w, dt, 0, s);
  };
  void* W = nullptr;

  // MLP: dm = dh3 . Wd ; [dg | du] in place ; db = [dg | du] . Wgu
  QL_TRY(weight(L.down, slots.down, &W));  // [H, I]
  QL_TRY(gemm_nn(dh3_16, L.H, W, L.I, w.dm, L.I, nullptr, L.n, L.I, L.H, dt, dt, 0, nullptr,
                 err, s, w.gws, w.gws_bytes));
  QL_TRY(glu_bwd(w.dm, S.gu, n, L.I, dt, s));
  QL_TRY(weight(L.gu, slots.gu, &W));  // [2 I, H]
  QL_TRY(gemm_nn(S.gu, 2LL * L.I, W, L.H, w.db, L.H, nullptr, L.n, L.H, 2 * L.I, dt, dt,
                 0, nullptr, err, s, w.gws, w.gws_bytes));
  RmsBwdC r2{};
  r2.dy = w.db; r2.ld_dy = L.H; r2.x = S.h2; r2.rstd = S.rstd2; r2.w = L.ln2; r2.dres = dh3;
  r2.dx = w.dh2; r2.dx16 = w.dh2_16; r2.n = L.n; r2.H = L.H; r2.rank = L.rank; r2.dtype = dt;
  r2.grad_scale = 1.f; r2.vec = 4; r2.threads = 1; r2.p_keep = 1.f; r2.keep_scale = 1.f;
  QL_TRY(rms_bwd(r2, s));
  // attention
  QL_TRY(weight(L.o, slots.o, &W));  // [H, HQ D]
  QL_TRY(gemm_nn(w.dh2_16, L.H, W, (int64_t)L.HQ * L.D, w.dout, (int64_t)L.HQ * L.D, nullptr, L.n,
                 L.HQ * L.D, L.H, dt, dt, 0, nullptr, err, s, w.gws, w.gws_bytes));
  AttnBwdC ab{};
  ab.q = S.q; ab.k = S.k; ab.v = S.v; ab.out = S.out; ab.dout = w.dout; ab.lse = S.lse;
  ab.cu_seqlens = L.cu_seqlens; ab.dvec = w.dvec; ab.dq = w.dq; ab.dk = w.dk; ab.dv = w.dv;
  ab.scale = L.scale; ab.n = L.n; ab.B = L.B; ab.max_len = L.max_len; ab.HQ = L.HQ;
  ab.HKV = L.HKV; ab.D = L.D; ab.dtype = dt; ab.partials = w.attn_part;
  QL_TRY(attn_bwd(ab, s));
  RopeBwdC rb{};
  rb.dq = w.dq; rb.dk = w.dk; rb.dv = w.dv; rb.cos = L.cos; rb.sin = L.sin; rb.pos = L.pos;
  rb.dqkv = w.dqkv; rb.Bq = L.Bq; rb.Bv = L.Bv; rb.dxlo_q = w.dxq; rb.dxlo_v = w.dxv;
  rb.lora_scale = L.lora_scale; rb.n = L.n; rb.HQ = L.HQ; rb.HKV = L.HKV; rb.D = L.D;
  rb.kv_heads_in = L.HKV; rb.rank = L.rank; rb.dtype = dt; rb.grad_dtype = QL_F32;
  QL_TRY(rope_bwd(rb, s));
  // LoRA weight gradients in one launch: dB = s g^T x_lo, dA = dx_lo^T drop(a)
  const int64_t qcols = (int64_t)L.HQ * L.D, vcols = (int64_t)L.HKV * L.D;
  const uint8_t* dqkv = (const uint8_t*)w.dqkv;
  const ql_lora_grad_job jobs[4] = {
      {dqkv, C, S.xq, gBq, (int)qcols, dt, 0, L.lora_scale},
      {dqkv + (qcols + vcols) * esz(dt), C, S.xv, gBv, (int)vcols, dt, 0, L.lora_scale},
      {S.yq, L.H, w.dxq, gAq, L.H, QL_F32, 1, 1.f},
      {S.yv, L.H, w.dxv, gAv, L.H, QL_F32, 1, 1.f}};
  // the LoRA weight gradients need nothing of the data-gradient path below: a side stream runs
  // them next to the qkv data-gradient GEMM and RMSNorm backward, joined before returning
  SideStream& side = side_stream();
  if (side.s != nullptr) {
    if (cudaEventRecord(side.fork, s) != cudaSuccess || cudaStreamWaitEvent(side.s, side.fork, 0) != cudaSuccess)
      return QL_STATUS_CUDA;
    QL_TRY(lora_grads(jobs, 4, n, dt, w.lgw, w.lgw_bytes, side.s));
    if (cudaEventRecord(side.join, side.s) != cudaSuccess) return QL_STATUS_CUDA;
  } else {
    QL_TRY(lora_grads(jobs, 4, n, dt, w.lgw, w.lgw_bytes, s));
  }
  const int rc = layer_backward_input(L, S, w, C, dt, dh_out, dh16_out, err, s);
  if (side.s != nullptr && cudaStreamWaitEvent(s, side.join, 0) != cudaSuccess) return QL_STATUS_CUDA;
  return rc;
}

namespace {
// The gradient of the layer's input (none for the first layer: its input is the frozen
// embedding): da = dqkv . Wqkv, then the input RMSNorm's backward.
int layer_backward_input(const ql_layer_desc& L, const ql_layer_saved& S, const BwdWs& w,
                         int64_t C, int dt, float* dh_out, void* dh16_out, int* err,
                         cudaStream_t s) {
  if (dh_out == nullptr) return QL_STATUS_OK;
  const WeightSlots slots = weight_slots(L);
  void* W = nullptr;
  if (S.w16 != nullptr) {
    W = static_cast<uint8_t*>(S.w16) + slots.qkv * esz(dt);
  } else {
    W = w.w;
    QL_TRY(dequant(L.qkv, w.w, dt, 0, s));
  }
  QL_TRY(gemm_nn(w.dqkv, C, W, L.H, w.da, L.H, nullptr, L.n, L.H, (int)C, dt, dt, 0, nullptr,
                 err, s, w.gws, w.gws_bytes));  // [C, H] weight
  RmsBwdC r1{};
  r1.dy = w.da; r1.ld_dy = L.H; r1.x = S.h; r1.rstd = S.rstd1; r1.w = L.ln1; r1.dres = w.dh2;
  r1.dx = dh_out; r1.dx16 = dh16_out; r1.dxlo_q = w.dxq; r1.dxlo_v = w.dxv; r1.Aq = L.Aq;
  r1.Av = L.Av; r1.n = L.n; r1.H = L.H; r1.rank = L.rank; r1.dtype = dt; r1.grad_scale = 1.f;
  r1.tok = L.tok; r1.keep_q = S.keep_q; r1.keep_v = S.keep_v;
  fill_drop(L, r1.seed, r1.ctr_q, r1.ctr_v, r1.threads, r1.p_keep, r1.keep_scale, r1.vec,
            r1.drop_q, r1.drop_v);
  QL_TRY(rms_bwd(r1, s));
  return QL_STATUS_OK;
}
}  // namespace

}  // namespace ql
