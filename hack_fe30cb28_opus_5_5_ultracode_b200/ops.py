"""torch-facing wrappers of the C ABI: each takes CUDA tensors, checks layouts, and launches on
the current stream. Names follow the reference's launch wrappers (solution/engine.py:103-109,
947-1045) so the tests read like the reference's own.
"""

import torch

from . import _lib
from ._lib import call

_DT = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}
INT_MAX = 2147483647
STATUS_UNSUPPORTED = 3  # QL_STATUS_UNSUPPORTED of include/qlora_sm100.h: no kernel for this request
STATUS_TIMEOUT = 4  # QL_STATUS_TIMEOUT of include/qlora_sm100.h: a kernel gave up a bounded wait


def dtype_code(dtype):
    try:
        return _DT[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}") from None


def stream_ptr():
    """The current CUDA stream of the current device, as a raw pointer (called for every
    launch: the raw lookup skips torch.cuda.current_stream()'s Python-level device resolution)."""
    try:
        return torch._C._cuda_getCurrentRawStream(torch._C._cuda_getDevice())
    except AttributeError:  # pragma: no cover - other torch builds
        return torch.cuda.current_stream().cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("CUDA tensors required (the library has no CPU path)")


# ---------------------------------------------------------------------------------------------
# NF4
# ---------------------------------------------------------------------------------------------
def nf4_dequant(w, out=None, transpose=False, dtype=torch.float16):
    """Dequantize an NF4 weight (an object with packed, absmax, code, nested, code2, absmax2,
    offsets, bs2, seg1, seg2, shape = (rows, cols)) into out [rows, cols] (or its transpose)."""
    rows, cols = w.shape
    if out is None:
        out = torch.empty((cols, rows) if transpose else (rows, cols), device=w.packed.device,
                          dtype=dtype)
    _need_cuda(w.packed, out)
    assert out.is_contiguous()
    call("ql_nf4_dequant", _ptr(w.packed), _ptr(w.absmax), _ptr(w.code2), _ptr(w.absmax2),
         _ptr(w.offsets), _ptr(w.code), _ptr(out), rows, cols, int(w.nested), int(w.bs2),
         int(getattr(w, "seg1", INT_MAX)), int(getattr(w, "seg2", INT_MAX)),
         dtype_code(out.dtype), int(transpose), stream_ptr())
    return out


def nf4_weight_struct(w):
    """The ql_nf4_weight view of an NF4 weight object (as ops.nf4_dequant reads it)."""
    rows, cols = w.shape
    return _lib.struct("ql_nf4_weight", packed=_ptr(w.packed), absmax=_ptr(w.absmax),
                       code=_ptr(w.code), code2=_ptr(w.code2), absmax2=_ptr(w.absmax2),
                       offsets=_ptr(w.offsets), rows=rows, cols=cols,
                       seg1=int(getattr(w, "seg1", INT_MAX)), seg2=int(getattr(w, "seg2", INT_MAX)),
                       nested=int(w.nested), bs2=int(w.bs2))


def gemm_nf4(a, w, layout=0, out=None, bias=None, accumulate=False, out_dtype=None,
             residual=None):
    """out = a @ W^T (layout 0, W [N, K]) or a @ W (layout 1, W [K, N]) with the NF4 weight w
    dequantised inside the kernel (ql_gemm_nf4)."""
    M, K = a.shape
    rows, cols = w.shape
    N = rows if layout == 0 else cols
    if (cols if layout == 0 else rows) != K:
        raise ValueError(f"inner dimensions differ: {a.shape} x NF4 {w.shape} (layout {layout})")
    if out is None:
        out = torch.empty((M, N), device=a.device, dtype=out_dtype or a.dtype)
    ws = nf4_weight_struct(w)
    call("ql_gemm_nf4", _ptr(a), a.stride(0), ctypes_ref(ws), int(layout), _ptr(out),
         out.stride(0), _ptr(bias), M, dtype_code(a.dtype), dtype_code(out.dtype),
         int(accumulate), _ptr(residual), stream_ptr())
    return out


# ---------------------------------------------------------------------------------------------
# GEMM
# ---------------------------------------------------------------------------------------------
def gemm(a, b, out=None, bias=None, accumulate=False, out_dtype=None, residual=None,
         b_kn=False):
    """out[M, N] (+)= a[M, K] @ b[N, K]^T (+ bias) on tcgen05; with b_kn, b is [K, N] and
    out = a @ b (ql_gemm_nn). a and b: fp16 or bf16 with unit column stride; out: fp16 / bf16 /
    fp32 with unit column stride."""
    M, K = a.shape
    N, K2 = (b.shape[1], b.shape[0]) if b_kn else b.shape
    if K != K2:
        raise ValueError(f"inner dimensions differ: {a.shape} x {b.shape}")
    if a.dtype != b.dtype:
        raise ValueError("a and b must have the same dtype")
    if out is None:
        out = torch.empty((M, N), device=a.device, dtype=out_dtype or a.dtype)
    _need_cuda(a, b, out, bias)
    if a.stride(1) != 1 or b.stride(1) != 1 or out.stride(1) != 1:
        raise ValueError("gemm needs unit column strides")
    if bias is not None and bias.dtype != a.dtype:
        raise ValueError("bias must have the input dtype")
    if residual is not None and (residual.stride(0) != out.stride(0) or residual.stride(1) != 1):
        raise ValueError("residual must share the output's row stride")
    ws = gemm_workspace(a.device, int(_lib.lib().ql_gemm_workspace_bytes(M, N, K)))
    call("ql_gemm_nn" if b_kn else "ql_gemm_tn", _ptr(a), a.stride(0), _ptr(b), b.stride(0),
         _ptr(out), out.stride(0), _ptr(bias), M, N, K, dtype_code(a.dtype),
         dtype_code(out.dtype), int(accumulate), _ptr(residual), _ptr(ws),
         0 if ws is None else ws.numel(), stream_ptr())
    return out


def gemm_set_mode(mode):
    """Tile kind of the GEMMs (mode & 3): 0 per-shape cost model, 1 single-CTA tiles, 2 2-SM
    pair tiles; + 4: one 64-wide K chunk per pipeline stage (2-D copies) instead of two."""
    call("ql_gemm_set_mode", int(mode))


def attn_set_deterministic(on):
    """The layer backward's attention gradients summed in a fixed order (bit-reproducible run to
    run) or by fp32 bulk reductions (default; ql_attn_set_deterministic)."""
    call("ql_attn_set_deterministic", 1 if on else 0)


def attn_set_impl(impl):
    """Attention kernels for D = 128: 0 default (tcgen05), 1 warp-level mma.sync, 2 tcgen05."""
    call("ql_attn_set_impl", int(impl))


_GEMM_WS = {}


def gemm_workspace(device, nbytes):
    """A zero-initialised, grow-only split-K workspace per device (its counter region is left
    zero by every GEMM, so it is reused as is)."""
    if nbytes <= 0:
        return None
    ws = _GEMM_WS.get(device)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(nbytes, device=device, dtype=torch.uint8)
        _GEMM_WS[device] = ws
    return ws


PROFILE_KINDS = ("gemm", "dequant", "rms_fwd", "rms_bwd", "rope_fwd", "rope_bwd", "attn_fwd",
                 "attn_bwd", "glu_fwd", "glu_bwd", "lora_colsum", "ce", "other")


def profile_start(capacity=200000):
    """Time every library operation with CUDA events (see ql_profile_start)."""
    call("ql_profile_start", int(capacity))


def profile_stop():
    call("ql_profile_stop")


def profile_read():
    """{kind: {"count", "ms", "flops", "bytes"}} of the operations recorded since profile_start."""
    import ctypes

    n = len(PROFILE_KINDS)
    arrs = [(ctypes.c_double * n)() for _ in range(4)]
    call("ql_profile_read", *[ctypes.addressof(a) for a in arrs])
    return {k: {"count": arrs[0][i], "ms": arrs[1][i], "flops": arrs[2][i], "bytes": arrs[3][i]}
            for i, k in enumerate(PROFILE_KINDS) if arrs[0][i]}


def set_pdl(on):
    """Programmatic dependent launch on (default) or off for this library's launches
    (ql_set_pdl)."""
    call("ql_set_pdl", 1 if on else 0)


def launch_count():
    """Kernels launched through the library so far (its own counter)."""
    return int(_lib.lib().ql_launch_count())


def device_status(clear=True):
    """The library's device status word (QL_STATUS_TIMEOUT if a kernel gave up a wait)."""
    import ctypes

    v = ctypes.c_int(0)
    call("ql_device_status", ctypes.addressof(v), int(clear))
    return v.value


# ---------------------------------------------------------------------------------------------
# dropout / RMSNorm
# ---------------------------------------------------------------------------------------------
class Drop:
    """The LoRA dropout state of one layer's two masks (TorchDropout.draw, engine.py:787-797):
    tok = packed tokens' indices in the padded batch, seed, Philox counters of the q and v
    calls, the dropout kernel's threads, p, VEC."""

    def __init__(self, tok, seed, ctr_q, ctr_v, threads, p, vec=4, drop_q=True, drop_v=True):
        self.tok, self.seed, self.ctr_q, self.ctr_v = tok, int(seed), int(ctr_q), int(ctr_v)
        self.threads, self.p, self.vec = int(threads), float(p), int(vec)
        self.drop_q, self.drop_v = bool(drop_q), bool(drop_v)

    def fields(self):
        return dict(tok=_ptr(self.tok), seed=self.seed, ctr_q=self.ctr_q, ctr_v=self.ctr_v,
                    threads=self.threads, p_keep=1.0 - self.p, keep_scale=1.0 / (1.0 - self.p),
                    vec=self.vec, drop_q=int(self.drop_q), drop_v=int(self.drop_v))


def dropout_keep(nelem, seed, ctr, threads, p, vec=4, device="cuda"):
    out = torch.empty(nelem, device=device, dtype=torch.int8)
    call("ql_dropout_keep", _ptr(out), nelem, int(seed), int(ctr), int(threads), 1.0 - p,
         int(vec), stream_ptr())
    return out


def rms_fwd(x, w, eps, dtype=torch.float16, delta=None, write_y=True, drop=None, Aq=None,
            Av=None, want_yq=False, out_y=None, out_xsum=None, keep_bits=None):
    """(xsum, y, yq, yv, rstd, xq, xv) of reference _rms_fwd (engine.py:947-966), with the
    LoRA-A products xq / xv when Aq / Av are given. keep_bits: (keep_q, keep_v) int32
    [n, H / 32] tensors (or None) that receive the dropout masks as bits."""
    n, H = x.shape
    dev = x.device
    xsum = (out_xsum if out_xsum is not None else torch.empty_like(x)) if delta is not None else x
    y = (out_y if out_y is not None else torch.empty((n, H), device=dev, dtype=dtype)) \
        if write_y else None
    dq = drop is not None and drop.drop_q
    dv = drop is not None and drop.drop_v
    yq = torch.empty((n, H), device=dev, dtype=dtype) if dq and want_yq else None
    yv = torch.empty((n, H), device=dev, dtype=dtype) if dv and want_yq else None
    xq = torch.empty((n, 16), device=dev, dtype=dtype) if dq and Aq is not None else None
    xv = torch.empty((n, 16), device=dev, dtype=dtype) if dv and Av is not None else None
    rstd = torch.empty((n,), device=dev, dtype=torch.float32)
    fields = dict(x=_ptr(x), delta=_ptr(delta), w=_ptr(w), xsum=_ptr(xsum) if delta is not None
                  else None, y=_ptr(y), yq=_ptr(yq), yv=_ptr(yv), rstd=_ptr(rstd),
                  Aq=_ptr(Aq) if dq else None, Av=_ptr(Av) if dv else None, xq=_ptr(xq),
                  xv=_ptr(xv), n=n, H=H, rank=16, dtype=dtype_code(dtype), eps=float(eps),
                  vec=4)
    if keep_bits is not None:
        fields.update(keep_q=_ptr(keep_bits[0]), keep_v=_ptr(keep_bits[1]))
    if drop is not None:
        fields.update(drop.fields())
    args = _lib.struct("ql_rms_fwd_args", **fields)
    call("ql_rms_fwd", ctypes_ref(args), stream_ptr())
    return xsum, y, yq, yv, rstd, xq, xv


def rms_bwd(dy, x, rstd, w, dtype=torch.float16, dres=None, tq=None, tv=None, dxlo_q=None,
            dxlo_v=None, Aq=None, Av=None, drop=None, grad_scale=1.0, out=None, out16=None,
            keep_bits=None):
    """Reference _rms_bwd (engine.py:969-981); dx fp32 (and its 16-bit copy into out16).
    keep_bits: the forward's (keep_q, keep_v) mask bits, read instead of redrawing the masks."""
    n, H = x.shape
    dx = out if out is not None else torch.empty_like(x)
    fields = dict(dy=_ptr(dy), ld_dy=dy.stride(0), x=_ptr(x), rstd=_ptr(rstd), w=_ptr(w),
                  dres=_ptr(dres), dx=_ptr(dx), dx16=_ptr(out16), tq=_ptr(tq), tv=_ptr(tv),
                  dxlo_q=_ptr(dxlo_q), dxlo_v=_ptr(dxlo_v), Aq=_ptr(Aq), Av=_ptr(Av), n=n, H=H,
                  rank=16, dtype=dtype_code(dtype), grad_scale=float(grad_scale), vec=4)
    if keep_bits is not None:
        fields.update(keep_q=_ptr(keep_bits[0]), keep_v=_ptr(keep_bits[1]))
    if drop is not None:
        fields.update(drop.fields())
    args = _lib.struct("ql_rms_bwd_args", **fields)
    call("ql_rms_bwd", ctypes_ref(args), stream_ptr())
    return dx


def ctypes_ref(s):
    import ctypes

    return ctypes.addressof(s)


# ---------------------------------------------------------------------------------------------
# qkv + RoPE
# ---------------------------------------------------------------------------------------------
def rope_fwd(qkv, cos, sin, pos, HQ, HKV, D, lora_scale, lq=None, lv=None, xq=None, xv=None,
             Bq=None, Bv=None, out=None):
    n = qkv.shape[0]
    dev, dt = qkv.device, qkv.dtype
    if out is None:
        q = torch.empty((n, HQ, D), device=dev, dtype=dt)
        k = torch.empty((n, HKV, D), device=dev, dtype=dt)
        v = torch.empty((n, HKV, D), device=dev, dtype=dt)
    else:
        q, k, v = out
    args = _lib.struct("ql_rope_fwd_args", qkv=_ptr(qkv), lq=_ptr(lq), lv=_ptr(lv), xq=_ptr(xq),
                       xv=_ptr(xv), Bq=_ptr(Bq), Bv=_ptr(Bv), cos=_ptr(cos), sin=_ptr(sin),
                       pos=_ptr(pos), q=_ptr(q), k=_ptr(k), v=_ptr(v),
                       lora_scale=float(lora_scale), n=n, HQ=HQ, HKV=HKV, D=D, rank=16,
                       dtype=dtype_code(dt))
    call("ql_rope_fwd", ctypes_ref(args), stream_ptr())
    return q, k, v


def rope_bwd(dq, dk, dv, cos, sin, pos, HQ, HKV, D, dtype=torch.float16, Bq=None, Bv=None,
             lora_scale=1.0, out=None):
    """(dqkv, dxlo_q, dxlo_v): the pre-rotary qkv gradient and, with Bq / Bv, the LoRA-A
    output gradients s * (g . B) (fp32)."""
    n = dq.shape[0]
    dev = dq.device
    C = (HQ + 2 * HKV) * D
    dqkv = out if out is not None else torch.empty((n, C), device=dev, dtype=dtype)
    dxlo_q = torch.empty((n, 16), device=dev, dtype=torch.float32) if Bq is not None else None
    dxlo_v = torch.empty((n, 16), device=dev, dtype=torch.float32) if Bv is not None else None
    args = _lib.struct("ql_rope_bwd_args", dq=_ptr(dq), dk=_ptr(dk), dv=_ptr(dv), cos=_ptr(cos),
                       sin=_ptr(sin), pos=_ptr(pos), dqkv=_ptr(dqkv), Bq=_ptr(Bq), Bv=_ptr(Bv),
                       dxlo_q=_ptr(dxlo_q), dxlo_v=_ptr(dxlo_v), lora_scale=float(lora_scale),
                       n=n, HQ=HQ, HKV=HKV, D=D, kv_heads_in=dk.shape[1], rank=16,
                       dtype=dtype_code(dtype), grad_dtype=dtype_code(dq.dtype))
    call("ql_rope_bwd", ctypes_ref(args), stream_ptr())
    return dqkv, dxlo_q, dxlo_v


# ---------------------------------------------------------------------------------------------
# SwiGLU, LoRA weight gradients, embedding
# ---------------------------------------------------------------------------------------------
def glu_fwd(gu, I, out=None):
    n = gu.shape[0]
    m = out if out is not None else torch.empty((n, I), device=gu.device, dtype=gu.dtype)
    call("ql_glu_fwd", _ptr(gu), _ptr(m), n, I, dtype_code(gu.dtype), stream_ptr())
    return m


def glu_bwd(dm, gu, I):
    call("ql_glu_bwd", _ptr(dm), _ptr(gu), gu.shape[0], I, dtype_code(gu.dtype), stream_ptr())
    return gu


def lora_colsum(X, Y, scale=1.0, transpose=False, out=None, workspace=None):
    """scale * X^T Y as [ncols, R] (or [R, ncols] with transpose), fp32; X [n, ncols] may be a
    column slice (unit column stride)."""
    n, ncols = X.shape
    R = Y.shape[1]
    if out is None:
        out = torch.empty((R, ncols) if transpose else (ncols, R), device=X.device,
                          dtype=torch.float32)
    need = int(_lib.lib().ql_lora_colsum_workspace(n, ncols, R))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, device=X.device, dtype=torch.float32)
    call("ql_lora_colsum", _ptr(X), X.stride(0), dtype_code(X.dtype), _ptr(Y),
         dtype_code(Y.dtype), n, ncols, R, float(scale), int(transpose), _ptr(out),
         _ptr(workspace), workspace.numel(), stream_ptr())
    return out


_LG_WS = {}


def lora_grads(jobs):
    """The LoRA weight gradients of a layer in one launch (ql_lora_grads). jobs: up to 4 tuples
    (X [n, ncols] 16-bit with unit column stride, Y [n, 16] 16-bit or fp32, scale, transpose);
    returns the fp32 outputs ([ncols, 16], or [16, ncols] when transposed)."""
    import ctypes

    n = jobs[0][0].shape[0]
    x_dtype = jobs[0][0].dtype
    outs, structs = [], []
    for X, Y, scale, transpose in jobs:
        ncols = X.shape[1]
        out = torch.empty((16, ncols) if transpose else (ncols, 16), device=X.device,
                          dtype=torch.float32)
        outs.append(out)
        structs.append(dict(X=_ptr(X), ldx=X.stride(0), Y=_ptr(Y), out=_ptr(out), ncols=ncols,
                            y_dtype=dtype_code(Y.dtype), transpose=int(transpose),
                            scale=float(scale)))
    arr = (_lib.STRUCTS["ql_lora_grad_job"] * len(jobs))(
        *[_lib.struct("ql_lora_grad_job", **f) for f in structs])
    nc = (ctypes.c_int32 * len(jobs))(*[X.shape[1] for X, _, _, _ in jobs])
    need = int(_lib.lib().ql_lora_grads_workspace(n, ctypes.addressof(nc), len(jobs)))
    ws = _LG_WS.get(jobs[0][0].device)
    if ws is None or ws.numel() < need:
        ws = torch.zeros(need, device=jobs[0][0].device, dtype=torch.uint8)  # counters start at 0
        _LG_WS[jobs[0][0].device] = ws
    call("ql_lora_grads", ctypes.addressof(arr), len(jobs), n, dtype_code(x_dtype), _ptr(ws),
         ws.numel(), stream_ptr())
    return outs


def embed(ids, W, out=None):
    """Rows W[ids] as fp32 [n, H]; W on the GPU, or in page-locked host memory (read over the
    host link by ql_embed_host)."""
    n = ids.numel()
    h = out if out is not None else torch.empty((n, W.shape[1]), device=ids.device,
                                                dtype=torch.float32)
    call("ql_embed" if W.is_cuda else "ql_embed_host", _ptr(ids), _ptr(W), _ptr(h), n,
         W.shape[1], W.shape[0], dtype_code(W.dtype), stream_ptr())
    return h


# ---------------------------------------------------------------------------------------------
# cross-entropy head
# ---------------------------------------------------------------------------------------------
def ce_rows(logits, target, write_grad=True, zero_unsupervised=False, loss=None, entropy=None,
            correct=None):
    rows, V = logits.shape
    dev = logits.device
    loss = loss if loss is not None else torch.empty(rows, device=dev, dtype=torch.float32)
    entropy = entropy if entropy is not None else torch.empty(rows, device=dev,
                                                              dtype=torch.float32)
    correct = correct if correct is not None else torch.empty(rows, device=dev,
                                                              dtype=torch.int32)
    args = _lib.struct("ql_ce_rows_args", logits=_ptr(logits), target=_ptr(target),
                       loss=_ptr(loss), entropy=_ptr(entropy), correct=_ptr(correct), rows=rows,
                       V=V, ld=logits.stride(0), write_grad=int(write_grad),
                       zero_unsupervised=int(zero_unsupervised), dtype=dtype_code(logits.dtype))
    call("ql_ce_rows", ctypes_ref(args), stream_ptr())
    return loss, entropy, correct


def ce_piece(logits, w, target, state, best_idx, xt, alpha, wt, v0, n_sup, acc=None,
             part=None, part_valid=False, H=None):
    """Reference _ce_piece (engine.py:1033-1038) on a vocabulary piece [v0, v0 + width) of the
    logits. acc / part: the fp32 gradient accumulator moved to the new running max in place,
    acc = alpha (acc + part) (part folded in when part_valid)."""
    rows, width = logits.shape
    args = _lib.struct("ql_ce_piece_args", logits=_ptr(logits), w=_ptr(w), target=_ptr(target),
                       state=_ptr(state), best_idx=_ptr(best_idx), xt=_ptr(xt),
                       alpha=_ptr(alpha), wt=_ptr(wt), rows=rows, v0=int(v0), width=width,
                       ld=logits.stride(0), n_sup=int(n_sup),
                       H=int(H) if H is not None else w.shape[1],
                       dtype=dtype_code(logits.dtype), acc=_ptr(acc), part=_ptr(part),
                       part_valid=int(bool(part_valid)))
    call("ql_ce_piece", ctypes_ref(args), stream_ptr())


def ce_finish(state, best_idx, xt, target, loss, entropy, correct, acc, wt, dh, n_sup,
              part=None):
    args = _lib.struct("ql_ce_finish_args", state=_ptr(state), best_idx=_ptr(best_idx),
                       xt=_ptr(xt), target=_ptr(target), loss=_ptr(loss),
                       entropy=_ptr(entropy), correct=_ptr(correct), acc=_ptr(acc),
                       wt=_ptr(wt), dh=_ptr(dh), rows=state.shape[0], n_sup=int(n_sup),
                       H=acc.shape[1], dtype=dtype_code(dh.dtype), part=_ptr(part))
    call("ql_ce_finish", ctypes_ref(args), stream_ptr())


# ---------------------------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------------------------
def attn_fwd(q, k, v, cu_seqlens, max_len, scale, out=None, lse=None):
    n, HQ, D = q.shape
    HKV = k.shape[1]
    out = out if out is not None else torch.empty_like(q)
    lse = lse if lse is not None else torch.empty((HQ, n), device=q.device, dtype=torch.float32)
    args = _lib.struct("ql_attn_fwd_args", q=_ptr(q), k=_ptr(k), v=_ptr(v),
                       cu_seqlens=_ptr(cu_seqlens), out=_ptr(out), lse=_ptr(lse),
                       scale=float(scale), n=n, B=cu_seqlens.numel() - 1, max_len=int(max_len),
                       HQ=HQ, HKV=HKV, D=D, dtype=dtype_code(q.dtype))
    call("ql_attn_fwd", ctypes_ref(args), stream_ptr())
    return out, lse


def attn_bwd(dout, q, k, v, out, lse, cu_seqlens, max_len, scale, dq=None, dk=None, dv=None,
             dvec=None, deterministic=False):
    """Reference _attn_bwd (engine.py:864-869): dq, dk, dv (fp32; dk / dv per KV head). With
    deterministic, each contribution goes to its own slot of a partials workspace and one kernel
    sums them in a fixed order (D = 128)."""
    n, HQ, D = q.shape
    HKV = k.shape[1]
    dev = q.device
    parts = None
    if deterministic:
        floats = int(_lib.lib().ql_attn_bwd_partials_floats(n, int(max_len), HQ, HKV))
        parts = torch.empty(max(floats, 4), device=dev, dtype=torch.float32)
    dq = dq if dq is not None else torch.empty((n, HQ, D), device=dev, dtype=torch.float32)
    dk = dk if dk is not None else torch.empty((n, HKV, D), device=dev, dtype=torch.float32)
    dv = dv if dv is not None else torch.empty((n, HKV, D), device=dev, dtype=torch.float32)
    dvec = dvec if dvec is not None else torch.empty((HQ, n), device=dev, dtype=torch.float32)
    args = _lib.struct("ql_attn_bwd_args", q=_ptr(q), k=_ptr(k), v=_ptr(v), out=_ptr(out),
                       dout=_ptr(dout), lse=_ptr(lse), cu_seqlens=_ptr(cu_seqlens),
                       dvec=_ptr(dvec), dq=_ptr(dq), dk=_ptr(dk), dv=_ptr(dv),
                       scale=float(scale), n=n, B=cu_seqlens.numel() - 1, max_len=int(max_len),
                       HQ=HQ, HKV=HKV, D=D, dtype=dtype_code(q.dtype), partials=_ptr(parts))
    call("ql_attn_bwd", ctypes_ref(args), stream_ptr())
    return dq, dk, dv


def gather_rows(src, idx, out=None):
    n, H = idx.numel(), src.shape[1]
    out = out if out is not None else torch.empty((n, H), device=src.device, dtype=torch.float32)
    call("ql_gather_rows", _ptr(src), _ptr(idx), _ptr(out), n, H, stream_ptr())
    return out


def scatter_rows(src, idx, out, scale=None, out16=None):
    n, H = src.shape
    call("ql_scatter_rows", _ptr(src), _ptr(idx), _ptr(scale), _ptr(out), _ptr(out16), n, H,
         dtype_code(out16.dtype) if out16 is not None else 0, stream_ptr())
    return out
