"""torch-facing wrappers of the C ABI: each takes CUDA tensors, checks layouts, and launches on
the current stream. Names follow the reference's launch wrappers (solution/engine.py:103-109,
947-1045) so the tests read like the reference's own.
"""

import torch

from . import _lib
from ._lib import call

_DT = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}
INT_MAX = 2147483647


def dtype_code(dtype):
    try:
        return _DT[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}") from None


def stream_ptr():
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


# ---------------------------------------------------------------------------------------------
# GEMM
# ---------------------------------------------------------------------------------------------
def gemm(a, b, out=None, bias=None, accumulate=False, out_dtype=None):
    """out[M, N] (+)= a[M, K] @ b[N, K]^T (+ bias) on tcgen05. a and b: fp16 or bf16 with unit
    column stride; out: fp16 / bf16 / fp32 with unit column stride."""
    M, K = a.shape
    N, K2 = b.shape
    if K != K2:
        raise ValueError(f"inner dimensions differ: {a.shape} x {b.shape}^T")
    if a.dtype != b.dtype:
        raise ValueError("a and b must have the same dtype")
    if out is None:
        out = torch.empty((M, N), device=a.device, dtype=out_dtype or a.dtype)
    _need_cuda(a, b, out, bias)
    if a.stride(1) != 1 or b.stride(1) != 1 or out.stride(1) != 1:
        raise ValueError("gemm needs unit column strides")
    if bias is not None and bias.dtype != a.dtype:
        raise ValueError("bias must have the input dtype")
    call("ql_gemm_tn", _ptr(a), a.stride(0), _ptr(b), b.stride(0), _ptr(out), out.stride(0),
         _ptr(bias), M, N, K, dtype_code(a.dtype), dtype_code(out.dtype), int(accumulate),
         stream_ptr())
    return out


def device_status(clear=True):
    """The library's device status word (QL_STATUS_TIMEOUT if a kernel gave up a wait)."""
    import ctypes

    v = ctypes.c_int(0)
    call("ql_device_status", ctypes.addressof(v), int(clear))
    return v.value
