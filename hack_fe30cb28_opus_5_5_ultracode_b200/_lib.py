"""Loads libqlora_sm100a.so (built in-tree by build.py) and declares its C ABI for ctypes.

There is no fallback: if the library is missing or does not load, every op raises. The
signatures below mirror include/qlora_sm100.h one for one.
"""

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libqlora_sm100a.so")

P = ctypes.c_void_p
I32 = ctypes.c_int
I64 = ctypes.c_int64
F32 = ctypes.c_float
U64 = ctypes.c_uint64

# name -> argument types (every function returns int status unless listed in _RESTYPES)
SIGNATURES = {
    "ql_version": [],
    "ql_last_error": [],
    "ql_device_status": [P, I32],
    "ql_device_status_ptr": [],
    "ql_nf4_dequant": [P, P, P, P, P, P, P, I64, I64, I32, I32, I64, I64, I32, I32, P],
    "ql_gemm_tn": [P, I64, P, I64, P, I64, P, I32, I32, I32, I32, I32, I32, P],
}
_RESTYPES = {"ql_version": ctypes.c_char_p, "ql_last_error": ctypes.c_char_p,
             "ql_device_status_ptr": P}

_lib = None


class QLError(RuntimeError):
    """A failed call into the CUDA library (its status code and message)."""

    def __init__(self, name, status, message):
        super().__init__(f"{name} failed with status {status}: {message}")
        self.status = status


def lib():
    """The loaded library; raises if it was not built (no CPU or eager fallback exists)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with "
                              "`python -m hack_fe30cb28_opus_5_5_ultracode_b200.build`")
        handle = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, I32)
        _lib = handle
    return _lib


def call(name, *args):
    """Calls an entry point and raises QLError on a non-zero status."""
    status = getattr(lib(), name)(*args)
    if status != 0:
        msg = lib().ql_last_error().decode(errors="replace")
        raise QLError(name, status, msg)
    return status


def exported_symbols():
    return list(SIGNATURES)
