"""Loads libqlora_sm100a.so (built in-tree by build.py) and binds its C ABI for ctypes.

The argument structs and prototypes are read from include/qlora_sm100.h itself, so the Python
binding cannot drift from the header (tests/test_abi.py also checks the layouts against gcc).
There is no fallback: if the library is missing or does not load, every op raises.
"""

import ctypes
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libqlora_sm100a.so")
HEADER = os.path.join(os.path.dirname(_HERE), "include", "qlora_sm100.h")

_SCALARS = {"int": ctypes.c_int, "int32_t": ctypes.c_int32, "int64_t": ctypes.c_int64,
            "uint32_t": ctypes.c_uint32,
            "long long": ctypes.c_longlong,
            "float": ctypes.c_float, "double": ctypes.c_double, "void": None}


def _strip_comments(text):
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    return re.sub(r"//[^\n]*", " ", text)


def _ctype(decl_type, structs=None):
    t = decl_type.replace("const", " ").strip()
    if structs and "*" not in t and t in structs:
        return structs[t]
    if "*" in t:
        if re.sub(r"\s+", "", t) == "char*":
            return ctypes.c_char_p
        return ctypes.c_void_p
    t = re.sub(r"\s+", " ", t).strip()
    if t == "cudaStream_t":
        return ctypes.c_void_p
    if t not in _SCALARS:
        raise ValueError(f"unknown C type {decl_type!r}")
    return _SCALARS[t]


def parse_header(path=HEADER):
    """(structs: name -> ctypes.Structure subclass, functions: name -> (restype, argtypes))."""
    with open(path, encoding="utf-8") as fh:
        text = _strip_comments(fh.read())
    structs = {}
    for body, name in re.findall(r"typedef\s+struct\s*\{(.*?)\}\s*(\w+)\s*;", text, flags=re.S):
        fields = []
        for decl in body.split(";"):
            decl = " ".join(decl.split())
            if not decl:
                continue
            m = re.match(r"^((?:const\s+)?[A-Za-z_]\w*(?:\s*\*)?)\s*(.*)$", decl)
            base, names = m.group(1), m.group(2)
            for nm in names.split(","):
                nm = nm.strip()
                stars = nm.count("*")
                nm = nm.replace("*", "").strip()
                fields.append((nm, _ctype(base + "*" * stars, structs)))
        structs[name] = type(name, (ctypes.Structure,), {"_fields_": fields})
    functions = {}
    for ret, name, args in re.findall(r"\b((?:const\s+)?(?:long\s+long|[A-Za-z_]\w*)\s*\**)\s*(ql_\w+)\s*\(([^)]*)\)\s*;",
                                      text):
        argtypes = []
        args = args.strip()
        if args and args != "void":
            for a in args.split(","):
                a = " ".join(a.split())
                m = re.match(r"^(.*?)(\w+)$", a)
                argtypes.append(_ctype(m.group(1)))
        functions[name] = (_ctype(ret), argtypes)
    return structs, functions


STRUCTS, FUNCTIONS = parse_header()
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
        for name, (restype, argtypes) in FUNCTIONS.items():
            fn = getattr(handle, name)
            fn.argtypes = argtypes
            fn.restype = restype
        _lib = handle
    return _lib


def call(name, *args):
    """Calls an entry point returning a status and raises QLError unless it is 0."""
    status = getattr(lib(), name)(*args)
    if status != 0:
        msg = lib().ql_last_error().decode(errors="replace")
        raise QLError(name, status, msg)
    return status


def struct(name, **fields):
    """An argument struct of the header, zero-initialised, with the given fields set."""
    s = STRUCTS[name]()
    for k, v in fields.items():
        setattr(s, k, v)
    return s


def exported_symbols():
    return list(FUNCTIONS)
