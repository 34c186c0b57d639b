"""CPU: the C-ABI library loads, exports every entry point include/qlora_sm100.h declares, and the
argument structs the Python binding reads from the header have the C compiler's layout. No
compute call is made (there is no GPU here)."""

import ctypes
import os
import subprocess

import pytest

from hack_fe30cb28_opus_5_5_ultracode_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.lib()
    names = _lib.exported_symbols()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), name
    assert b"sm_100a" in lib.ql_version()
    assert lib.ql_last_error() == b""
    assert lib.ql_launch_count() >= 0


def test_struct_layouts_match_the_c_compiler(tmp_path):
    src = ['#include <stddef.h>', '#include <stdio.h>', '#include "qlora_sm100.h"',
           'int main(void) {']
    for name, cls in _lib.STRUCTS.items():
        src.append(f'  printf("{name} size %zu\\n", sizeof({name}));')
        for field, _ in cls._fields_:
            src.append(f'  printf("{name} {field} %zu\\n", offsetof({name}, {field}));')
    src += ['  return 0;', '}']
    c = tmp_path / "layout.c"
    c.write_text("\n".join(src))
    exe = tmp_path / "layout"
    res = subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), "-I",
                          "/usr/local/cuda/include", str(c), "-o", str(exe)],
                         capture_output=True, text=True)
    if res.returncode != 0:
        pytest.skip(f"gcc could not build the layout probe: {res.stderr[:200]}")
    lines = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    checked = 0
    for line in filter(None, lines):
        parts = line.split()
        cls = _lib.STRUCTS[parts[0]]
        if parts[1] == "size":
            assert ctypes.sizeof(cls) == int(parts[2]), parts
        else:
            assert getattr(cls, parts[1]).offset == int(parts[2]), parts
        checked += 1
    assert checked > 100


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "missing.so"))
    with pytest.raises(ImportError):
        _lib.lib()


def test_status_constant_matches_the_header():
    import re

    from hack_fe30cb28_opus_5_5_ultracode_b200 import _lib, ops

    text = open(_lib.HEADER, encoding="utf-8").read()
    assert int(re.search(r"QL_STATUS_TIMEOUT\s*=\s*(\d+)", text).group(1)) == ops.STATUS_TIMEOUT
    assert int(re.search(r"QL_STATUS_UNSUPPORTED\s*=\s*(\d+)", text).group(1)) == \
        ops.STATUS_UNSUPPORTED
