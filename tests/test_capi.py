"""The C ABI surface of libpyrite_b200.so (CPU: no compute calls).

* The library loads and exports every function include/pyrite_b200.h declares.
* The reference-compatible table call returns the reference's 21 ids in the
  reference's order (pyrite/kernels/native.c:451-473, 484-494).
* Argument validation runs before any device work and returns the reference's
  codes (-1 unknown type, -2 bad shape, -3 buffer/length; native.c:496-525).
* The Python shim mirrors the reference module's surface and, without a CUDA
  device, reports itself unavailable and raises -- it never computes on the CPU.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from pyrite_b200 import _lib
from pyrite_b200.kernels import native

HEADER = Path(__file__).resolve().parent.parent / "include" / "pyrite_b200.h"
REFERENCE_ORDER = [0, 1, 2, 3, 6, 7, 8, 9, 10, 11, 12, 13, 14, 20, 23, 24, 25, 26, 27, 28, 30]


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"\b(pyrite_\w+)\s*\(", text)


@pytest.fixture(scope="module")
def lib():
    lib = _lib.load()
    assert lib is not None, "libpyrite_b200.so failed to build/load"
    return lib


def test_library_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 9
    assert set(names) == set(_lib.SIGNATURES), "binding table and header disagree"
    for name in names:
        assert hasattr(lib, name), f"{name} not exported"


def test_type_table_is_the_reference_table(lib):
    assert lib.pyrite_native_types(None, 0) == 21
    assert _lib.type_ids(lib) == REFERENCE_ORDER
    buf = (ctypes.c_int * 4)()
    assert lib.pyrite_native_types(buf, 4) == 4
    assert list(buf) == REFERENCE_ORDER[:4]


def test_type_geometry(lib):
    bs, bpb = ctypes.c_size_t(), ctypes.c_size_t()
    for t, want in {8: (32, 34), 12: (256, 144), 13: (256, 176), 14: (256, 210), 23: (256, 136), 0: (1, 4)}.items():
        assert lib.pyrite_type_geometry(t, ctypes.byref(bs), ctypes.byref(bpb)) == 0
        assert (bs.value, bpb.value) == want
    assert lib.pyrite_type_geometry(15, ctypes.byref(bs), ctypes.byref(bpb)) == -1  # Q8_K: not decodable


def test_validation_codes_match_the_reference(lib):
    pd = ctypes.POINTER(ctypes.c_double)
    x = np.zeros(64)
    out = np.zeros(4)
    buf = np.zeros(68, dtype=np.uint8)

    def mv(t, n, rows, cols, data=True):
        return lib.pyrite_matvec(t, buf.ctypes.data if data else None, n, x.ctypes.data_as(pd),
                                 out.ctypes.data_as(pd), rows, cols)

    assert mv(99, 68, 1, 64) == -1           # unknown type
    assert mv(16, 68, 1, 64) == -1           # known to GGML, not decodable
    assert mv(8, 68, 0, 64) == -2            # zero rows
    assert mv(8, 68, 1, 0) == -2             # zero cols
    assert mv(8, 68, 1, 48) == -2            # cols not a multiple of 32
    assert mv(8, 67, 1, 64) == -3            # payload length mismatch
    assert mv(8, 68, 1, 64, data=False) == -3
    assert lib.pyrite_dequantize_rows(8, buf.ctypes.data, 68, None, 1, 64) == -3
    dev = ctypes.c_void_p(1 << 20)           # never dereferenced: validation fails first
    assert lib.pyrite_cuda_matvec(12, dev, 143, dev, 256, dev, 1, 1, 256, 1, 0, None, 0, None) == -3
    assert lib.pyrite_cuda_matvec(12, dev, 144, dev, 256, dev, 1, 1, 255, 1, 0, None, 0, None) == -2
    assert lib.pyrite_cuda_matvec(12, dev, 144, dev, 256, dev, 1, 1, 256, 0, 0, None, 0, None) == -3


def test_error_strings(lib):
    for code in (0, -1, -2, -3, -4):
        assert lib.pyrite_error_string(code)


def test_shim_mirrors_the_reference_surface():
    for name in ("matvec", "dequantize_rows", "supports_native", "native_available", "native_type_ids",
                 "sorted_native_types", "NATIVE_TYPES"):
        assert hasattr(native, name)
    assert native.NATIVE_TYPES == frozenset(REFERENCE_ORDER)
    assert native.native_type_ids() == tuple(REFERENCE_ORDER)
    assert "Q4_K" in native.sorted_native_types()


def test_without_a_device_the_shim_refuses_instead_of_computing_on_cpu():
    if _lib.device_count() > 0:
        pytest.skip("a CUDA device is present")
    assert native.native_available() is False
    assert native.supports_native(8) is False
    with pytest.raises(ValueError, match="no native kernel"):
        native.matvec(8, bytes(34), [0.0] * 32, 1, 32)
    lib = _lib.load()
    pd = ctypes.POINTER(ctypes.c_double)
    x = np.zeros(32)
    out = np.zeros(1)
    buf = np.zeros(34, dtype=np.uint8)
    assert lib.pyrite_matvec(8, buf.ctypes.data, 34, x.ctypes.data_as(pd), out.ctypes.data_as(pd), 1, 32) == -4


def test_post_op_struct_layout_matches_the_header(tmp_path):
    """The ctypes mirror of pyrite_post_op has the C compiler's layout."""
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    fields = [f for f, _ in _lib.PostOp._fields_]
    src = tmp_path / "layout.c"
    src.write_text("#include <stdio.h>\n#include <stddef.h>\n#include \"pyrite_b200.h\"\nint main(void){\n"
                   + "".join(f'printf("%zu\\n", offsetof(pyrite_post_op, {f}));\n' for f in fields)
                   + 'printf("%zu\\n", sizeof(pyrite_post_op));\nreturn 0;}\n')
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    want = [getattr(_lib.PostOp, f).offset for f in fields] + [ctypes.sizeof(_lib.PostOp)]
    assert got == want
