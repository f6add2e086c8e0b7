"""The C ABI library: it builds, loads without a GPU, and exports every symbol that
include/polykern.h declares (no compute calls here)."""

import ctypes
import re

from conftest import ROOT


def declared_symbols():
    text = (ROOT / "include" / "polykern.h").read_text()
    return sorted(set(re.findall(r"PK_API\s+[\w\s\*]+?\b(pk_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "pk_poly_gemm" in names and "pk_last_error" in names


def test_library_exports_declared_symbols():
    from polytensors_b200 import _build, _lib

    path = _build.build()
    lib = ctypes.CDLL(str(path))
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    lib.pk_version.restype = ctypes.c_char_p
    assert lib.pk_version().startswith(b"polykern")


def test_argument_errors_need_no_gpu():
    from polytensors_b200 import _lib

    lib = _lib.load()
    assert lib.pk_poly_gemm_workspace_size(0, 99, 1, 8, 8, 8, 0, 0) == 0   # degree out of range
    assert lib.pk_poly_gemm_workspace_size(0, 2, 1, 128, 128, 64, 3, 3) > 0
    status = lib.pk_poly_gemm(0, 99, 1, 8, 8, 8, None, 0, 0, 0, None, 0, 0, 0, None, 0, 0, 0, 0, None, 0, None)
    assert status == -2
    assert "degree" in _lib.last_error()
