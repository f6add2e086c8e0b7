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


def test_workspace_query_decides_in_place_operands():
    """pk_poly_gemm_workspace_query only inspects pointer alignment and strides (host-side), so
    it runs without a GPU on made-up plane addresses."""
    from polytensors_b200 import _lib

    lib = _lib.load()
    n, M, N, K = 2, 256, 512, 192

    def query(dtype, a_ptrs, a_strides, b_ptrs, b_strides, batch=1):
        pa = (ctypes.c_void_p * len(a_ptrs))(*a_ptrs)
        pb = (ctypes.c_void_p * len(b_ptrs))(*b_ptrs)
        need = ctypes.c_size_t(7)
        status = lib.pk_poly_gemm_workspace_query(dtype, n, batch, M, N, K, pa, *a_strides, pb, *b_strides,
                                                  n + 1, n + 1, ctypes.byref(need))
        assert status == 0, _lib.last_error()
        return need.value

    aligned = [0x10000 * (i + 1) for i in range(n + 1)]
    odd = [p + 2 for p in aligned]
    kmaj_a, mn_a = (0, K, 1), (0, 1, M)          # (batch, row, k) strides of A
    kmaj_b, mn_b = (0, 1, K), (0, N, 1)          # (batch, k, col) strides of B
    assert query(_lib.PK_BF16, aligned, kmaj_a, aligned, kmaj_b) == 0
    assert query(_lib.PK_BF16, aligned, mn_a, aligned, mn_b) == 0
    staged_a = query(_lib.PK_BF16, odd, kmaj_a, aligned, kmaj_b)
    assert 0 < staged_a < lib.pk_poly_gemm_workspace_size(_lib.PK_BF16, n, 1, M, N, K, n + 1, n + 1)
    assert query(_lib.PK_BF16, aligned, (0, K + 3, 1), aligned, kmaj_b) > 0      # row stride not 16-byte
    assert query(_lib.PK_F32, aligned, kmaj_a, aligned, kmaj_b) > 0              # float32 is always split
    assert query(_lib.PK_BF16, aligned, (M * K, K, 1), aligned, (N * K, 1, K), batch=4) == 0
    assert query(_lib.PK_BF16, aligned, (K, K, 1), aligned, kmaj_b, batch=4) > 0  # overlapping batch entries
