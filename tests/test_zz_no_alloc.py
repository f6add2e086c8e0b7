"""pk_poly_gemm_noalloc: the polynomial matrix product for callers that cannot allocate
device memory (a plugin host that owns every allocation, a process that must not grow its
device footprint, code with no allocator to link).  It takes its scratch from a fixed
64 MiB array inside the library instead of a caller workspace.

Checked through the C ABI against pk_poly_gemm (the entry point with a caller-allocated
workspace), on two calls in a row so that the second call runs on scratch that still
holds the first call's contents.  Tolerance: per-plane max |diff| / max |ref| <= 1e-4
for float32 and 1e-10 for float64 (the kernels are the same, so the results agree far
more closely)."""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def planes(shape, n, seed, dtype):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(*shape, generator=g, dtype=torch.float64) / math.factorial(k)).to(dtype).cuda()
            for k in range(n + 1)]


def call(lib, entry, code, A, B, use_workspace):
    from polytensors_b200 import _lib

    M, K = A[0].shape
    N = B[0].shape[1]
    degree = len(A) - 1
    C = [torch.full((M, N), float("nan"), dtype=A[0].dtype, device="cuda") for _ in A]
    pa, ka = _lib.pointer_array(A)
    pb, kb = _lib.pointer_array(B)
    pc, kc = _lib.pointer_array(C)
    stream = torch.cuda.current_stream().cuda_stream
    args = (code, degree, 1, M, N, K, pa, 0, K, 1, pb, 0, N, 1, pc, 0, N, degree + 1, degree + 1)
    if use_workspace:
        size = lib.pk_poly_gemm_workspace_size(code, degree, 1, M, N, K, degree + 1, degree + 1)
        ws = torch.empty(size, dtype=torch.uint8, device="cuda")
        status = entry(*args, ws.data_ptr(), size, stream)
    else:
        status = entry(*args, stream)
    _lib.check(status, entry.__name__)
    torch.cuda.synchronize()
    return C


def max_plane_error(got, want):
    errs = []
    for g, w in zip(got, want):
        denom = w.abs().max().item()
        errs.append((g.double() - w.double()).abs().max().item() / denom)
    return max(errs)


@pytest.mark.parametrize("dtype,code,tol", [(torch.float32, 0, 1e-4), (torch.float64, 1, 1e-10)])
def test_noalloc_matches_workspace_entry_point(dtype, code, tol):
    from polytensors_b200 import _lib

    lib = _lib.load()
    for call_index in range(2):   # second call reuses scratch left over from the first
        A = planes((384, 320), 2, 10 + call_index, dtype)
        B = planes((320, 272), 2, 20 + call_index, dtype)
        want = call(lib, lib.pk_poly_gemm, code, A, B, use_workspace=True)
        got = call(lib, lib.pk_poly_gemm_noalloc, code, A, B, use_workspace=False)
        assert all(torch.isfinite(c).all() for c in got)
        assert max_plane_error(got, want) <= tol


def test_noalloc_rejects_products_beyond_its_scratch():
    from polytensors_b200 import _lib

    lib = _lib.load()
    degree, M = 4, 8192
    need = lib.pk_poly_gemm_workspace_size(0, degree, 1, M, M, M, degree + 1, degree + 1)
    assert need > (64 << 20)
    # A row stride of M + 1 floats (not a multiple of 4) makes both operands go through the
    # workspace staging, so the call needs more scratch than the array holds and is rejected
    # before anything is launched (the 1-element planes are never read).
    dummy = [torch.empty(1, device="cuda") for _ in range(degree + 1)]
    pa, ka = _lib.pointer_array(dummy)
    size = ctypes.c_size_t(0)
    assert lib.pk_poly_gemm_workspace_query(0, degree, 1, M, M, M, pa, 0, M + 1, 1, pa, 0, M + 1, 1,
                                            degree + 1, degree + 1, ctypes.byref(size)) == 0
    assert size.value > (64 << 20)
    status = lib.pk_poly_gemm_noalloc(0, degree, 1, M, M, M, pa, 0, M + 1, 1, pa, 0, M + 1, 1, pa, 0, M,
                                      degree + 1, degree + 1, torch.cuda.current_stream().cuda_stream)
    assert status == -2
    assert "scratch" in _lib.last_error()
