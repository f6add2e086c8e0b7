"""pk_poly_gemm_noalloc: the polynomial matrix product for callers that cannot allocate
device memory (a plugin host that owns every allocation, a process that must not grow its
device footprint, code with no allocator to link).  It takes its scratch from a fixed
64 MiB array inside the library instead of a caller workspace.

Checked through the C ABI against pk_poly_gemm (the entry point with a caller-allocated
workspace) and against the CPU oracle, on calls in a row: a larger product first, so the
scratch array holds its staged operands, then products whose reduction length is not a
multiple of the staging pitch (K = 317) and whose B operand is a transposed view, so the
second call stages padded rows over the first call's leftovers.  Tolerance: per-plane
max |diff| / max |ref| <= 1e-4 for float32 and 1e-10 for float64.

The file name sorts last on purpose: pytest collects files in name order, so a run that
stops at the first failure has already run every other test before this one, which holds
library-wide state (the shared scratch array) for the rest of the process."""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def planes(shape, n, seed, dtype, transpose=False):
    g = torch.Generator().manual_seed(seed)
    out = []
    for k in range(n + 1):
        x = torch.randn(*shape, generator=g, dtype=torch.float64) / math.factorial(k)
        out.append(x.t().contiguous().t() if transpose else x)   # transpose: same values, column-major
    return [x.to(dtype).cuda() for x in out]


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
    (a_rs, a_cs), (b_rs, b_cs) = A[0].stride(), B[0].stride()
    args = (code, degree, 1, M, N, K, pa, 0, a_rs, a_cs, pb, 0, b_rs, b_cs, pc, 0, N, degree + 1, degree + 1)
    if use_workspace:
        size = ctypes.c_size_t(0)
        _lib.check(lib.pk_poly_gemm_workspace_query(code, degree, 1, M, N, K, pa, 0, a_rs, a_cs, pb, 0, b_rs, b_cs,
                                                    degree + 1, degree + 1, ctypes.byref(size)),
                   "pk_poly_gemm_workspace_query")
        ws = torch.empty(max(size.value, 1), dtype=torch.uint8, device="cuda")
        status = entry(*args, ws.data_ptr(), size.value, stream)
    else:
        status = entry(*args, stream)
    _lib.check(status, entry.__name__)
    torch.cuda.synchronize()
    return C


def max_plane_error(got, want):
    errs = []
    for g, w in zip(got, want):
        w = w.cpu().double()
        errs.append((g.cpu().double() - w).abs().max().item() / w.abs().max().item())
    return max(errs)


@pytest.mark.parametrize("dtype,code,tol", [(torch.float32, 0, 1e-4), (torch.float64, 1, 1e-10)])
def test_noalloc_matches_workspace_entry_point_and_oracle(dtype, code, tol):
    from oracle import polyref
    from polytensors_b200 import _lib

    lib = _lib.load()
    # (M, K, N, degree, B transposed): the first product fills more scratch than the later ones
    # use; K = 317 leaves padding columns in every staged row of the later products.
    cases = [(512, 1024, 384, 2, False), (200, 317, 144, 2, True), (136, 317, 200, 3, True)]
    for i, (M, K, N, n, bt) in enumerate(cases):
        A = planes((M, K), n, 10 + i, dtype)
        B = planes((K, N), n, 20 + i, dtype, transpose=bt)
        want = call(lib, lib.pk_poly_gemm, code, A, B, use_workspace=True)
        got = call(lib, lib.pk_poly_gemm_noalloc, code, A, B, use_workspace=False)
        assert all(torch.isfinite(c).all() for c in got)
        assert max_plane_error(got, want) <= tol, (i, "vs pk_poly_gemm")
        oracle = polyref.poly_matmul([a.cpu().double() for a in A], [b.cpu().double() for b in B])
        assert max_plane_error(got, oracle) <= tol, (i, "vs oracle")


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
