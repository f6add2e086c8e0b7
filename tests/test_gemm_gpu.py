"""Parity of the polynomial matrix product (pk_poly_gemm) with the CPU oracle.

Tolerances (per coefficient plane, max |got - want| / max |want|): float32 1e-4,
float64 / complex128 1e-10, bfloat16 storage 2e-2."""

import math

import pytest
import torch

from oracle import polyref as ref

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.float64: 1e-10, torch.complex128: 1e-10, torch.bfloat16: 2e-2}


def series(shape, n, seed, dtype=torch.float32, complex_from=None):
    g = torch.Generator().manual_seed(seed)
    out = []
    for k in range(n + 1):
        x = torch.randn(*shape, generator=g, dtype=torch.float64) / math.factorial(k)
        if complex_from is not None and k >= complex_from:
            x = torch.complex(x, torch.randn(*shape, generator=g, dtype=torch.float64) / math.factorial(k))
        out.append(x if x.is_complex() else x.to(dtype))
    return out


def cuda(planes):
    return [p.cuda() for p in planes]


def check(A, B, tol, got=None):
    from polytensors_b200 import _kernels

    got = _kernels.poly_matmul(cuda(A), cuda(B)) if got is None else got
    want = ref.poly_matmul([a.double() if not a.is_complex() else a for a in A],
                           [b.double() if not b.is_complex() else b for b in B])
    for g, w in zip(got, want):
        assert g.shape == w.shape
    errs = ref.plane_errors(got, want)
    assert max(errs) <= tol, errs
    return errs


@pytest.mark.parametrize("n", [2, 4, 8])
def test_f32_square_1024(n):
    A, B = series((1024, 1024), n, 1), series((1024, 1024), n, 2)
    check(A, B, TOL[torch.float32])


@pytest.mark.parametrize("M,N,K,n", [(257, 129, 200, 3), (1, 300, 77, 2), (130, 1, 64, 1), (64, 96, 8, 0),
                                     (333, 517, 1031, 2)])
def test_f32_ragged(M, N, K, n):
    A, B = series((M, K), n, 3), series((K, N), n, 4)
    check(A, B, TOL[torch.float32])


def test_f32_transposed_and_batched():
    from polytensors_b200 import _kernels

    A = series((3, 100, 70), 2, 5)
    W = series((3, 90, 70), 2, 6)                     # B = W^T: a non-contiguous operand
    Bt = [w.transpose(-2, -1) for w in W]
    got = _kernels.poly_matmul(cuda(A), [w.cuda().transpose(-2, -1) for w in W])
    check(A, Bt, TOL[torch.float32], got=got)


def test_f32_large_wide_tiles():
    A, B = series((2048, 4096), 2, 7), series((4096, 3072), 2, 8)
    check(A, B, TOL[torch.float32])


@pytest.mark.parametrize("M,N,K,n", [(256, 320, 192, 3), (129, 65, 33, 2), (1, 1, 1, 4)])
def test_f64(M, N, K, n):
    A, B = series((M, K), n, 9, torch.float64), series((K, N), n, 10, torch.float64)
    check(A, B, TOL[torch.float64])


def test_c128_directions():
    A = series((128, 80), 2, 11, torch.float64, complex_from=1)
    B = series((80, 96), 2, 12, torch.float64, complex_from=1)
    check(A, B, TOL[torch.complex128])


def test_c128_one_side_complex():
    A = series((64, 48), 3, 13, torch.float64)
    B = series((48, 40), 3, 14, torch.float64, complex_from=1)
    check(A, B, TOL[torch.complex128])


def test_bf16_storage():
    A, B = series((512, 384), 2, 15, torch.bfloat16), series((384, 256), 2, 16, torch.bfloat16)
    check(A, B, TOL[torch.bfloat16])


def _layout(planes, how):
    """CUDA copies of (batch, R, K) planes laid out K-contiguous ("k"), rows-contiguous ("rows"),
    or at a 2-byte offset that no tensor map can start from ("odd")."""
    out = []
    for p in planes:
        if how == "k":
            out.append(p.cuda().contiguous())
        elif how == "rows":
            out.append(p.transpose(-2, -1).contiguous().cuda().transpose(-2, -1))
        else:
            big = torch.zeros(*p.shape[:-1], p.shape[-1] + 1, dtype=p.dtype, device="cuda")
            big[..., 1:] = p.cuda()
            out.append(big[..., 1:])
    return out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("a_how", ["k", "rows", "odd"])
@pytest.mark.parametrize("b_how", ["k", "rows", "odd"])
def test_16bit_operands_read_in_place(a_how, b_how, dtype):
    """bf16 / f16 planes are read where they lie (K-major or MN-major tensor maps, no staging) when
    aligned, and staged otherwise; every combination, batched, with ragged M / N / K tails.
    Tolerance 1e-2 of the plane max-norm: exact 16-bit products, fp32 sums, 16-bit output."""
    from polytensors_b200 import _kernels, _lib

    batch, M, N, K, n = 3, 200, 296, 136, 2
    A = series((batch, M, K), n, 21, dtype)
    W = series((batch, N, K), n, 22, dtype)         # B = W^T
    a = _layout(A, a_how)
    b = [w.transpose(-2, -1) for w in _layout(W, b_how)]   # "k": k contiguous in B
    got = _kernels.poly_matmul(a, b)
    check(A, [w.transpose(-2, -1) for w in W], 1e-2, got=got)
    # the workspace query reports no scratch for the in-place operands
    lib = _lib.load()
    pa, ka = _lib.pointer_array(a)
    pb, kb = _lib.pointer_array(b)
    import ctypes
    need = ctypes.c_size_t(1)
    code = _lib.PK_BF16 if dtype == torch.bfloat16 else _lib.PK_F16
    assert lib.pk_poly_gemm_workspace_query(code, n, batch, M, N, K, pa, *a[0].stride(), pb,
                                            *b[0].stride(), n + 1, n + 1, ctypes.byref(need)) == 0
    assert (need.value == 0) == (a_how != "odd" and b_how != "odd")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float64])
def test_accumulate_into_strided_views(dtype):
    """pk_poly_gemm_accumulate: C_k += sum A_i B_{k-i} into views of larger planes (addmm with
    beta = 1), against the oracle product plus the prior contents."""
    from polytensors_b200 import _kernels

    n, batch, M, N, K = 2, 2, 136, 200, 72
    A, B = series((batch, M, K), n, 31, dtype), series((batch, K, N), n, 32, dtype)
    C0 = series((batch, M + 8, N + 16), n, 33, dtype)
    big = cuda(C0)
    views = [c[:, 8:, 16:] for c in big]
    _kernels.poly_matmul(cuda(A), cuda(B), out=views, accumulate=True)
    prod = ref.poly_matmul([a.double() for a in A], [b.double() for b in B])
    want = [p + c[:, 8:, 16:].double() for p, c in zip(prod, C0)]
    tol = {torch.float32: 1e-4, torch.bfloat16: 1e-2, torch.float64: 1e-10}[dtype]
    assert max(ref.plane_errors(views, want)) <= tol
    for c, c0 in zip(big, C0):   # untouched outside the views
        assert torch.equal(c[:, :8].cpu(), c0[:, :8]) and torch.equal(c[:, :, :16].cpu(), c0[:, :, :16])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float64])
@pytest.mark.parametrize("band,offset", [(1, 0), (2, 0), (1, 200), (2, -150), (1, -64)])
def test_banded_product(dtype, band, offset):
    """pk_poly_gemm_banded: A zero outside the band (1: k >= m + offset, 2: k <= m + offset) gives
    the plain product; row tiles whose band holds no k block write zeros (or add nothing)."""
    from polytensors_b200 import _kernels

    batch, M, N, K, n = 2, 300, 136, 260, 2
    A, B = series((batch, M, K), n, 41, dtype), series((batch, K, N), n, 42, dtype)
    m = torch.arange(M).view(M, 1)
    k = torch.arange(K).view(1, K)
    keep = (k >= m + offset) if band == 1 else (k <= m + offset)
    A = [a * keep.to(a.dtype) for a in A]
    tol = {torch.bfloat16: 1e-2, torch.float32: 1e-4, torch.float64: 1e-10}[dtype]
    got = _kernels.poly_matmul(cuda(A), cuda(B), band=band, band_offset=offset)
    check(A, B, tol, got=got)
    C0 = series((batch, M, N), n, 43, dtype)
    out = cuda(C0)
    _kernels.poly_matmul(cuda(A), cuda(B), out=out, accumulate=True, band=band, band_offset=offset)
    want = [w + c.double() for w, c in zip(ref.poly_matmul([a.double() for a in A], [b.double() for b in B]), C0)]
    assert max(ref.plane_errors(out, want)) <= tol


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("N", [1, 17, 64])
@pytest.mark.parametrize("n", [1, 3])
def test_narrow_products(dtype, N, n):
    """N <= 64 runs in 64-column tiles: plain, B read transposed, batched, banded, accumulated."""
    from polytensors_b200 import _kernels

    tol = {torch.bfloat16: 1e-2, torch.float32: 1e-4}[dtype]
    batch, M, K = 2, 300, 260
    A, B = series((batch, M, K), n, 51, dtype), series((batch, K, N), n, 52, dtype)
    check(A, B, tol)
    Bt = [b.transpose(1, 2).contiguous() for b in B]  # rows of B contiguous in memory
    got = _kernels.poly_matmul(cuda(A), [b.cuda().transpose(1, 2) for b in Bt])
    check(A, B, tol, got=got)
    keep = torch.arange(K).view(1, K) >= torch.arange(M).view(M, 1) - 40
    Ab = [a * keep.to(a.dtype) for a in A]
    check(Ab, B, tol, got=_kernels.poly_matmul(cuda(Ab), cuda(B), band=1, band_offset=-40))
    C0 = series((batch, M, N), n, 53, dtype)
    out = cuda(C0)
    _kernels.poly_matmul(cuda(A), cuda(B), out=out, accumulate=True)
    want = [w + c.double() for w, c in zip(ref.poly_matmul([a.double() for a in A], [b.double() for b in B]), C0)]
    assert max(ref.plane_errors(out, want)) <= tol


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n", [1, 2, 3])
@pytest.mark.parametrize("layout", ["k", "rows"])
def test_all_planes_product(dtype, n, layout):
    """Degree <= 3 bf16 / f16 products with at least one 128 x 128 output tile per SM run the
    all-planes kernel (every output plane of a tile in tensor memory): plain, banded and
    accumulating, ragged M / N / K, K-major or MN-major operands."""
    from polytensors_b200 import _kernels

    batch, M, N, K = 10, 2000, 200, 200
    A = series((batch, M, K), n, 51, dtype)
    B = series((batch, K, N), n, 52, dtype)
    a = cuda(A) if layout == "k" else [x.transpose(1, 2).contiguous().cuda().transpose(1, 2) for x in A]
    b = cuda(B) if layout == "rows" else [x.transpose(1, 2).contiguous().cuda().transpose(1, 2) for x in B]
    check(A, B, 1e-2, got=_kernels.poly_matmul(a, b))
    # banded (k >= m - 1500: the first row tiles keep every k, later ones skip k blocks)
    keep = (torch.arange(K).view(1, K) >= torch.arange(M).view(M, 1) - 1500)
    Ab = [x * keep.to(x.dtype) for x in A]
    ab = cuda(Ab) if layout == "k" else [x.transpose(1, 2).contiguous().cuda().transpose(1, 2) for x in Ab]
    check(Ab, B, 1e-2, got=_kernels.poly_matmul(ab, b, band=1, band_offset=-1500))
    C0 = series((batch, M, N), n, 53, dtype)
    out = cuda(C0)
    _kernels.poly_matmul(a, b, out=out, accumulate=True)
    want = [w + c.double() for w, c in zip(ref.poly_matmul([x.double() for x in A], [y.double() for y in B]), C0)]
    assert max(ref.plane_errors(out, want)) <= 1e-2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("offset", [0, -200, 100])
def test_causal_output_band(dtype, offset):
    """Band 3: the outputs with n <= m + offset equal the plain product (others unspecified); the
    all-planes kernel (bf16 / f16 with enough tiles) and the per-plane kernel (float32)."""
    from polytensors_b200 import _kernels

    batch, M, N, K, n = 10, 1100, 900, 72, 2
    A, B = series((batch, M, K), n, 61, dtype), series((batch, K, N), n, 62, dtype)
    got = _kernels.poly_matmul(cuda(A), cuda(B), band=3, band_offset=offset)
    want = ref.poly_matmul([a.double() for a in A], [b.double() for b in B])
    keep = (torch.arange(N).view(1, N) <= torch.arange(M).view(M, 1) + offset)
    tol = {torch.bfloat16: 1e-2, torch.float16: 1e-2, torch.float32: 1e-4}[dtype]
    errs = ref.plane_errors([g.cpu().double() * keep for g in got], [w * keep for w in want])
    assert max(errs) <= tol, errs


@pytest.mark.parametrize("a_how", ["k", "rows", "odd"])
@pytest.mark.parametrize("b_how", ["k", "rows"])
def test_f32_operand_layouts(a_how, b_how):
    """float32 planes K-major, MN-major or at an odd offset are staged into bf16 hi/lo (direct or
    transposing staging kernels, the generic one for odd strides).  Batched, ragged tails, K not a
    multiple of 64, tolerance 1e-4."""
    from polytensors_b200 import _kernels

    batch, M, N, K, n = 3, 200, 296, 136, 3
    A = series((batch, M, K), n, 71)
    W = series((batch, N, K), n, 72)
    a = _layout(A, a_how)
    b = [w.transpose(-2, -1) for w in _layout(W, b_how)]
    got = _kernels.poly_matmul(a, b)
    check(A, [w.transpose(-2, -1) for w in W], TOL[torch.float32], got=got)


def test_empty_reduction_and_empty_output():
    from polytensors_b200 import _kernels

    A, B = series((5, 0), 2, 17), series((0, 7), 2, 18)
    got = _kernels.poly_matmul(cuda(A), cuda(B))
    assert all(torch.count_nonzero(g).item() == 0 and g.shape == (5, 7) for g in got)
    got = _kernels.poly_matmul(cuda(series((0, 4), 1, 19)), cuda(series((4, 3), 1, 20)))
    assert all(g.shape == (0, 3) for g in got)


def test_golden_vectors(golden):
    from polytensors_b200 import _kernels

    for name, tol in (("matmul_f64_n2", 1e-10), ("matmul_f64_n4", 1e-10), ("matmul_f32_n4", 1e-4),
                      ("bmm_f64_n3", 1e-10), ("matmul_c128_n2", 1e-10)):
        g = golden(name)
        got = _kernels.poly_matmul(cuda(g["A"]), cuda(g["B"]))
        errs = ref.plane_errors(got, g["C"])
        assert max(errs) <= tol, (name, errs)


@pytest.mark.parametrize("shape,n", [((4, 1000), 3), ((7, 13), 0), ((3, 5, 1023), 5), ((1,), 2)])
def test_split_hilo_kernel_is_bit_exact(shape, n):
    """pk_split_hilo: hi = bf16(x), lo = bf16(x - hi), round to nearest, bit for bit against the
    same split done with torch conversions (vector and element-by-element tails, odd sizes, a
    non-contiguous input made contiguous first)."""
    from polytensors_b200 import _kernels

    g = torch.Generator().manual_seed(sum(shape) + n)
    planes = [(torch.randn(*shape, generator=g) * 10 ** (k - 2)).cuda() for k in range(n + 1)]
    if len(shape) > 1:
        planes = [p.transpose(0, -1) for p in planes]
    got = _kernels.split_hilo(planes)
    assert len(got) == 2 * len(planes)
    for k, x in enumerate(planes):
        hi = x.to(torch.bfloat16)
        lo = (x - hi.float()).to(torch.bfloat16)
        assert got[2 * k].shape == x.shape and got[2 * k].dtype == torch.bfloat16
        assert torch.equal(got[2 * k].view(torch.int16), hi.contiguous().view(torch.int16))
        assert torch.equal(got[2 * k + 1].view(torch.int16), lo.contiguous().view(torch.int16))


def test_device_status_clean():
    from polytensors_b200 import _lib

    assert _lib.load().pk_device_status(1) == 0


@pytest.mark.parametrize("M,N,K,n,a_mn,b_mn", [(256, 192, 320, 3, False, False), (200, 136, 512, 3, True, False),
                                               (384, 64, 1000, 2, True, True), (130, 264, 256, 1, False, True)])
def test_hilo_product_reads_presplit_operands(M, N, K, n, a_mn, b_mn):
    """pk_poly_gemm_hilo: A (and B) given as bf16 hi/lo planes, k-contiguous or rows-contiguous
    (MN-major), read in place; against the float32 product of the same values (hi + lo) and the
    float64 oracle, plain and accumulated (tolerance 1e-4 of the plane max-norm)."""
    from gpu_util import assert_close
    from polytensors_b200 import _kernels as K_

    A = [a.cuda() for a in series((M, K), n, 71, torch.float32)]
    B = [b.cuda() for b in series((K, N), n, 72, torch.float32)]
    Ahl, Bhl = K_.split_hilo(A), K_.split_hilo(B)
    if a_mn:
        Ahl = [t.t().contiguous().t() for t in Ahl]
    if b_mn:
        Bhl = [t.t().contiguous().t() for t in Bhl]
    # the values the pre-split operands carry exactly
    A2 = [Ahl[2 * k].float() + Ahl[2 * k + 1].float() for k in range(n + 1)]
    B2 = [Bhl[2 * k].float() + Bhl[2 * k + 1].float() for k in range(n + 1)]
    want = ref.poly_matmul([a.cpu().double() for a in A2], [b.cpu().double() for b in B2])
    for a_args, b_args in (((Ahl, True), (B, False)), ((A, False), (Bhl, True)), ((Ahl, True), (Bhl, True))):
        got = K_.poly_matmul_hilo(*a_args, *b_args)
        assert_close([g.cpu() for g in got], want, 1e-4, f"hilo {a_args[1]} {b_args[1]}")
    C = [torch.ones(M, N, device="cuda") for _ in range(n + 1)]
    K_.poly_matmul_hilo(Ahl, True, Bhl, True, out=C, accumulate=True)
    assert_close([c.cpu() for c in C], [w + 1 for w in want], 1e-4, "accumulate")
