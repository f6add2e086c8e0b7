"""Tensor-level wrappers around the libpolykern C ABI.

Each function takes coefficient planes as CUDA tensors, allocates outputs (and any
workspace) with the PyTorch caching allocator, and enqueues the kernel on the current
CUDA stream.  Unsupported inputs raise ``NotImplementedError``; there is no CPU or
eager-PyTorch fallback.
"""

import ctypes

import torch

from . import _lib

_DTYPE_CODE = {torch.float32: _lib.PK_F32, torch.float64: _lib.PK_F64,
               torch.bfloat16: _lib.PK_BF16, torch.float16: _lib.PK_F16}


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(tensors, what):
    for t in tensors:
        if not t.is_cuda:
            raise NotImplementedError(f"{what}: the polykern kernels need CUDA tensors (no CPU path)")


def _uniform(planes):
    """Planes sharing one stride pattern (the C ABI takes one set of strides per operand)."""
    strides = planes[0].stride()
    if all(p.stride() == strides for p in planes):
        return list(planes)
    return [p.contiguous() for p in planes]


def _complex_from(planes):
    for k, p in enumerate(planes):
        if p.is_complex():
            return k
    return len(planes)


def gemm_dtype(a_planes, b_planes):
    """(dtype code, a_complex_from, b_complex_from, output dtypes) or None if unsupported."""
    P = len(a_planes)
    base = a_planes[0].dtype
    if any(p.dtype != base for p in (*a_planes, *b_planes)):
        # real float64 base with complex128 directions on either operand
        ok = all(p.dtype in (torch.float64, torch.complex128) for p in (*a_planes, *b_planes))
        if not ok or a_planes[0].dtype != torch.float64 or b_planes[0].dtype != torch.float64:
            return None
        acf, bcf = _complex_from(a_planes), _complex_from(b_planes)
        if any(p.dtype != torch.complex128 for p in a_planes[acf:]) or \
           any(p.dtype != torch.complex128 for p in b_planes[bcf:]):
            return None
        outs = [torch.complex128 if (k >= acf or k >= bcf) else torch.float64 for k in range(P)]
        return _lib.PK_C128, acf, bcf, outs
    if base not in _DTYPE_CODE:
        return None
    return _DTYPE_CODE[base], P, P, [base] * P


def _band_count(M, K, band, off):
    """Admissible (row, column) pairs of an M x K band: 1: k >= m + off, 2: k <= m + off."""
    m = torch.arange(M, dtype=torch.int64)
    if band == 1:
        return int((K - (m + off).clamp(0, K)).sum())
    return int((m + off + 1).clamp(0, K).sum())


def product_flops(code, degree, batch, M, N, K, acf, bcf, band=0, band_offset=0):
    """Algorithmic flops of one polynomial product: 2*M*N*K per real plane product over the
    (n+1)(n+2)/2 products; a complex128 plane product counts 4 real products (2 when one side
    is real), and banded products count only their admissible region."""
    P = degree + 1
    terms = 0
    for k in range(P):
        for i in range(k + 1):
            if code == _lib.PK_C128:
                ca, cb = i >= acf, (k - i) >= bcf
                terms += 4 if (ca and cb) else (2 if (ca or cb) else 1)
            else:
                terms += 1
    if band in (1, 2):
        pairs = _band_count(M, K, band, band_offset) * N
    elif band == 3:
        pairs = _band_count(M, N, 2, band_offset) * K
    else:
        pairs = M * N * K
    return 2.0 * batch * pairs * terms


def poly_matmul(a_planes, b_planes, out=None, accumulate=False, band=0, band_offset=0):
    """C_k = sum_{i+j=k} A_i @ B_j for planes of shape (M, K) x (K, N) or (B, M, K) x (B, K, N).

    Mirrors plain_polynomial_product(matrix=True) (src/polytensors/_plain.py:118-128)
    including real-base / complex-direction promotion (src/polytensors/_plain.py:77-80).
    ``out``: optional output planes (views with unit column stride) written in place;
    ``accumulate``: add the product to ``out`` (C_k += ...) as addmm with beta = 1 does.
    ``band``/``band_offset``: A is zero outside a band (1: k >= m + offset, 2: k <= m + offset), as
    in causal attention, and k blocks outside it are skipped; or (3) only the outputs with
    n <= m + offset are wanted, the rest being unspecified (pk_poly_gemm_banded).
    """
    P = len(a_planes)
    if P != len(b_planes) or P == 0:
        raise ValueError("poly_matmul: operands must have the same number of planes")
    if P > _lib.PK_MAX_PLANES:
        raise NotImplementedError(f"poly_matmul: degree {P - 1} exceeds the kernel limit {_lib.PK_MAX_PLANES - 1}")
    _require_cuda((*a_planes, *b_planes), "poly_matmul")
    spec = gemm_dtype(a_planes, b_planes)
    if spec is None:
        raise NotImplementedError(f"poly_matmul: unsupported plane dtypes "
                                  f"{[p.dtype for p in a_planes]} x {[p.dtype for p in b_planes]}")
    code, acf, bcf, out_dtypes = spec
    a_planes, b_planes = _uniform(a_planes), _uniform(b_planes)
    a0, b0 = a_planes[0], b_planes[0]
    if a0.dim() != b0.dim() or a0.dim() not in (2, 3):
        raise NotImplementedError("poly_matmul: expected 2-D or batched 3-D planes")
    batched = a0.dim() == 3
    if batched:
        batch, M, K = a0.shape
        if b0.shape[0] != batch:
            raise ValueError("poly_matmul: batch sizes differ")
        N = b0.shape[2]
        a_bs, a_rs, a_cs = a0.stride()
        b_bs, b_rs, b_cs = b0.stride()
    else:
        batch, (M, K), N = 1, a0.shape, b0.shape[1]
        a_bs, (a_rs, a_cs) = 0, a0.stride()
        b_bs, (b_rs, b_cs) = 0, b0.stride()
    if b0.shape[-2] != K:
        raise ValueError(f"poly_matmul: inner dimensions differ ({K} vs {b0.shape[-2]})")
    shape = (batch, M, N) if batched else (M, N)
    if out is None:
        if accumulate:
            raise ValueError("poly_matmul: accumulate needs output planes")
        outs = [torch.empty(shape, dtype=dt, device=a0.device) for dt in out_dtypes]
        c_bs, c_rs = (M * N, N)
    else:
        outs = list(out)
        if len(outs) != P or any(tuple(o.shape) != shape or o.dtype != dt or o.stride() != outs[0].stride()
                                 for o, dt in zip(outs, out_dtypes)):
            raise ValueError("poly_matmul: output planes must match the product's shape, dtypes and strides")
        st = outs[0].stride()
        if st[-1] != 1:
            raise NotImplementedError("poly_matmul: output planes need unit column stride")
        c_bs, c_rs = (st[0], st[1]) if batched else (0, st[0])
    lib = _lib.load()
    degree = P - 1
    if _lib.profiling():
        _lib.add_gemm_flops(product_flops(code, degree, batch, M, N, K, acf, bcf, band, band_offset))
    pa, ka = _lib.pointer_array(a_planes)
    pb, kb = _lib.pointer_array(b_planes)
    pc, kc = _lib.pointer_array(outs)
    ws_bytes = ctypes.c_size_t(0)
    _lib.check(lib.pk_poly_gemm_workspace_query(code, degree, batch, M, N, K, pa, a_bs, a_rs, a_cs,
                                                pb, b_bs, b_rs, b_cs, acf, bcf, ctypes.byref(ws_bytes)),
               "pk_poly_gemm_workspace_query")
    ws = torch.empty(ws_bytes.value, dtype=torch.uint8, device=a0.device) if ws_bytes.value else None
    ws_ptr, ws_n = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
    if band:
        status = lib.pk_poly_gemm_banded(code, degree, batch, M, N, K, pa, a_bs, a_rs, a_cs, pb, b_bs, b_rs, b_cs,
                                         pc, c_bs, c_rs, acf, bcf, 1 if accumulate else 0, int(band),
                                         int(band_offset), ws_ptr, ws_n, _stream(a0.device))
        _lib.check(status, "pk_poly_gemm_banded")
        return outs
    fn = lib.pk_poly_gemm_accumulate if accumulate else lib.pk_poly_gemm
    status = fn(code, degree, batch, M, N, K, pa, a_bs, a_rs, a_cs, pb, b_bs, b_rs, b_cs, pc, c_bs, c_rs,
                acf, bcf, ws_ptr, ws_n, _stream(a0.device))
    _lib.check(status, "pk_poly_gemm_accumulate" if accumulate else "pk_poly_gemm")
    return outs


def split_hilo(planes):
    """float32 planes -> [hi_0, lo_0, hi_1, lo_1, ...] bfloat16 planes with x ~= hi + lo (the
    operand form pk_poly_gemm_hilo reads in place)."""
    planes = [x if x.is_contiguous() else x.contiguous() for x in planes]
    _require_cuda(planes, "split_hilo")
    if any(x.dtype != torch.float32 for x in planes) or len(planes) > _lib.PK_MAX_PLANES:
        raise NotImplementedError("split_hilo: float32 planes, degree <= 15")
    out = [torch.empty_like(planes[i // 2], dtype=torch.bfloat16) for i in range(2 * len(planes))]
    px, k1 = _lib.pointer_array(planes)
    po, k2 = _lib.pointer_array(out)
    _lib.check(_lib.load().pk_split_hilo(len(planes) - 1, planes[0].numel(), px, po, _stream(planes[0].device)),
               "pk_split_hilo")
    return out


def poly_matmul_hilo(a, a_hilo, b, b_hilo, out=None, accumulate=False, band=0, band_offset=0):
    """float32 polynomial product (pk_poly_gemm_hilo) whose operands are float32 planes (n+1) or,
    with ``*_hilo``, pre-split bf16 planes [hi_0, lo_0, ...] (2(n+1)) read in place.  Shapes
    (M, K) x (K, N) or batched (B, M, K) x (B, K, N); returns / fills float32 output planes."""
    P = len(a) // (2 if a_hilo else 1)
    if P != len(b) // (2 if b_hilo else 1) or P == 0:
        raise ValueError("poly_matmul_hilo: operands must have the same degree")
    _require_cuda((*a, *b), "poly_matmul_hilo")
    for planes, hilo in ((a, a_hilo), (b, b_hilo)):
        want = torch.bfloat16 if hilo else torch.float32
        if any(t.dtype != want for t in planes):
            raise NotImplementedError(f"poly_matmul_hilo: expected {want} planes")
    a, b = _uniform(a), _uniform(b)
    a0, b0 = a[0], b[0]
    batched = a0.dim() == 3
    if batched:
        batch, M, K = a0.shape
        N = b0.shape[2]
        (a_bs, a_rs, a_cs), (b_bs, b_rs, b_cs) = a0.stride(), b0.stride()
    else:
        batch, (M, K), N = 1, a0.shape, b0.shape[1]
        a_bs, (a_rs, a_cs) = 0, a0.stride()
        b_bs, (b_rs, b_cs) = 0, b0.stride()
    shape = (batch, M, N) if batched else (M, N)
    if out is None:
        if accumulate:
            raise ValueError("poly_matmul_hilo: accumulate needs output planes")
        outs = [torch.empty(shape, dtype=torch.float32, device=a0.device) for _ in range(P)]
    else:
        outs = list(out)
        if any(tuple(o.shape) != shape or o.dtype != torch.float32 or o.stride() != outs[0].stride() for o in outs):
            raise ValueError("poly_matmul_hilo: output planes must match the product's shape and strides")
        if outs[0].stride(-1) != 1:
            raise NotImplementedError("poly_matmul_hilo: output planes need unit column stride")
    st = outs[0].stride()
    c_bs, c_rs = (st[0], st[1]) if batched else (0, st[0])
    lib = _lib.load()
    if _lib.profiling():
        _lib.add_gemm_flops(product_flops(_lib.PK_F32, P - 1, batch, M, N, K, P, P, band, band_offset))
    pa, ka = _lib.pointer_array(a)
    pb, kb = _lib.pointer_array(b)
    pc, kc = _lib.pointer_array(outs)
    ws_bytes = ctypes.c_size_t(0)
    _lib.check(lib.pk_poly_gemm_hilo_workspace_query(P - 1, batch, M, N, K, pa, a_bs, a_rs, a_cs, int(a_hilo),
                                                     pb, b_bs, b_rs, b_cs, int(b_hilo), ctypes.byref(ws_bytes)),
               "pk_poly_gemm_hilo_workspace_query")
    ws = torch.empty(ws_bytes.value, dtype=torch.uint8, device=a0.device) if ws_bytes.value else None
    status = lib.pk_poly_gemm_hilo(P - 1, batch, M, N, K, pa, a_bs, a_rs, a_cs, int(a_hilo), pb, b_bs, b_rs, b_cs,
                                   int(b_hilo), pc, c_bs, c_rs, 1 if accumulate else 0, int(band), int(band_offset),
                                   ws.data_ptr() if ws is not None else None, ws_bytes.value, _stream(a0.device))
    _lib.check(status, "pk_poly_gemm_hilo")
    return outs


# ------------------------------------------------------------------------------------
# elementwise series operations, reductions, gathers

def dtype_code(dtype):
    code = _DTYPE_CODE.get(dtype)
    if code is None:
        raise NotImplementedError(f"polykern: coefficient dtype {dtype} is not supported by the kernels")
    return code


def _same_strides(planes):
    s = planes[0].stride()
    return all(p.stride() == s for p in planes)


def _collapse(shape, *stride_sets):
    """Merge adjacent dimensions that are contiguous with each other in every operand."""
    dims = [(shape[d], [st[d] for st in stride_sets]) for d in range(len(shape)) if shape[d] != 1]
    if not dims:
        return [1], [[0] for _ in stride_sets]
    out = [dims[0]]
    for size, strides in dims[1:]:
        psize, pstrides = out[-1]
        if all(ps == s * size for ps, s in zip(pstrides, strides)):
            out[-1] = (psize * size, strides)
        else:
            out.append((size, strides))
    return [d[0] for d in out], [[d[1][i] for d in out] for i in range(len(stride_sets))]


def series_map(op, degree, a, b=None, p0=0.0, p1=0.0, out=None):
    """One elementwise series operation over all planes (pk_series_map).

    ``a``/``b`` are lists of planes (degree+1 planes, or 1 plane for a constant operand);
    they broadcast against each other.  Returns the ``out`` planes (allocated contiguous
    when not given; an in-place update passes ``out=a``)."""
    np_ = degree + 1
    if np_ > _lib.PK_MAX_PLANES:
        raise NotImplementedError(f"polykern: degree {degree} exceeds {_lib.PK_MAX_PLANES - 1}")
    opcode = _lib.OP[op]
    planes = list(a) + (list(b) if b is not None else []) + (list(out) if out is not None else [])
    _require_cuda(planes, f"series {op}")
    if any(x.is_complex() for x in planes):
        return _series_map_complex(op, degree, a, b, p0, p1, out)
    dtype = a[0].dtype
    code = dtype_code(dtype)
    shape = a[0].shape if b is None else torch.broadcast_shapes(a[0].shape, b[0].shape)
    if out is not None:
        shape = out[0].shape
    a = [x.expand(shape) for x in a]
    if not _same_strides(a):
        a = [x.contiguous() for x in a]
    if b is not None:
        b = [x.to(dtype).expand(shape) for x in b]
        if not _same_strides(b):
            b = [x.contiguous() for x in b]
    if out is None:
        out = [torch.empty(shape, dtype=dtype, device=a[0].device) for _ in range(np_)]
    elif not _same_strides(out):
        raise NotImplementedError("series update into planes with differing layouts")
    if any(o.dtype != dtype for o in out):
        raise NotImplementedError("series update into planes of another dtype")
    if out[0].numel() == 0:
        return out
    sets = [out[0].stride(), a[0].stride()] + ([b[0].stride()] if b is not None else [])
    cshape, cstrides = _collapse(list(shape), *sets)
    if len(cshape) > 6:
        raise NotImplementedError("series operation on more than 6 non-mergeable dimensions")
    shp, ks = _lib.int64_array(cshape)
    so, k1 = _lib.int64_array(cstrides[0])
    sa, k2 = _lib.int64_array(cstrides[1])
    sb, k3 = _lib.int64_array(cstrides[2] if b is not None else [0] * len(cshape))
    po, kp1 = _lib.pointer_array(out)
    pa, kp2 = _lib.pointer_array(a)
    pb, kp3 = _lib.pointer_array(b if b is not None else [None])
    status = _lib.load().pk_series_map(opcode, code, degree, len(cshape), shp, po, so, pa, len(a), sa,
                                        pb if b is not None else None, len(b) if b is not None else 0, sb,
                                        float(p0), float(p1), _stream(a[0].device))
    _lib.check(status, f"pk_series_map({op})")
    return out


# operations whose output plane k depends only on the input planes k (the others mix lower planes in)
_PLANEWISE_OPS = ("copy", "affine", "add")
# operations whose base function is evaluated on the real part only (real base required)
_REAL_BASE_OPS = {"tanh": 0, "gelu": 0, "gelu_bwd": 1}


def _series_map_complex(op, degree, a, b, p0, p1, out):
    """series_map on series with complex planes (pk_series_map_complex): a real base with complex
    directions, or complex throughout.  Planes are brought to one precision (float64/complex128 if
    any plane is double, else float32/complex64); an output plane is complex when an input plane
    it depends on is (the same plane for add/affine/copy, any plane up to it otherwise), which for
    series built by the constructor (all directions one dtype) is the reference's per-plane
    result-type rule."""
    np_ = degree + 1
    ops_in = [list(a)] + ([list(b)] if b is not None else [])
    every = [p for grp in ops_in for p in grp] + (list(out) if out is not None else [])
    if any(p.dtype not in (torch.float32, torch.float64, torch.complex64, torch.complex128) for p in every):
        raise NotImplementedError(f"series {op} with complex planes: float32/float64 (complex64/complex128) only")
    if op in _REAL_BASE_OPS and ops_in[_REAL_BASE_OPS[op]][0].is_complex():
        raise NotImplementedError(f"series {op}: a complex base (plane 0) is not supported; complex directions are")
    wide = any(p.dtype in (torch.float64, torch.complex128) for p in every)
    real_t, cplx_t = (torch.float64, torch.complex128) if wide else (torch.float32, torch.complex64)
    conv = [[p.to(cplx_t if p.is_complex() else real_t) for p in grp] for grp in ops_in]
    shape = conv[0][0].shape if b is None else torch.broadcast_shapes(conv[0][0].shape, conv[1][0].shape)
    if out is not None:
        shape = out[0].shape
    conv = [[p.expand(shape) for p in grp] for grp in conv]
    conv = [grp if _same_strides(grp) else [p.contiguous() for p in grp] for grp in conv]
    if out is None:
        dtypes = []
        for k in range(np_):
            lo = k if op in _PLANEWISE_OPS else 0
            dep = [p for grp in conv for j, p in enumerate(grp) if lo <= j <= k]
            dtypes.append(cplx_t if any(p.is_complex() for p in dep) else real_t)
        out = [torch.empty(shape, dtype=dt, device=conv[0][0].device) for dt in dtypes]
    else:
        out = list(out)
        if any(o.dtype not in (real_t, cplx_t) for o in out) or not _same_strides(out):
            raise NotImplementedError(f"series {op}: in-place update into planes of another precision or layout")
        for k, o in enumerate(out):
            lo = k if op in _PLANEWISE_OPS else 0
            if not o.is_complex() and any(p.is_complex() for grp in conv for j, p in enumerate(grp) if lo <= j <= k):
                raise RuntimeError("cannot copy complex PolyTensor coefficients into real coefficient storage")
    if out[0].numel() == 0:
        return out

    def mask(grp):
        return sum(1 << k for k, p in enumerate(grp) if p.is_complex())

    sets = [out[0].stride()] + [grp[0].stride() for grp in conv]
    cshape, cstrides = _collapse(list(shape), *sets)
    if len(cshape) > 6:
        raise NotImplementedError("series operation on more than 6 non-mergeable dimensions")
    shp, ks = _lib.int64_array(cshape)
    so, k1 = _lib.int64_array(cstrides[0])
    sa, k2 = _lib.int64_array(cstrides[1])
    sb, k3 = _lib.int64_array(cstrides[2] if b is not None else [0] * len(cshape))
    po, kp1 = _lib.pointer_array(out)
    pa, kp2 = _lib.pointer_array(conv[0])
    pb, kp3 = _lib.pointer_array(conv[1] if b is not None else [None])
    status = _lib.load().pk_series_map_complex(
        _lib.OP[op], _lib.PK_F64 if wide else _lib.PK_F32, degree, len(cshape), shp, po, so, mask(out),
        pa, len(conv[0]), sa, mask(conv[0]), pb if b is not None else None, len(conv[1]) if b is not None else 0,
        sb, mask(conv[1]) if b is not None else 0, float(p0), float(p1), _stream(conv[0][0].device))
    _lib.check(status, f"pk_series_map_complex({op})")
    return out


def attn_dsum(dO, O):
    """(sum_d dO (*) O) per row of (rows..., D) planes: a (rows, n+1) table in the compute dtype
    (pk_attn_dsum)."""
    cols = O[0].shape[-1]
    g = [p.reshape(-1, cols) if p.dtype == O[0].dtype else p.to(O[0].dtype).reshape(-1, cols) for p in dO]
    o = [p.reshape(-1, cols) for p in O]
    if not _same_strides(g) or g[0].stride(-1) != 1:
        g = [p.contiguous() for p in g]
    if not _same_strides(o) or o[0].stride(-1) != 1:
        o = [p.contiguous() for p in o]
    _require_cuda((*g, *o), "attention dsum")
    out = torch.empty(g[0].shape[0], len(g), dtype=compute_dtype(g[0].dtype), device=g[0].device)
    pg, k1 = _lib.pointer_array(g)
    po, k2 = _lib.pointer_array(o)
    status = _lib.load().pk_attn_dsum(dtype_code(g[0].dtype), len(g) - 1, g[0].shape[0], cols, pg, g[0].stride(0),
                                      po, o[0].stride(0), out.data_ptr(), _stream(g[0].device))
    _lib.check(status, "pk_attn_dsum")
    return out


def series_reduce(planes, outer, red, inner, scale=1.0):
    """out[o, i] = scale * sum_r x[o, r, i] for contiguous planes viewed as (outer, red, inner)."""
    x = [p.contiguous() for p in planes]
    _require_cuda(x, "series reduction")
    code = dtype_code(x[0].dtype)
    out = [torch.empty(outer * inner, dtype=x[0].dtype, device=x[0].device) for _ in x]
    px, k1 = _lib.pointer_array(x)
    po, k2 = _lib.pointer_array(out)
    status = _lib.load().pk_series_reduce(code, len(x) - 1, outer, red, inner, px, po, float(scale),
                                          _stream(x[0].device))
    _lib.check(status, "pk_series_reduce")
    return out


def _check_indices(idx, upper, what, ignore=None):
    """Raise IndexError, as the reference's torch ops do, when an index lies outside
    [0, upper) (``ignore`` is an allowed sentinel, e.g. cross entropy's ignore_index).
    The kernels skip such rows instead of faulting, so the check runs on the host side
    before the launch: one reduction over the indices and one read of its result."""
    if idx.numel() == 0:
        return
    bad = (idx < 0) | (idx >= upper)
    if ignore is not None:
        bad &= idx != ignore
    if bool(bad.any()):
        first = idx[bad].reshape(-1)[0].item()
        raise IndexError(f"{what}: index {first} is out of range [0, {upper})")


def _as_real_rows(planes, fn):
    """Row gathers and scatters move whole rows, so a complex plane goes through as a real plane of
    twice the width ((re, im) pairs); real and complex planes run as separate groups."""
    out = [None] * len(planes)
    for is_c in (False, True):
        idx = [i for i, p in enumerate(planes) if p.is_complex() == is_c]
        if not idx:
            continue
        group = [torch.view_as_real(planes[i].contiguous()).flatten(-2) if is_c else planes[i] for i in idx]
        for i, r in zip(idx, fn(group)):
            out[i] = torch.view_as_complex(r.unflatten(-1, (-1, 2))) if is_c else r
    return out


def gather_rows(weight_planes, idx):
    """out[i, :] = W[idx[i], :] per plane (embedding)."""
    if any(p.is_complex() for p in weight_planes):
        return _as_real_rows(list(weight_planes), lambda g: gather_rows(g, idx))
    _check_indices(idx, weight_planes[0].shape[0], "embedding")
    w = weight_planes if _same_strides(weight_planes) and weight_planes[0].stride(-1) == 1 else \
        [p.contiguous() for p in weight_planes]
    _require_cuda((*w, idx), "embedding")
    V, d = w[0].shape
    flat = idx.reshape(-1).to(torch.int64).contiguous()
    out = [torch.empty(flat.numel(), d, dtype=w[0].dtype, device=w[0].device) for _ in w]
    pw, k1 = _lib.pointer_array(w)
    po, k2 = _lib.pointer_array(out)
    status = _lib.load().pk_series_gather_rows(dtype_code(w[0].dtype), len(w) - 1, flat.numel(), d,
                                               flat.data_ptr(), pw, w[0].stride(0), V, po, _stream(w[0].device))
    _lib.check(status, "pk_series_gather_rows")
    return [o.view(*idx.shape, d) for o in out]


def scatter_add_rows(grad_planes, idx, num_rows, padding_idx=-1):
    """out[idx[i], :] += G[i, :] over zeroed (num_rows, d) planes (embedding backward)."""
    if any(p.is_complex() for p in grad_planes):
        return _as_real_rows(list(grad_planes), lambda g: scatter_add_rows(g, idx, num_rows, padding_idx))
    _check_indices(idx, num_rows, "embedding backward")
    d = grad_planes[0].shape[-1]
    g = [p.reshape(-1, d) for p in grad_planes]
    if not _same_strides(g) or g[0].stride(-1) != 1:
        g = [p.contiguous() for p in g]
    flat = idx.reshape(-1).to(torch.int64).contiguous()
    _require_cuda((*g, flat), "embedding backward")
    out = [torch.empty(num_rows, d, dtype=g[0].dtype, device=g[0].device) for _ in g]
    pg, k1 = _lib.pointer_array(g)
    po, k2 = _lib.pointer_array(out)
    status = _lib.load().pk_series_scatter_add_rows(dtype_code(g[0].dtype), len(g) - 1, flat.numel(), d,
                                                    flat.data_ptr(), padding_idx, pg, g[0].stride(0), num_rows,
                                                    po, _stream(g[0].device))
    _lib.check(status, "pk_series_scatter_add_rows")
    return out


# ------------------------------------------------------------------------------------
# row-wise kernels: planes viewed as (rows, cols) with contiguous rows

def _rows(planes, cols):
    x = [p.reshape(-1, cols) if p.is_contiguous() else p.contiguous().view(-1, cols) for p in planes]
    if not _same_strides(x) or x[0].stride(-1) != 1:
        x = [p.contiguous() for p in x]
    return x


def compute_dtype(dtype):
    return torch.float64 if dtype == torch.float64 else torch.float32


def rmsnorm_fwd(x_planes, cols, w_planes, eps):
    x = _rows(x_planes, cols)
    _require_cuda(x, "rms_norm")
    code = dtype_code(x[0].dtype)
    rows = x[0].shape[0]
    y = [torch.empty_like(p) for p in x]
    rstd = torch.empty(rows, len(x), dtype=compute_dtype(x[0].dtype), device=x[0].device)
    w = None
    if w_planes is not None:
        w = [p.to(x[0].dtype).reshape(-1).contiguous() for p in w_planes]
    px, k1 = _lib.pointer_array(x)
    pw, k2 = _lib.pointer_array(w) if w is not None else (None, None)
    py, k3 = _lib.pointer_array(y)
    status = _lib.load().pk_rmsnorm_fwd(code, len(x) - 1, rows, cols, px, x[0].stride(0), pw,
                                        len(w) if w is not None else 0, float(eps), py, y[0].stride(0),
                                        rstd.data_ptr(), _stream(x[0].device))
    _lib.check(status, "pk_rmsnorm_fwd")
    return [t.view(x_planes[0].shape) for t in y], rstd


def rmsnorm_bwd(x_planes, cols, w_planes, g_planes, rstd, want_dw):
    x = _rows(x_planes, cols)
    g = _rows([p.to(x[0].dtype).expand(x_planes[0].shape) for p in g_planes], cols)
    code = dtype_code(x[0].dtype)
    rows = x[0].shape[0]
    dx = [torch.empty_like(p) for p in x]
    w = None
    if w_planes is not None:
        w = [p.to(x[0].dtype).reshape(-1).contiguous() for p in w_planes]
    dw = [torch.empty(cols, dtype=x[0].dtype, device=x[0].device) for _ in x] if want_dw else None
    lib = _lib.load()
    ws = None
    if want_dw:
        ws = torch.empty(lib.pk_rmsnorm_bwd_workspace_size(code, len(x) - 1, rows, cols), dtype=torch.uint8,
                         device=x[0].device)
    px, k1 = _lib.pointer_array(x)
    pw, k2 = _lib.pointer_array(w) if w is not None else (None, None)
    pg, k3 = _lib.pointer_array(g)
    pdx, k4 = _lib.pointer_array(dx)
    pdw, k5 = _lib.pointer_array(dw) if dw is not None else (None, None)
    status = lib.pk_rmsnorm_bwd(code, len(x) - 1, rows, cols, px, x[0].stride(0), pw,
                                len(w) if w is not None else 0, pg, g[0].stride(0), rstd.data_ptr(), pdx,
                                dx[0].stride(0), pdw, ws.data_ptr() if ws is not None else None,
                                ws.numel() if ws is not None else 0, _stream(x[0].device))
    _lib.check(status, "pk_rmsnorm_bwd")
    return [t.view(x_planes[0].shape) for t in dx], dw


def softmax_fwd(x_planes, log):
    """Softmax (or log-softmax) series along the last dimension."""
    cols = x_planes[0].shape[-1]
    x = _rows(x_planes, cols)
    _require_cuda(x, "softmax")
    y = [torch.empty_like(p) for p in x]
    px, k1 = _lib.pointer_array(x)
    py, k2 = _lib.pointer_array(y)
    status = _lib.load().pk_softmax_fwd(dtype_code(x[0].dtype), len(x) - 1, x[0].shape[0], cols, px,
                                        x[0].stride(0), 1 if log else 0, py, y[0].stride(0), _stream(x[0].device))
    _lib.check(status, "pk_softmax_fwd")
    return [t.view(x_planes[0].shape) for t in y]


def softmax_bwd(g_planes, y_planes, log):
    cols = y_planes[0].shape[-1]
    y = _rows(y_planes, cols)
    g = _rows([p.to(y[0].dtype).expand(y_planes[0].shape) for p in g_planes], cols)
    _require_cuda((*y, *g), "softmax backward")
    dx = [torch.empty_like(p) for p in y]
    pg, k1 = _lib.pointer_array(g)
    py, k2 = _lib.pointer_array(y)
    pd, k3 = _lib.pointer_array(dx)
    status = _lib.load().pk_softmax_bwd(dtype_code(y[0].dtype), len(y) - 1, y[0].shape[0], cols, pg,
                                        g[0].stride(0), py, y[0].stride(0), 1 if log else 0, pd, dx[0].stride(0),
                                        _stream(y[0].device))
    _lib.check(status, "pk_softmax_bwd")
    return [t.view(y_planes[0].shape) for t in dx]


def cross_entropy_fwd(z_planes, target, ignore_index, softcap):
    """Per-row loss series (float32, or float64 for float64 logits) and row statistics."""
    rows, cols = z_planes[0].shape
    _check_indices(target, cols, "cross_entropy target", ignore=int(ignore_index))
    z = z_planes if (_same_strides(z_planes) and z_planes[0].stride(-1) == 1) else [p.contiguous() for p in z_planes]
    t = target.to(torch.int64).contiguous()
    _require_cuda((*z, t), "cross_entropy")
    cdt = compute_dtype(z[0].dtype)
    loss = [torch.empty(rows, dtype=cdt, device=z[0].device) for _ in z]
    stats = torch.empty(rows, len(z), dtype=cdt, device=z[0].device)
    pz, k1 = _lib.pointer_array(z)
    pl, k2 = _lib.pointer_array(loss)
    status = _lib.load().pk_cross_entropy_fwd(dtype_code(z[0].dtype), len(z) - 1, rows, cols, pz, z[0].stride(0),
                                              t.data_ptr(), int(ignore_index), float(softcap or 0.0), pl,
                                              stats.data_ptr(), _stream(z[0].device))
    _lib.check(status, "pk_cross_entropy_fwd")
    return loss, stats


def cross_entropy_bwd(z_planes, target, ignore_index, softcap, stats, g_planes):
    rows, cols = z_planes[0].shape
    z = z_planes if (_same_strides(z_planes) and z_planes[0].stride(-1) == 1) else [p.contiguous() for p in z_planes]
    t = target.to(torch.int64).contiguous()
    cdt = stats.dtype
    g = [p.to(cdt).expand(rows).contiguous() for p in g_planes]
    dz = [torch.empty(rows, cols, dtype=z[0].dtype, device=z[0].device) for _ in z]
    pz, k1 = _lib.pointer_array(z)
    pg, k2 = _lib.pointer_array(g)
    pd, k3 = _lib.pointer_array(dz)
    status = _lib.load().pk_cross_entropy_bwd(dtype_code(z[0].dtype), len(z) - 1, rows, cols, pz, z[0].stride(0),
                                              t.data_ptr(), int(ignore_index), float(softcap or 0.0),
                                              stats.data_ptr(), pg, pd, cols, _stream(z[0].device))
    _lib.check(status, "pk_cross_entropy_bwd")
    return dz
