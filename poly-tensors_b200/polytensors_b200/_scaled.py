"""Extended-range (default-mode) series arithmetic on the GPU.

Outside ``PolyTensor.plain_range()`` the reference keeps, next to the public coefficient tensors, a
hidden copy of every coefficient as mantissa * 2**exponent (``ScaledTensor``,
src/polytensors/_scaled.py) and runs its range rules on it (src/polytensors/_range_ops.py:26-279,
src/polytensors/_range.py): results whose values leave the dtype's range stay finite in the hidden
copy, and only the public tensors over- or underflow.  This module is that mode for the range
operations on the kernels: each coefficient is a pair of device tensors, a float32 / float64
mantissa and an int32 exponent (``csrc/pk_scaled.cu``), attached to the PolyTensor it belongs to
with a snapshot of its coefficients' version counters (a write to a public coefficient invalidates
it, as in the reference).  Handled: add / sub / mul / div (series and constants, in place too),
exp (the base's exponential from its logarithm, the series in scaled arithmetic), neg, rsub,
reciprocal, mm / bmm / matmul / mv / dot / linear / addmm, sum / mean, views, clone,
detach and copy_.  Other operations run on the public coefficients (the hidden copy is not
carried through them).  Complex coefficients run on the public coefficients as well.
"""

import math

import torch

from . import _kernels as K
from . import _lib

NOT_HANDLED = object()
aten = torch.ops.aten


class SC:
    """One coefficient: mantissa (float32 / float64) and int32 exponent tensors of one shape."""

    __slots__ = ("m", "e")

    def __init__(self, m, e):
        self.m, self.e = m, e

    def map(self, fn):
        return SC(fn(self.m), fn(self.e))

    @property
    def shape(self):
        return self.m.shape


def _mdtype(dtype):
    return torch.float64 if dtype == torch.float64 else torch.float32


def from_planes(planes, base=0):
    """Public coefficient tensors -> normalised SC coefficients (pk_scaled_from), per dtype group."""
    K._require_cuda(planes, "extended-range series")
    out = [None] * len(planes)
    groups = {}
    for i, p in enumerate(planes):
        groups.setdefault(p.dtype, []).append(i)
    for dtype, idx in groups.items():
        xs = [planes[i].contiguous() for i in idx]
        md = _mdtype(dtype)
        ms = [torch.empty(x.shape, dtype=md, device=x.device) for x in xs]
        es = [torch.empty(x.shape, dtype=torch.int32, device=x.device) for x in xs]
        for chunk in range(0, len(xs), _lib.PK_MAX_PLANES):
            sl = slice(chunk, chunk + _lib.PK_MAX_PLANES)
            px, k1 = _lib.pointer_array(xs[sl])
            pm, k2 = _lib.pointer_array(ms[sl])
            pe, k3 = _lib.pointer_array(es[sl])
            _lib.check(_lib.load().pk_scaled_from(K.dtype_code(dtype), len(xs[sl]) - 1, xs[0].numel(), px, pm, pe,
                                                  int(base), K._stream(xs[0].device)), "pk_scaled_from")
        for i, m, e in zip(idx, ms, es):
            out[i] = SC(m, e)
    return out


def to_planes(scs, dtypes, offset=0):
    """SC coefficients -> public tensors of the given dtypes (pk_scaled_to: only this step can over-
    or underflow, as the reference's to_tensor)."""
    out = []
    for c, dt in zip(scs, dtypes):
        m, e = c.m.contiguous(), c.e.contiguous()
        if m.dtype == torch.float64 and dt != torch.float64:
            m = m.float()
        y = torch.empty(m.shape, dtype=dt, device=m.device)
        pm, k1 = _lib.pointer_array([m])
        pe, k2 = _lib.pointer_array([e])
        py, k3 = _lib.pointer_array([y])
        _lib.check(_lib.load().pk_scaled_to(K.dtype_code(dt), K.dtype_code(m.dtype), 0, m.numel(), pm, pe,
                                            int(offset), py, K._stream(m.device)), "pk_scaled_to")
        out.append(y)
    return out


def _cast(c, md):
    return c if c.m.dtype == md else SC(c.m.to(md), c.e)


def series_op(op, degree, A, B=None, p0=0.0, p1=0.0):
    """pk_scaled_series_map over SC coefficient lists (1 or degree+1 coefficients each; a single
    coefficient is a constant whose higher coefficients are zero)."""
    md = torch.float64 if any(c.m.dtype == torch.float64 for c in (A + (B or []))) else torch.float32
    A = [_cast(c, md) for c in A]
    B = [_cast(c, md) for c in B] if B is not None else None
    shape = A[0].shape if B is None else torch.broadcast_shapes(A[0].shape, B[0].shape)
    A = [c.map(lambda t: t.expand(shape).contiguous()) for c in A]
    if B is not None:
        B = [c.map(lambda t: t.expand(shape).contiguous()) for c in B]
    dev = A[0].m.device
    out = [SC(torch.empty(shape, dtype=md, device=dev), torch.empty(shape, dtype=torch.int32, device=dev))
           for _ in range(degree + 1)]
    if out[0].m.numel() == 0:
        return out
    n = max(1, math.prod(shape))
    shp, k0 = _lib.int64_array([n])
    st, k1 = _lib.int64_array([1])
    pom, k2 = _lib.pointer_array([c.m for c in out])
    poe, k3 = _lib.pointer_array([c.e for c in out])
    pam, k4 = _lib.pointer_array([c.m for c in A])
    pae, k5 = _lib.pointer_array([c.e for c in A])
    pbm, k6 = _lib.pointer_array([c.m for c in B] if B is not None else [None])
    pbe, k7 = _lib.pointer_array([c.e for c in B] if B is not None else [None])
    _lib.check(_lib.load().pk_scaled_series_map(
        _lib.OP[op], K.dtype_code(md), degree, 1, shp, pom, poe, st, pam, pae, len(A), st,
        pbm if B is not None else None, pbe if B is not None else None, len(B) if B is not None else 0, st,
        float(p0), float(p1), K._stream(dev)), f"pk_scaled_series_map({op})")
    return out


def reduce(scs, dims, keepdim, mean):
    """Sum / mean of SC coefficients over dims (pk_scaled_reduce; mean divides by the count)."""
    nd = scs[0].m.dim()
    shape = list(scs[0].shape)
    if nd == 0:
        return [SC(c.m.clone(), c.e.clone()) for c in scs]
    dims = list(range(nd)) if dims is None else sorted({d % nd for d in dims})
    red = math.prod(shape[d] for d in dims)
    keep = [d for d in range(nd) if d not in dims]
    outer = math.prod(shape[d] for d in keep)
    src = [c.map(lambda t: t.permute(*keep, *dims).contiguous()) for c in scs]
    md = src[0].m.dtype
    dev = src[0].m.device
    out = [SC(torch.empty(outer, dtype=md, device=dev), torch.empty(outer, dtype=torch.int32, device=dev))
           for _ in src]
    pm, k1 = _lib.pointer_array([c.m for c in src])
    pe, k2 = _lib.pointer_array([c.e for c in src])
    pom, k3 = _lib.pointer_array([c.m for c in out])
    poe, k4 = _lib.pointer_array([c.e for c in out])
    _lib.check(_lib.load().pk_scaled_reduce(K.dtype_code(md), len(src) - 1, outer, red, 1, pm, pe, pom, poe,
                                            K._stream(dev)), "pk_scaled_reduce")
    out_shape = [1 if d in dims else s for d, s in enumerate(shape)] if keepdim else [shape[d] for d in keep]
    out = [c.map(lambda t: t.view(out_shape)) for c in out]
    if mean:
        divisor = from_planes([torch.full((), float(red) if red else float("nan"), dtype=md, device=dev)])
        out = series_op("div", len(out) - 1, out, divisor)
    return out


def _product(a, b):
    """One scaled matrix product A_i @ B_j (src/polytensors/_scaled.py:150-214): when the exponent
    spans of both operands together fit the native range, both mantissa sets are rescaled by their
    largest exponent (so every product of rescaled mantissas is representable) and multiplied on the
    product kernel; the result carries the sum of those exponents, however large.  (The reference
    also leaves its native path when that sum itself is out of range, for its mantissa adjoints;
    the values agree.)  Spans beyond the native range raise."""
    md = a.m.dtype
    safe = (126 if md == torch.float32 else 1022) - 4
    amax, amin = int(a.e.max()), int(a.e.min())
    bmax, bmin = int(b.e.max()), int(b.e.min())
    if not (amax - amin + bmax - bmin < safe):
        raise NotImplementedError("default-mode matrix product whose exponent span exceeds the native range "
                                  "(the reference's blocked scaled product) is not implemented on the kernels")
    x = to_planes([a], [md], offset=amax)[0]
    y = to_planes([b], [md], offset=bmax)[0]
    prod = K.poly_matmul([x], [y])[0]
    return from_planes([prod], base=amax + bmax)[0]


def poly_matmul(A, B):
    """C_k = sum_i A_i @ B_{k-i} with scaled products and scaled sums (the reference's default-mode
    series matrix product, src/polytensors/_scaled_matmul.py:38-40)."""
    md = torch.float64 if any(c.m.dtype == torch.float64 for c in A + B) else torch.float32
    A = [_cast(c, md) for c in A]
    B = [_cast(c, md) for c in B]
    out = []
    for k in range(len(A)):
        acc = None
        for i in range(k + 1):
            p = _product(A[i], B[k - i])
            acc = [p] if acc is None else series_op("add", 0, acc, [p], p0=1.0)
        out.append(acc[0])
    return out


# ---------------------------------------------------------------------------------------------
# hidden copies attached to PolyTensors (src/polytensors/_range.py)

def _snapshot(coeffs):
    return tuple((id(c), c._version) for c in coeffs)


def attach(poly, scs):
    if any(c.is_inference() for c in poly.coeffs):
        return poly
    poly._pk_scaled = tuple(scs)
    poly._pk_scaled_versions = _snapshot(poly.coeffs)
    return poly


def get(poly):
    scs = getattr(poly, "_pk_scaled", None)
    if scs is None:
        return None
    if getattr(poly, "_pk_scaled_versions", None) != _snapshot(poly.coeffs):
        del poly._pk_scaled
        return None
    return scs


def _is_poly(x):
    return hasattr(x, "coeffs")


def lift(x, like):
    """A series operand as SC coefficients: the hidden copy when valid, else its public coefficients;
    a constant as a one-coefficient list (its higher coefficients are zero)."""
    if _is_poly(x):
        scs = get(x)
        return list(scs) if scs is not None else from_planes(list(x.coeffs))
    if not isinstance(x, torch.Tensor):
        x = torch.full((), x, dtype=like.dtype, device=like.device)
    elif x.device != like.device and x.dim() == 0:
        x = x.to(like.device)
    if not x.is_floating_point():
        x = x.to(like.dtype)
    return from_planes([x])


def constant(value, dtype):
    """A Python scalar rounded to `dtype`, as the reference lifts a constant operand
    (torch.full((), value, dtype=result_type(like, value)), src/polytensors/_range_ops.py:40-42),
    returned as the float the kernels take."""
    return float(torch.tensor(value, dtype=dtype))


def _padded(scs, degree):
    zero = SC(torch.zeros_like(scs[0].m), torch.zeros_like(scs[0].e))
    return scs + [zero] * (degree + 1 - len(scs))


def _rep(x):
    return x.coeffs[0] if _is_poly(x) else x


def _complex(*xs):
    for x in xs:
        if _is_poly(x) and any(c.is_complex() for c in x.coeffs):
            return True
        if isinstance(x, complex) or (isinstance(x, torch.Tensor) and not _is_poly(x) and x.is_complex()):
            return True
    return False


ADD = (aten.add.Tensor, aten.add.Scalar, aten.add_.Tensor, aten.add_.Scalar)
SUB = (aten.sub.Tensor, aten.sub.Scalar, aten.sub_.Tensor, aten.sub_.Scalar)
MUL = (aten.mul.Tensor, aten.mul.Scalar, aten.mul_.Tensor, aten.mul_.Scalar)
DIV = (aten.div.Tensor, aten.div.Scalar, aten.div_.Tensor, aten.div_.Scalar)
MATMUL = (aten.mm.default, aten.bmm.default, aten.matmul.default, aten.mv.default, aten.dot.default)
REDUCE = (aten.sum.default, aten.sum.dim_IntList, aten.mean.default, aten.mean.dim)
# operations whose plain rule runs as usual, after which carry() moves the hidden copy along
CARRY = (aten.t.default, aten.transpose.int, aten.permute.default, aten.view.default, aten._unsafe_view.default,
         aten.expand.default, aten.slice.Tensor, aten.select.int, aten.unsqueeze.default, aten.squeeze.dim,
         aten.squeeze.default, aten.squeeze.dims, aten.alias.default, aten.detach.default, aten.clone.default,
         aten.reshape.default, aten.flatten.using_ints, aten._reshape_alias.default)


def _output(c, scs, dtype):
    return attach(c.wrap(to_planes(scs, [dtype] * len(scs))), scs)


def _write(target, scs):
    planes = to_planes(scs, [p.dtype for p in target.coeffs])
    for dest, src in zip(target.coeffs, planes):
        dest.copy_(src)
    return attach(target, scs)


def _matmul_shapes(func, A, B):
    """SC operands of mv / dot / matmul in the 2-D or batched 3-D product shapes, and the function
    restoring the output's shape (None for ranks the product kernel does not take)."""
    a_dim, b_dim = A[0].m.dim(), B[0].m.dim()
    if func is aten.mv.default or (func is aten.matmul.default and a_dim == 2 and b_dim == 1):
        return A, [c.map(lambda t: t.unsqueeze(1)) for c in B], lambda t: t.squeeze(1)
    if func is aten.dot.default or (func is aten.matmul.default and a_dim == 1 and b_dim == 1):
        return ([c.map(lambda t: t.unsqueeze(0)) for c in A], [c.map(lambda t: t.unsqueeze(1)) for c in B],
                lambda t: t.reshape(()))
    if a_dim in (2, 3) and a_dim == b_dim:
        return A, B, lambda t: t
    return None


def dispatch(c):
    """A default-mode rule for c.func, or NOT_HANDLED."""
    func, args, kwargs, D, like = c.func, c.args, c.kwargs, c.degree, c.like
    if func in (*ADD, *SUB, *MUL, *DIV):
        a, b = args[:2]
        if _complex(a, b) or (func in DIV and kwargs.get("rounding_mode") is not None):
            return NOT_HANDLED
        inplace = func._schema.is_mutable
        dtype = a.coeffs[0].dtype if inplace else torch.result_type(_rep(a), _rep(b))
        A, B = lift(a, like), lift(b, like)
        alpha = kwargs.get("alpha", 1)
        if func in ADD or func in SUB:
            out = series_op("add", D, A, B, p0=alpha if func in ADD else -alpha)
        elif func in MUL:
            out = series_op("mul", D, A, B)
        else:
            out = series_op("div", D, A, B)
        return _write(a, out) if inplace else _output(c, out, dtype)
    if func is aten.exp.default and not _complex(args[0]):
        # the series from the public input coefficients in scaled arithmetic, the public coefficients
        # converted from it, so that overflowing directions are +-inf rather than inf - inf
        # (src/polytensors/_dispatch.py:431-437, _series.py:23-42)
        x = args[0]
        scs = series_op("exp", D, from_planes(list(x.coeffs)))
        return _output(c, scs, x.coeffs[0].dtype)
    if func is aten.neg.default and not _complex(args[0]):
        return _output(c, series_op("affine", D, lift(args[0], like), p0=-1.0), args[0].coeffs[0].dtype)
    if func is aten.rsub.Scalar and not _complex(*args[:2]) and not isinstance(args[1], torch.Tensor):
        x, other = args[:2]
        dtype = torch.result_type(_rep(x), other)
        return _output(c, series_op("affine", D, lift(x, like), p0=-kwargs.get("alpha", 1), p1=constant(other, dtype)),
                       dtype)
    if func is aten.reciprocal.default and not _complex(args[0]):
        x = args[0]
        one = from_planes([torch.ones((), dtype=x.coeffs[0].dtype, device=like.device)])
        return _output(c, series_op("div", D, one, lift(x, like)), x.coeffs[0].dtype)
    if func in MATMUL or func in (aten.linear.default, aten.addmm.default):
        if func is aten.linear.default:
            x, w = args[:2]
            bias = args[2] if len(args) > 2 else kwargs.get("bias")
        elif func is aten.addmm.default:
            bias, x, w = args[:3]
        else:
            (x, w), bias = args[:2], None
        if _complex(x, w, bias) or not (_is_poly(x) or _is_poly(w)):
            return NOT_HANDLED
        A, B = _padded(lift(x, like), D), _padded(lift(w, like), D)
        dtype = torch.promote_types(_rep(x).dtype, _rep(w).dtype)
        if func is aten.linear.default:
            lead = A[0].shape[:-1]
            A = [s.map(lambda t: t.reshape(-1, t.shape[-1])) for s in A]
            B = [s.map(lambda t: t.t()) for s in B]
            out = [s.map(lambda t: t.reshape(*lead, t.shape[-1])) for s in poly_matmul(A, B)]
        else:
            shaped = _matmul_shapes(func, A, B)
            if shaped is None:
                return NOT_HANDLED
            A, B, restore = shaped
            out = [s.map(restore) for s in poly_matmul(A, B)]
        if func is aten.addmm.default:
            beta, alpha = kwargs.get("beta", 1), kwargs.get("alpha", 1)
            if alpha != 1:
                out = series_op("affine", D, out, p0=alpha)
            if beta != 0 and bias is not None:
                out = series_op("add", D, out, lift(bias, like), p0=beta)
        elif bias is not None:
            out = series_op("add", D, out, lift(bias, like), p0=1.0)
        return _output(c, out, dtype)
    if func in REDUCE and not _complex(args[0]):
        x = args[0]
        dim = args[1] if len(args) > 1 else kwargs.get("dim")
        dim = tuple(dim) if isinstance(dim, list) else dim
        if dim == ():
            dim = None
        if isinstance(dim, int):
            dim = (dim,)
        keepdim = args[2] if len(args) > 2 else kwargs.get("keepdim", False)
        mean = func in (aten.mean.default, aten.mean.dim)
        dtype = kwargs.get("dtype") or x.coeffs[0].dtype
        return _output(c, reduce(lift(x, like), dim, keepdim, mean), dtype)
    if func is aten.copy_.default and _is_poly(args[0]) and not _complex(*args[:2]):
        shape = args[0].coeffs[0].shape
        src = _padded(lift(args[1], like), D)
        return _write(args[0], [s.map(lambda t: t.expand(shape)) for s in src])
    return NOT_HANDLED


def carry(func, args, kwargs, result):
    """After a view / clone / detach of a series with a hidden copy, give the result the same
    operation applied to the copy's mantissas and exponents (the reference's map_tensor)."""
    src = args[0] if args else None
    if not (_is_poly(src) and _is_poly(result)):
        return result
    scs = get(src)
    if scs is None:
        return result
    rest = args[1:]
    try:
        moved = [c.map(lambda t: func(t, *rest, **kwargs)) for c in scs]
    except (RuntimeError, TypeError):
        return result
    return attach(result, moved)
