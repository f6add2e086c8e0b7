"""PyTorch operator rules for PolyTensor, below autograd.

Mirrors the routing of the reference (src/polytensors/_dispatch.py:90-852 with the
plain-range rules of src/polytensors/_plain.py:276-355 and src/polytensors/_range_ops.py):
the same operators, operand lifting (an ordinary tensor or number is a constant series),
degree check, in-place guard and error messages.  The arithmetic itself runs in
libpolykern: one launch per operation over all coefficient planes.  Shape and storage
operations (views, copies, factories) apply the native operation to each plane.
Operators without a rule raise ``NotImplementedError``.
"""

import math

import torch
from torch.utils._python_dispatch import return_and_correct_aliasing

from . import _kernels as K
from . import _scaled
from . import _state

aten = torch.ops.aten

_RULES = {}


def rule(*ops):
    def register(fn):
        for op in ops:
            _RULES[op] = fn
        return fn
    return register


def _is_wrapper(x):
    from ._tensor import PolyTensor

    return type(x) is PolyTensor


def is_poly(x):
    return _is_wrapper(x) and hasattr(x, "coeffs")


def _collect(x, polys, wrappers):
    if _is_wrapper(x):
        wrappers.append(x)
        if hasattr(x, "coeffs"):
            polys.append(x)
    elif isinstance(x, (tuple, list)):
        for y in x:
            _collect(y, polys, wrappers)
    elif isinstance(x, dict):
        for y in x.values():
            _collect(y, polys, wrappers)


def _has_poly(x):
    if is_poly(x):
        return True
    if isinstance(x, (tuple, list)):
        return any(_has_poly(y) for y in x)
    if isinstance(x, dict):
        return any(_has_poly(y) for y in x.values())
    return False


def _plain(x):
    """Replace PolyTensors by their constant coefficient (for index / target arguments)."""
    if _is_wrapper(x):
        return x.value
    if isinstance(x, tuple):
        return tuple(_plain(y) for y in x)
    if isinstance(x, list):
        return [_plain(y) for y in x]
    return x


class Ctx:
    """One dispatched call: the operator, its arguments and the common degree."""

    __slots__ = ("func", "args", "kwargs", "degree", "like")

    def __init__(self, func, args, kwargs, degree, like):
        self.func, self.args, self.kwargs, self.degree, self.like = func, args, kwargs, degree, like

    def lift(self, x):
        """Coefficient planes of a series operand; constants get zero higher planes."""
        if is_poly(x):
            return list(x.coeffs)
        if not isinstance(x, torch.Tensor):
            x = torch.full((), x, dtype=torch.result_type(self.like, x), device=self.like.device)
        if not (x.is_floating_point() or x.is_complex()):
            x = x.to(self.like.dtype)
        return [x] + [torch.zeros_like(x) for _ in range(self.degree)]

    def wrap(self, planes):
        from ._tensor import PolyTensor

        return PolyTensor(tuple(planes), requires_grad=False)

    def correct(self, out):
        """Native aliasing metadata for view operations (the wrapper's outer kernel owns it)."""
        with torch._C._SetExcludeDispatchKeyGuard(torch._C.DispatchKey.ADInplaceOrView, True):
            return return_and_correct_aliasing(self.func, self.args, self.kwargs, out)


def dispatch(func, args, kwargs):
    polys, wrappers = [], []
    _collect(args, polys, wrappers)
    _collect(kwargs, polys, wrappers)
    if len(polys) != len(wrappers):
        raise RuntimeError(
            "PolyTensor wrapper reached dispatch without coefficient storage. Keep every PolyTensor "
            "wrapper alive through forward and backward (PolyTensor.retain_wrappers()); silently "
            "replacing this value with zero would corrupt derivatives.")
    if not polys:
        return func(*args, **kwargs)
    if _state.coefficient_autograd.get():
        return _coefficient_dispatch(func, args, kwargs, polys)
    degree = polys[0].degree
    if any(p.degree != degree for p in polys[1:]):
        raise ValueError("PolyTensor operands must have the same degree")
    schema = getattr(func, "_schema", None)
    name = getattr(schema, "name", "")
    mutates = bool(getattr(schema, "is_mutable", False)) or name.rsplit("::", 1)[-1].endswith("_")
    if args and mutates and not is_poly(args[0]) and _has_poly((args[1:], kwargs)):
        target = args[0]
        raise RuntimeError(
            "cannot update a regular Tensor in-place with a PolyTensor; "
            f"func={func}, target_shape={getattr(target, 'shape', None)}, "
            f"target_dtype={getattr(target, 'dtype', None)}, "
            f"source_types=[{', '.join(type(a).__name__ for a in args[1:4])}]")
    ctx = Ctx(func, args, kwargs, degree, polys[0].value)
    default_mode = not _state.plain_mode()
    if default_mode:
        # outside plain_range(): the range operations on the extended-range kernels, with hidden
        # mantissa / exponent copies (src/polytensors/_range_ops.py:26-279)
        out = _scaled.dispatch(ctx)
        if out is not _scaled.NOT_HANDLED:
            return out
    fn = _RULES.get(func)
    if fn is None:
        raise NotImplementedError(f"PolyTensor does not implement {func}")
    out = fn(ctx)
    if default_mode and func in _scaled.CARRY:
        out = _scaled.carry(func, args, kwargs, out)
    return out


# ======================================================================================
# coefficient_autograd(): ordinary autograd graphs on the coefficient tensors
#
# In this mode (the reference's src/polytensors/_tensor.py:290-323) the user makes coefficient
# tensors autograd leaves and differentiates output coefficients with torch.autograd.grad.  The
# reference gets that by running its rules, which are torch operations, with autograd enabled.
# Here a rule launches kernels, so each operation becomes ONE autograd Function over all input
# coefficient planes: forward runs the rule, backward evaluates the coefficient map's
# vector-Jacobian product through the swapped-cotangent identity the reference documents for its
# fused kernels (src/polytensors/_fused_attention.py:18-22): for output cotangents c_0..c_n, the
# cotangent of input plane m is coefficient n - m of the wrapper gradient series of the same
# operation for the gradient series G_k = c_{n-k}; the operation is re-run under wrapper autograd
# in backward to obtain it.  Further (second-order) derivatives in this mode are not supported.

def _replace_polys(x, mapping):
    if is_poly(x) and id(x) in mapping:
        return mapping[id(x)]
    if isinstance(x, (list, tuple)):
        return type(x)(_replace_polys(v, mapping) for v in x)
    if isinstance(x, dict):
        return {k: _replace_polys(v, mapping) for k, v in x.items()}
    return x


class _CoefficientMap(torch.autograd.Function):
    @staticmethod
    def forward(ctx, func, args, kwargs, polys, *planes):
        from ._tensor import PolyTensor

        with torch.no_grad():
            out = dispatch(func, args, kwargs)
        if not isinstance(out, PolyTensor):
            raise NotImplementedError(f"PolyTensor.coefficient_autograd(): {func} does not return one PolyTensor")
        ctx.func, ctx.args, ctx.kwargs, ctx.polys = func, args, kwargs, polys
        ctx.out_meta = [(c.shape, c.dtype) for c in out.coeffs]
        ctx.save_for_backward(*planes)
        # outputs must not alias the inputs (view rules return per-plane views)
        return tuple(c.clone() if c._is_view() else c for c in out.coeffs)

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, *cots):
        from ._tensor import PolyTensor

        planes = ctx.saved_tensors
        mapping, leaves, pos = {}, [], 0
        for p in ctx.polys:
            n = p.degree + 1
            leaf = PolyTensor(tuple(t.detach() for t in planes[pos:pos + n]), requires_grad=True)
            mapping[id(p)] = leaf
            leaves.append(leaf)
            pos += n
        args = _replace_polys(ctx.args, mapping)
        kwargs = _replace_polys(ctx.kwargs, mapping)
        cots = [torch.zeros(shape, dtype=dt, device=planes[0].device) if c is None else c
                for c, (shape, dt) in zip(cots, ctx.out_meta)]
        token = _state.coefficient_autograd.set(False)
        try:
            with torch.enable_grad(), PolyTensor.retain_wrappers():
                y = ctx.func(*args, **kwargs)
                grads = torch.autograd.grad(y, leaves, PolyTensor(tuple(reversed(cots))), allow_unused=True)
        finally:
            _state.coefficient_autograd.reset(token)
        out = []
        for leaf, g in zip(leaves, grads):
            n = leaf.degree + 1
            out.extend([None] * n if g is None else [c.to(t.dtype) for c, t in zip(reversed(g.coeffs), leaf.coeffs)])
        return (None, None, None, None, *out)


def _coefficient_dispatch(func, args, kwargs, polys):
    from ._tensor import PolyTensor

    token = _state.coefficient_autograd.set(False)
    try:
        planes = [c for p in polys for c in p.coeffs]
        others = []
        _collect_plain_tensors((args, kwargs), others)
        if any(t.requires_grad for t in others):
            raise NotImplementedError("PolyTensor.coefficient_autograd(): ordinary tensors that require grad "
                                      "cannot be mixed with PolyTensors in this mode")
        if not (torch.is_grad_enabled() and any(c.requires_grad for c in planes)):
            with torch.no_grad():
                return dispatch(func, args, kwargs)
        schema = getattr(func, "_schema", None)
        if schema is not None and schema.is_mutable:
            raise NotImplementedError(f"PolyTensor.coefficient_autograd(): in-place {func} on coefficients "
                                      "that require grad")
        outs = _CoefficientMap.apply(func, args, kwargs, polys, *planes)
        return PolyTensor(tuple(outs), requires_grad=False)
    finally:
        _state.coefficient_autograd.reset(token)


def _collect_plain_tensors(x, out):
    if is_poly(x):
        return
    if isinstance(x, torch.Tensor):
        out.append(x)
    elif isinstance(x, (list, tuple)):
        for v in x:
            _collect_plain_tensors(v, out)
    elif isinstance(x, dict):
        for v in x.values():
            _collect_plain_tensors(v, out)


# ======================================================================================
# helpers

def _complex_dtype(dtype):
    return {torch.float16: torch.complex32, torch.float32: torch.complex64,
            torch.float64: torch.complex128}.get(dtype)


def _real_planes(planes, what):
    if any(p.is_complex() for p in planes):
        raise NotImplementedError(f"{what}: complex directions are not supported by this operation's kernels")
    return planes


def _cast(p, dtype):
    """Plane p in the precision of dtype, keeping a complex plane complex (a real base with complex
    directions stays so: the reference's per-plane dtypes, src/polytensors/_range_ops.py:46-64)."""
    if p.is_complex() and not dtype.is_complex:
        target = _complex_dtype(dtype) or p.dtype
    else:
        target = dtype
    return p if p.dtype == target else p.to(target)


def _write(c, target, planes):
    """In-place result: copy computed planes into the target's planes (unless they are them)."""
    for dest, src in zip(target.coeffs, planes):
        if src is not dest:
            if src.is_complex() and not dest.is_complex():
                raise RuntimeError("cannot copy complex PolyTensor coefficients into real coefficient storage")
            dest.copy_(src)
    return target


def _scalar(x):
    """A real Python number (the affine fast path takes real coefficients only)."""
    return isinstance(x, (int, float, bool)) and not isinstance(x, torch.Tensor)


def _host_number(x):
    if isinstance(x, torch.Tensor) and not is_poly(x) and x.dim() == 0 and x.device.type == "cpu" \
            and not x.is_complex():
        return x.item()
    return x


# ======================================================================================
# arithmetic (src/polytensors/_range_ops.py:105-158, constant fast path :109-132)

ADD = (aten.add.Tensor, aten.add.Scalar, aten.add_.Tensor, aten.add_.Scalar)
SUB = (aten.sub.Tensor, aten.sub.Scalar, aten.sub_.Tensor, aten.sub_.Scalar)
MUL = (aten.mul.Tensor, aten.mul.Scalar, aten.mul_.Tensor, aten.mul_.Scalar)
DIV = (aten.div.Tensor, aten.div.Scalar, aten.div_.Tensor, aten.div_.Scalar)


def _rep(x):
    return x.coeffs[0] if is_poly(x) else x


@rule(*ADD, *SUB, *MUL, *DIV)
def _arith(c):
    func = c.func
    a, b = c.args[:2]
    alpha = c.kwargs.get("alpha", 1)
    if func in DIV and c.kwargs.get("rounding_mode") is not None:
        raise NotImplementedError("PolyTensor does not implement rounded division")
    inplace = func._schema.is_mutable
    if inplace:
        dtype = a.coeffs[0].dtype
    else:
        dtype = torch.result_type(_rep(a), _rep(b))
    # Python numbers reach dispatch as 0-dim CPU "wrapped number" tensors: read them on the
    # host instead of copying them to the device (a blocking copy per operation).
    a, b = _host_number(a), _host_number(b)
    D = c.degree
    out = list(a.coeffs) if inplace else None

    def planes(x):
        if is_poly(x):
            return [_cast(p, dtype) for p in x.coeffs]
        t = x if isinstance(x, torch.Tensor) else torch.full((), x, dtype=dtype, device=c.like.device)
        if t.device != c.like.device and t.dim() == 0:
            t = t.to(c.like.device)
        return [_cast(t, dtype)]

    sign = -alpha if func in SUB else alpha
    if func in ADD or func in SUB:
        if is_poly(a) and _scalar(b):
            res = K.series_map("affine", D, planes(a), p0=1.0, p1=sign * b, out=out)
        elif is_poly(a):
            res = K.series_map("add", D, planes(a), planes(b), p0=sign, out=out)
        else:  # constant + series: (a) + sign * (b)
            res = K.series_map("add", D, planes(a), planes(b), p0=sign, out=out)
    elif func in MUL:
        if is_poly(a) and _scalar(b):
            res = K.series_map("affine", D, planes(a), p0=b, out=out)
        elif is_poly(b) and _scalar(a):
            res = K.series_map("affine", D, planes(b), p0=a, out=out)
        else:
            res = K.series_map("mul", D, planes(a), planes(b), out=out)
    else:
        res = K.series_map("div", D, planes(a), planes(b), out=out)
    if inplace:
        return a
    return c.wrap(res)


@rule(aten.rsub.Scalar, aten.rsub.Tensor)
def _rsub(c):
    x, other = c.args[:2]
    other = _host_number(other)
    alpha = c.kwargs.get("alpha", 1)
    if is_poly(x) and _scalar(other):
        return c.wrap(K.series_map("affine", c.degree, c.lift(x), p0=-alpha, p1=other))
    # other - alpha * x with a tensor or series `other`
    dtype = torch.result_type(_rep(x), _rep(other))
    X = [_cast(p, dtype) for p in c.lift(x)]
    O = [_cast(p, dtype) for p in c.lift(other)]
    return c.wrap(K.series_map("add", c.degree, O, X, p0=-alpha))


@rule(aten.neg.default)
def _neg(c):
    return c.wrap(K.series_map("affine", c.degree, c.lift(c.args[0]), p0=-1.0))


@rule(aten.pow.Tensor_Scalar)
def _pow(c):
    x, n = c.args[:2]
    if isinstance(n, float) and n.is_integer():
        n = int(n)
    if not isinstance(n, int) or isinstance(n, bool) or n < 0:
        raise NotImplementedError("only nonnegative integer powers")
    return c.wrap(K.series_map("powi", c.degree, c.lift(x), p0=float(n)))


def _unary(name):
    def fn(c):
        return c.wrap(K.series_map(name, c.degree, c.lift(c.args[0])))
    return fn


for _op, _name in ((aten.exp.default, "exp"), (aten.log.default, "log"), (aten.sqrt.default, "sqrt"),
                   (aten.rsqrt.default, "rsqrt"), (aten.reciprocal.default, "reciprocal"),
                   (aten.tanh.default, "tanh"), (aten.sigmoid.default, "sigmoid")):
    _RULES[_op] = _unary(_name)


@rule(aten.gelu.default)
def _gelu(c):
    approximate = c.args[1] if len(c.args) > 1 else c.kwargs.get("approximate", "none")
    if approximate != "none":
        raise NotImplementedError("PolyTensor implements exact GELU (approximate='none') only")
    return c.wrap(K.series_map("gelu", c.degree, c.lift(c.args[0])))


@rule(aten.gelu_backward.default)
def _gelu_backward(c):
    approximate = c.args[2] if len(c.args) > 2 else c.kwargs.get("approximate", "none")
    if approximate != "none":
        raise NotImplementedError("PolyTensor implements exact GELU (approximate='none') only")
    G, X = c.lift(c.args[0]), c.lift(c.args[1])
    dtype = X[0].dtype
    return c.wrap(K.series_map("gelu_bwd", c.degree, [_cast(g, dtype) for g in G], X))


@rule(aten.tanh_backward.default)
def _tanh_backward(c):
    G, Y = c.lift(c.args[0]), c.lift(c.args[1])
    return c.wrap(K.series_map("tanh_bwd", c.degree, [_cast(g, Y[0].dtype) for g in G], Y))


@rule(aten.sigmoid_backward.default)
def _sigmoid_backward(c):
    G, Y = c.lift(c.args[0]), c.lift(c.args[1])
    return c.wrap(K.series_map("sigmoid_bwd", c.degree, [_cast(g, Y[0].dtype) for g in G], Y))


# ======================================================================================
# matrix products (src/polytensors/_range_ops.py:160-176)

def _gemm_planes(c, a, b):
    A, B = c.lift(a), c.lift(b)
    dt = torch.promote_types(A[0].dtype, B[0].dtype)
    if not dt.is_complex and all(not p.is_complex() for p in (*A, *B)):
        A = [p.to(dt) for p in A]
        B = [p.to(dt) for p in B]
    return A, B


@rule(aten.mm.default, aten.bmm.default)
def _mm(c):
    A, B = _gemm_planes(c, *c.args[:2])
    return c.wrap(K.poly_matmul(A, B))


@rule(aten.mv.default)
def _mv(c):
    A, B = _gemm_planes(c, *c.args[:2])
    out = K.poly_matmul(A, [v.unsqueeze(1) for v in B])
    return c.wrap([o.squeeze(1) for o in out])


@rule(aten.dot.default)
def _dot(c):
    A, B = _gemm_planes(c, *c.args[:2])
    out = K.poly_matmul([a.unsqueeze(0) for a in A], [b.unsqueeze(1) for b in B])
    return c.wrap([o.reshape(()) for o in out])


@rule(aten.addmm.default)
def _addmm(c):
    bias, a, b = c.args[:3]
    beta, alpha = c.kwargs.get("beta", 1), c.kwargs.get("alpha", 1)
    A, B = _gemm_planes(c, a, b)
    out = K.poly_matmul(A, B)
    if alpha != 1:
        out = K.series_map("affine", c.degree, out, p0=alpha)
    if beta != 0:
        Bias = [p.to(out[0].dtype) for p in c.lift(bias)]
        out = K.series_map("add", c.degree, out, Bias, p0=beta)
    return c.wrap(out)


@rule(aten.linear.default)
def _linear(c):
    x, w = c.args[:2]
    bias = c.args[2] if len(c.args) > 2 else c.kwargs.get("bias")
    X, W = _gemm_planes(c, x, w)
    lead = X[0].shape[:-1]
    out = K.poly_matmul([p.reshape(-1, p.shape[-1]) for p in X], [p.t() for p in W])
    out = [o.view(*lead, o.shape[-1]) for o in out]
    if bias is not None:
        out = K.series_map("add", c.degree, out, [p.to(out[0].dtype) for p in c.lift(bias)], p0=1.0)
    return c.wrap(out)


@rule(aten.matmul.default)
def _matmul(c):
    a, b = c.args[:2]
    A, B = _gemm_planes(c, a, b)
    if A[0].dim() == 1 and B[0].dim() == 1:
        return _dot(c)
    if A[0].dim() == 2 and B[0].dim() == 2:
        return c.wrap(K.poly_matmul(A, B))
    raise NotImplementedError("PolyTensor matmul of this rank should decompose into mm/bmm before dispatch")


# ======================================================================================
# reductions (src/polytensors/_range_ops.py:178-207)

def reduce_planes(planes, dims, keepdim, mean, dtype=None):
    x = planes
    if dtype is not None:
        x = [p.to(dtype) for p in x]
    nd = x[0].dim()
    shape = list(x[0].shape)
    if nd == 0:
        return [p.clone() for p in x]
    if dims is None:
        dims = list(range(nd))
    dims = sorted({d % nd for d in dims})
    red = 1
    for d in dims:
        red *= shape[d]
    out_shape = [1 if d in dims else s for d, s in enumerate(shape)] if keepdim else \
        [s for d, s in enumerate(shape) if d not in dims]
    work_dtype = x[0].dtype
    if work_dtype in (torch.float16, torch.bfloat16):
        x = [p.float() for p in x]
    if dims == list(range(dims[0], dims[-1] + 1)):
        outer = math.prod(shape[:dims[0]])
        inner = math.prod(shape[dims[-1] + 1:])
        src = x
    else:
        keep = [d for d in range(nd) if d not in dims]
        src = [p.permute(*keep, *dims) for p in x]
        outer, inner = math.prod(shape[d] for d in keep), 1
    scale = (1.0 / red if red else float("nan")) if mean else 1.0
    if not any(p.is_complex() for p in src):
        out = K.series_reduce(src, outer, red, inner, scale)
        return [o.view(out_shape).to(work_dtype) for o in out]
    # complex planes (a real base with complex directions): the sum is linear, so a complex plane
    # is reduced as its (re, im) pairs, i.e. as a real plane with twice the inner extent
    out = [None] * len(src)
    for is_c in (False, True):
        idx = [i for i, p in enumerate(src) if p.is_complex() == is_c]
        if not idx:
            continue
        group = [torch.view_as_real(src[i].contiguous()) if is_c else src[i] for i in idx]
        res = K.series_reduce(group, outer, red, inner * (2 if is_c else 1), scale)
        for i, r in zip(idx, res):
            out[i] = torch.view_as_complex(r.view(-1, 2)).view(out_shape) if is_c else r.view(out_shape)
    return out


@rule(aten.sum.default, aten.sum.dim_IntList, aten.mean.default, aten.mean.dim)
def _sum(c):
    x = c.args[0]
    dim = c.args[1] if len(c.args) > 1 else c.kwargs.get("dim")
    dim = tuple(dim) if isinstance(dim, list) else dim
    if dim == ():
        dim = None
    if isinstance(dim, int):
        dim = (dim,)
    keepdim = c.args[2] if len(c.args) > 2 else c.kwargs.get("keepdim", False)
    mean = c.func in (aten.mean.default, aten.mean.dim)
    return c.wrap(reduce_planes(c.lift(x), dim, keepdim, mean, c.kwargs.get("dtype")))


@rule(aten.sum_to_size.default, aten._grad_sum_to_size.default)
def _sum_to_size(c):
    x, shape = c.args[0], c.args[1]
    if shape is None:
        return x
    planes = c.lift(x)
    cur = list(planes[0].shape)
    lead = len(cur) - len(shape)
    dims = list(range(lead)) + [i + lead for i, s in enumerate(shape) if s == 1 and cur[i + lead] != 1]
    if not dims:
        return c.wrap([p.reshape(shape).clone() for p in planes])
    out = reduce_planes(planes, dims, True, False)
    return c.wrap([o.reshape(shape) for o in out])


# ======================================================================================
# shape, view and storage operations: the native operation on every plane

VIEW_OPS = (
    aten.t.default, aten.transpose.int, aten.permute.default, aten.view.default, aten._unsafe_view.default,
    aten.expand.default, aten.slice.Tensor, aten.select.int, aten.unsqueeze.default, aten.squeeze.dim,
    aten.squeeze.default, aten.squeeze.dims, aten.alias.default, aten.detach.default, aten.as_strided.default,
    aten.diagonal.default, aten.unfold.default, aten._reshape_alias.default,
)


@rule(*VIEW_OPS)
def _view(c):
    x = c.args[0]
    return c.correct(c.wrap(c.func(p, *c.args[1:], **c.kwargs) for p in x.coeffs))


@rule(aten.reshape.default, aten.flatten.using_ints, aten.index_select.default, aten.gather.default,
      aten.index.Tensor, aten.flip.default, aten.roll.default, aten.repeat.default, aten.clone.default,
      aten.tril.default, aten.triu.default, aten.constant_pad_nd.default)
def _per_plane(c):
    x = c.args[0]
    args = _plain(c.args[1:])
    return c.wrap(c.func(p, *args, **c.kwargs) for p in x.coeffs)


@rule(aten.split.Tensor, aten.split_with_sizes.default, aten.unbind.int, aten.chunk.default)
def _split(c):
    x = c.args[0]
    parts = [c.func(p, *c.args[1:], **c.kwargs) for p in x.coeffs]
    out = tuple(c.wrap(group) for group in zip(*parts))
    return c.correct(list(out) if c.func is not aten.unbind.int else out)


@rule(aten.cat.default, aten.stack.default)
def _cat(c):
    sources = c.args[0]
    dim = c.args[1] if len(c.args) > 1 else c.kwargs.get("dim", 0)
    groups = [c.lift(s) for s in sources]
    out = []
    for k in range(c.degree + 1):
        items = [g[k] for g in groups]
        dt = items[0].dtype
        for t in items[1:]:
            dt = torch.promote_types(dt, t.dtype)
        out.append(c.func([t.to(dt) for t in items], dim))
    return c.wrap(out)


@rule(aten.detach_.default)
def _detach_(c):
    x = c.args[0]
    x._set_coeffs(p.detach() for p in x.coeffs)
    return x


@rule(aten.copy_.default)
def _copy_(c):
    dest, src = c.args[:2]
    return _write(c, dest, c.lift(src))


@rule(aten.zero_.default)
def _zero_(c):
    for p in c.args[0].coeffs:
        p.zero_()
    return c.args[0]


@rule(aten.masked_fill.Scalar, aten.masked_fill.Tensor, aten.masked_fill_.Scalar, aten.masked_fill_.Tensor)
def _masked_fill(c):
    source, mask, value = c.args[:3]
    if is_poly(mask):
        mask = mask.value
    fills = c.lift(value)
    planes = [torch.where(mask, f.to(p.dtype), p) for p, f in zip(c.lift(source), fills)]
    if c.func._schema.is_mutable:
        return _write(c, source, planes)
    return c.wrap(planes)


@rule(aten.where.self, aten.where.ScalarOther, aten.where.ScalarSelf, aten.where.Scalar)
def _where(c):
    cond, a, b = c.args[:3]
    if is_poly(cond):
        cond = cond.value
    A, B = c.lift(a), c.lift(b)
    out = []
    for x, y in zip(A, B):
        dt = torch.promote_types(x.dtype, y.dtype)
        out.append(torch.where(cond, x.to(dt), y.to(dt)))
    return c.wrap(out)


@rule(aten.isnan.default)
def _isnan(c):
    planes = c.lift(c.args[0])
    out = torch.isnan(planes[0])
    for p in planes[1:]:
        out = out | torch.isnan(p)
    return out


# ======================================================================================
# factories and conversions (src/polytensors/_dispatch.py:770-840)

def _coefficient_dtype(coefficient, dtype):
    if not coefficient.is_complex() or dtype is None or dtype.is_complex:
        return dtype
    cd = _complex_dtype(dtype)
    if cd is None:
        raise TypeError(f"{dtype} cannot represent complex PolyTensor directions")
    return cd


def _options(coefficient, kwargs):
    kwargs = dict(kwargs)
    if "dtype" in kwargs:
        kwargs["dtype"] = _coefficient_dtype(coefficient, kwargs["dtype"])
    return kwargs


@rule(aten.ones_like.default)
def _ones_like(c):
    x0 = c.lift(c.args[0])[0]
    one = c.func(x0, *c.args[1:], **c.kwargs)
    return c.wrap([one] + [torch.zeros_like(one) for _ in range(c.degree)])


@rule(aten.full_like.default)
def _full_like(c):
    kwargs = dict(c.kwargs)
    fill = c.args[1] if len(c.args) > 1 else kwargs.pop("fill_value")
    first = torch.full_like(c.lift(c.args[0])[0], fill, *c.args[2:], **kwargs)
    return c.wrap([first] + [torch.zeros_like(first) for _ in range(c.degree)])


@rule(aten.zeros_like.default, aten.empty_like.default)
def _zeros_like(c):
    return c.wrap(c.func(p, *c.args[1:], **_options(p, c.kwargs)) for p in c.lift(c.args[0]))


@rule(aten.new_empty_strided.default, aten.new_empty.default, aten.new_zeros.default)
def _new_factory(c):
    return c.wrap(c.func(p, *c.args[1:], **_options(p, c.kwargs)) for p in c.lift(c.args[0]))


@rule(aten.new_ones.default, aten.new_full.default)
def _new_const(c):
    first = c.func(c.lift(c.args[0])[0], *c.args[1:], **c.kwargs)
    return c.wrap([first] + [torch.zeros_like(first) for _ in range(c.degree)])


@rule(aten._to_copy.default, aten.to.dtype, aten.to.device, aten.to.dtype_layout)
def _to_copy(c):
    def convert(p):
        args = list(c.args[1:])
        kwargs = _options(p, c.kwargs)
        if c.func in (aten.to.dtype, aten.to.dtype_layout) and args:
            args[0] = _coefficient_dtype(p, args[0])
        elif c.func is aten.to.device and len(args) > 1:
            args[1] = _coefficient_dtype(p, args[1])
        return c.func(p, *args, **kwargs)

    return c.wrap(convert(p) for p in c.lift(c.args[0]))


# ======================================================================================
# softmax family (src/polytensors/_plain.py:262-273, :326-354)

def _along_last(planes, dim):
    nd = planes[0].dim()
    dim = dim % nd if nd else 0
    if nd == 0 or dim == nd - 1:
        return planes, None
    return [p.transpose(dim, -1) for p in planes], dim


def _restore(planes, moved):
    return planes if moved is None else [p.transpose(moved, -1) for p in planes]


@rule(aten._softmax.default, aten._log_softmax.default)
def _softmax(c):
    x, dim = c.args[0], c.args[1]
    half_to_float = c.args[2] if len(c.args) > 2 else False
    X = _real_planes(c.lift(x), "softmax")
    if half_to_float:
        X = [p.float() for p in X]
    if X[0].dim() == 0:
        X = [p.reshape(1) for p in X]
        out = K.softmax_fwd(X, log=c.func is aten._log_softmax.default)
        return c.wrap([o.reshape(()) for o in out])
    Xm, moved = _along_last(X, dim)
    out = K.softmax_fwd(Xm, log=c.func is aten._log_softmax.default)
    return c.wrap(p.contiguous() if moved is not None else p for p in _restore(out, moved))


@rule(aten._softmax_backward_data.default, aten._log_softmax_backward_data.default)
def _softmax_backward(c):
    grad, output, dim = c.args[:3]
    input_dtype = c.args[3] if len(c.args) > 3 else c.kwargs.get("input_dtype")
    G, Y = c.lift(grad), c.lift(output)
    log = c.func is aten._log_softmax_backward_data.default
    Gm, moved = _along_last(G, dim)
    Ym, _ = _along_last(Y, dim)
    out = _restore(K.softmax_bwd(Gm, Ym, log), moved)
    out = [p.contiguous() if moved is not None else p for p in out]
    if input_dtype is not None:
        out = [p.to(input_dtype) for p in out]
    return c.wrap(out)


@rule(aten.logsumexp.default)
def _logsumexp(c):
    x = c.args[0]
    dim = c.args[1] if len(c.args) > 1 else c.kwargs["dim"]
    keepdim = c.args[2] if len(c.args) > 2 else c.kwargs.get("keepdim", False)
    if isinstance(dim, (tuple, list)):
        if len(dim) != 1:
            raise NotImplementedError("PolyTensor logsumexp supports one dimension")
        dim = dim[0]
    X = _real_planes(c.lift(x), "logsumexp")
    Xm, moved = _along_last(X, dim)
    ls = K.softmax_fwd(Xm, log=True)
    # logsumexp_k = x_k - log_softmax_k at any element of the row (the first)
    out = [(xp[..., :1] - lp[..., :1]) for xp, lp in zip(Xm, ls)]
    out = _restore(out, moved)
    if not keepdim:
        out = [p.squeeze(dim) for p in out]
    return c.wrap(p.contiguous() for p in out)


# ======================================================================================
# losses, embedding, dropout (src/polytensors/_dispatch.py:530-562, :640-685)

@rule(aten.nll_loss_forward.default)
def _nll_forward(c):
    if _has_poly((c.args[1:], c.kwargs)):
        raise NotImplementedError("PolyTensor NLL loss requires ordinary targets and class weights")
    rest = _plain(c.args[1:])
    outs = [c.func(p, *rest, **c.kwargs) for p in _real_planes(c.lift(c.args[0]), "nll_loss")]
    return c.wrap(o[0] for o in outs), outs[0][1]


@rule(aten.nll_loss_backward.default)
def _nll_backward(c):
    if _has_poly((c.args[2:], c.kwargs)):
        raise NotImplementedError("PolyTensor NLL loss requires ordinary targets, class weights, and total weight")
    rest = _plain(c.args[1:])
    return c.wrap(c.func(g, *rest, **c.kwargs) for g in c.lift(c.args[0]))


@rule(aten.embedding.default)
def _embedding(c):
    weight, indices = c.args[:2]
    if is_poly(indices):
        raise NotImplementedError("PolyTensor embedding indices must be ordinary tensors")
    return c.wrap(K.gather_rows(c.lift(weight), indices))


@rule(aten.embedding_dense_backward.default)
def _embedding_backward(c):
    grad, indices, num_weights, padding_idx, scale_grad_by_freq = c.args[:5]
    if scale_grad_by_freq:
        raise NotImplementedError("PolyTensor embedding backward with scale_grad_by_freq")
    return c.wrap(K.scatter_add_rows(c.lift(grad), _plain(indices), num_weights, padding_idx))


@rule(aten.native_dropout.default)
def _native_dropout(c):
    x = c.args[0]
    p = c.args[1] if len(c.args) > 1 else c.kwargs["p"]
    train = c.args[2] if len(c.args) > 2 else c.kwargs["train"]
    X = c.lift(x)
    y0, mask = c.func(X[0], p, train)
    if not train or p == 0:
        return c.wrap((y0, *X[1:])), mask
    if p == 1:
        return c.wrap(torch.zeros_like(t) for t in X), mask
    scale = 1.0 / (1.0 - p)
    m = mask.to(X[0].dtype)
    return c.wrap((y0, *(t * m * scale for t in X[1:]))), mask


@rule(aten.native_dropout_backward.default)
def _native_dropout_backward(c):
    rest = _plain(c.args[1:])
    return c.wrap(c.func(g, *rest, **c.kwargs) for g in c.lift(c.args[0]))
