"""The PolyTensor wrapper subclass: the public API of the reference, with the series
arithmetic routed to libpolykern.

Interface parity with samuel-gunn/poly-tensors (src/polytensors/_tensor.py): the same
constructor rules, properties, context managers and ``backward`` seeding; the same
``__torch_function__`` (decompositions above autograd) / ``__torch_dispatch__`` (series
rules below autograd) split.  What differs is underneath: every rule on the hot path
is one CUDA kernel over all coefficient planes (see ``_dispatch.py`` and ``_fused.py``).
"""

import contextlib
import functools
import operator

import torch

from . import _state
from ._dispatch import dispatch

# Complex dtype that may carry the directions of a real constant coefficient.
_DIRECTION_DTYPE = {torch.float16: torch.complex32, torch.float32: torch.complex64, torch.float64: torch.complex128}


def _shares_memory(a, b):
    return torch._C._overlaps(a, b)


def _is_canonical(planes):
    """True when ``planes`` can be used as they are: plain dense tensors on one device with one
    shape, a floating or complex constant coefficient, every higher coefficient of a single
    dtype (the constant's, or its complex counterpart), and no two coefficients sharing memory."""
    if not planes or any(type(c) is not torch.Tensor or c.layout != torch.strided for c in planes):
        return False
    head, rest = planes[0], planes[1:]
    if not (head.dtype.is_floating_point or head.dtype.is_complex):
        return False
    if any(c.shape != head.shape or c.device != head.device for c in rest):
        return False
    if rest:
        kinds = {c.dtype for c in rest}
        if len(kinds) != 1 or kinds.pop() not in (head.dtype, _DIRECTION_DTYPE.get(head.dtype)):
            return False
    return not any(_shares_memory(planes[i], planes[j]) for i in range(1, len(planes)) for j in range(i))


def _degree_argument(degree):
    if degree is None:
        return None
    if isinstance(degree, bool):
        raise TypeError("PolyTensor degree must be an int, not a bool")
    degree = operator.index(degree)   # TypeError for floats and other non-integers
    if degree < 0:
        raise ValueError(f"PolyTensor degree must be nonnegative, got {degree}")
    return degree


def _to_tensors(items):
    """Coefficients as tensors.  The constant coefficient fixes the device; a Python integer
    there becomes the default floating dtype.  Later Python numbers are created directly at the
    precision they promote to against the constant (no float32 round trip)."""
    head = items[0]
    if isinstance(head, torch.Tensor):
        anchor = head
    else:
        anchor = torch.as_tensor(head)
        if not (anchor.is_floating_point() or anchor.is_complex()):
            anchor = anchor.to(torch.get_default_dtype())
    out = []
    for c in items:
        if isinstance(c, torch.Tensor):
            out.append(c)
        else:
            kind = torch.promote_types(anchor.dtype, torch.as_tensor(c).dtype)
            out.append(torch.as_tensor(c, dtype=kind, device=anchor.device))
    return out


def _check_kinds(tensors):
    device = tensors[0].device
    for c in tensors:
        if isinstance(c, PolyTensor):
            raise TypeError("PolyTensor coefficients cannot themselves be PolyTensors (nested series)")
        if c.layout != torch.strided:
            raise TypeError(f"PolyTensor coefficients must be dense strided tensors, got layout {c.layout}")
        if not (c.is_floating_point() or c.is_complex()):
            raise TypeError(f"PolyTensor coefficients must have a floating-point or complex dtype, got {c.dtype}")
        if c.device != device:
            raise ValueError(f"PolyTensor coefficients must all be on the same device ({device} and {c.device})")


def _planes_from(coeffs, degree=None):
    """The coefficient tuple a PolyTensor stores for ``coeffs`` (a sequence or a PolyTensor)."""
    items = tuple(coeffs.coeffs if isinstance(coeffs, PolyTensor) else coeffs)
    if degree is None and _is_canonical(items):
        return items
    if not items:
        raise ValueError("a PolyTensor needs at least one coefficient")
    degree = _degree_argument(degree)
    tensors = _to_tensors(items)
    _check_kinds(tensors)
    # one promoted dtype: the constant keeps its real precision unless it is complex itself;
    # once any direction is complex, every direction is stored complex
    widest = functools.reduce(torch.promote_types, (c.dtype for c in tensors))
    real = widest.to_real() if widest.is_complex else widest
    directions_complex = any(c.is_complex() for c in tensors[1:])
    kinds = [widest if (c.is_complex() or (k and directions_complex)) else real for k, c in enumerate(tensors)]
    tensors = [c.to(kind) for c, kind in zip(tensors, kinds)]
    if degree is not None:
        if degree + 1 < len(tensors):
            raise ValueError(f"degree {degree} is lower than the {len(tensors) - 1} the coefficients need "
                             "(it must be at least their degree)")
        filler = tensors[-1]
        tensors.extend(torch.zeros_like(filler) for _ in range(degree + 1 - len(tensors)))
    shape = torch.broadcast_shapes(*(c.shape for c in tensors))
    planes = []
    for c in tensors:
        if c.shape != shape:
            c = c.expand(shape).clone()   # every order gets storage of its own shape
        elif any(_shares_memory(c, q) for q in planes):
            c = c.clone()                 # an in-place update of one order must not touch another
        planes.append(c)
    return tuple(planes)


class PolyTensor(torch.Tensor):
    """A truncated tensor-valued power series in one scalar variable ``t``.

    ``PolyTensor((x, v), degree=n)`` represents ``x + t*v`` kept through order ``n``;
    after a supported smooth function, coefficient ``k`` is the order-k directional
    derivative divided by ``k!``.  Operands must share the degree.  A real constant
    coefficient may carry complex directions; ``dtype`` is the constant coefficient's.
    Coefficients broadcast to one shape on one device; Python integers become floating
    point, integer tensors are rejected, and missing orders are zero-filled.
    """

    # ------------------------------------------------------------------ construction

    @staticmethod
    def _coerce_coeffs(coeffs, degree=None):
        """The normalised coefficient tuple (the constructor's rules; see ``_planes_from``)."""
        return _planes_from(coeffs, degree)

    def _set_coeffs(self, coeffs):
        self.coeffs = _planes_from(coeffs)
        self.degree = len(self.coeffs) - 1

    @staticmethod
    def __new__(cls, coeffs, *, degree=None, requires_grad=False):
        planes = _planes_from(coeffs, degree)
        head = planes[0]
        self = torch.Tensor._make_wrapper_subclass(
            cls, head.shape, strides=head.stride(), storage_offset=head.storage_offset(), dtype=head.dtype,
            layout=head.layout, device=head.device, requires_grad=requires_grad)
        self.coeffs, self.degree = planes, len(planes) - 1
        # Autograd may hold only the C++ side of a saved wrapper; every open retention scope keeps
        # the Python object (and so its coefficients) alive until the scope closes.
        for scope in _state.retention_scopes.get():
            scope.append(self)
        return self

    def __init__(self, coeffs, *, degree=None, requires_grad=False):
        pass

    # ------------------------------------------------------------------ inspection

    @property
    def value(self):
        return self.coeffs[0]

    @property
    def tangent(self):
        """The first coefficient (the first directional derivative)."""
        if self.degree == 0:
            raise ValueError("a degree-zero PolyTensor has no tangent")
        return self.coeffs[1]

    @classmethod
    def constant(cls, x, degree):
        """A value whose higher coefficients are all zero."""
        return cls((x,), degree=degree)

    # ------------------------------------------------------------------ modes

    @classmethod
    @contextlib.contextmanager
    def retain_wrappers(cls, isolated=False):
        """Keep intermediate PolyTensor wrappers alive through backward.

        Enclose each forward and its backward (and optimizer update) in one scope.  Scopes
        nest; an outer scope also retains its nested scopes' wrappers unless the inner scope
        is ``isolated``.  The yielded list is for diagnostics only.
        """
        refs = []
        token = _state.retention_scopes.set((refs,) if isolated else (*_state.retention_scopes.get(), refs))
        try:
            yield refs
        finally:
            _state.retention_scopes.reset(token)
            refs.clear()

    @classmethod
    @contextlib.contextmanager
    def plain_range(cls):
        """Ordinary floating-point range for coefficient arithmetic (the mode the kernels
        implement).  Context-local; run backward inside the same context."""
        token = _state.plain_range.set(True)
        _state.enter_plain()
        try:
            yield
        finally:
            _state.exit_plain()
            _state.plain_range.reset(token)

    @classmethod
    @contextlib.contextmanager
    def fused_attention(cls, enabled=True):
        """Enable or disable the fused attention kernel (default enabled).  Disabled, SDPA
        uses the reference decomposition (series matmul, masking, series softmax)."""
        token = _state.fused_attention.set(bool(enabled))
        try:
            yield
        finally:
            _state.fused_attention.reset(token)

    @classmethod
    @contextlib.contextmanager
    def fused_cross_entropy(cls, enabled=True):
        """Enable or disable the fused cross-entropy kernel (default enabled).  Disabled,
        cross entropy runs as series log-softmax followed by NLL."""
        token = _state.fused_cross_entropy.set(bool(enabled))
        try:
            yield
        finally:
            _state.fused_cross_entropy.reset(token)

    @classmethod
    @contextlib.contextmanager
    def coefficient_autograd(cls):
        """Ordinary autograd graphs on the coefficient tensors (the reference's mode of the same
        name): make coefficient tensors autograd leaves, build PolyTensors with
        ``requires_grad=False`` and differentiate output coefficients with ``torch.autograd.grad``.
        Each kernel-backed operation is one node of that graph (first-order derivatives)."""
        token = _state.coefficient_autograd.set(True)
        try:
            yield
        finally:
            _state.coefficient_autograd.reset(token)

    @staticmethod
    def cross_entropy(logits, target, softcap=None, ignore_index=-100, reduction="mean"):
        """Cross entropy of (N, C) logits, optionally capped as ``softcap * tanh(logits / softcap)``
        first, in one fused pass (forward and backward).  Accepts ordinary tensors and
        PolyTensors; returns at least float32."""
        from ._fused import cross_entropy

        return cross_entropy(logits, target, softcap=softcap, ignore_index=ignore_index, reduction=reduction)

    @staticmethod
    def linear_cross_entropy(input, weight, target, ignore_index=-100, reduction="mean", softcap=None,
                             chunk_rows=None):
        """``F.cross_entropy(F.linear(input, weight), target)`` without materialising all logits:
        row chunks of the series linear go straight into the streaming cross-entropy kernel, and
        backward recomputes each chunk (no counterpart in the reference)."""
        from ._fused import linear_cross_entropy

        return linear_cross_entropy(input, weight, target, ignore_index=ignore_index, reduction=reduction,
                                    softcap=softcap, chunk_rows=chunk_rows)

    def backward(self, gradient=None, retain_graph=None, create_graph=False, inputs=None):
        """Reverse-mode through the series: the seed is ``gradient`` as a PolyTensor of this degree
        (an ordinary tensor is its constant term); with no gradient, a real scalar seeds 1."""
        torch.autograd.backward(self, self._seed(gradient), retain_graph=retain_graph,
                                create_graph=create_graph, inputs=inputs)

    def _seed(self, gradient):
        if isinstance(gradient, PolyTensor):
            return gradient
        if gradient is not None:
            return PolyTensor.constant(gradient, self.degree)
        if self.numel() != 1:
            raise RuntimeError("backward() of a non-scalar PolyTensor needs an explicit gradient "
                               "(grad can be implicitly created only for scalar outputs)")
        if self.is_complex():
            raise RuntimeError("backward() of a complex PolyTensor needs an explicit gradient")
        return PolyTensor.constant(torch.ones_like(self.value), self.degree)

    def __repr__(self):
        planes = getattr(self, "coeffs", None)
        body = "<uninitialized>" if planes is None else repr(planes)
        return f"PolyTensor({body}, requires_grad={self.requires_grad})"

    # ------------------------------------------------------------------ interception

    @classmethod
    def __torch_function__(cls, func, types, args=(), kwargs=None):
        kwargs = {} if kwargs is None else kwargs
        from ._fused import maybe_fused

        result = maybe_fused(func, args, kwargs)
        if result is not NotImplemented:
            return result
        with torch._C.DisableTorchFunctionSubclass():
            return func(*args, **kwargs)

    @classmethod
    def __torch_dispatch__(cls, func, types, args=(), kwargs=None):
        # Coefficients may carry conjugate / negative view bits of their own; restore their
        # value semantics (and native view tracking) while the rules run below autograd.  In
        # coefficient_autograd() mode the autograd keys are re-enabled as well, so that the
        # operations on the coefficient tensors record their own graph.
        keys = [torch._C.DispatchKey.Conjugate, torch._C.DispatchKey.Negative, torch._C.DispatchKey.ADInplaceOrView]
        if _state.coefficient_autograd.get():
            keys += [torch._C.DispatchKey.Autograd, torch._C.DispatchKey.AutogradFunctionality,
                     torch._C.DispatchKey.AutogradOther, torch._C.DispatchKey.AutogradCPU,
                     torch._C.DispatchKey.AutogradCUDA]
        with contextlib.ExitStack() as stack:
            for key in keys:
                stack.enter_context(torch._C._SetExcludeDispatchKeyGuard(key, False))
            return dispatch(func, args, {} if kwargs is None else kwargs)
