"""The PolyTensor wrapper subclass: the public API of the reference, with the series
arithmetic routed to libpolykern.

Interface parity with samuel-gunn/poly-tensors (src/polytensors/_tensor.py): the same
constructor rules, properties, context managers and ``backward`` seeding; the same
``__torch_function__`` (decompositions above autograd) / ``__torch_dispatch__`` (series
rules below autograd) split.  What differs is underneath: every rule on the hot path
is one CUDA kernel over all coefficient planes (see ``_dispatch.py`` and ``_fused.py``).
"""

import contextlib
import contextvars
import operator

import torch

from . import _state
from ._dispatch import dispatch

_COMPLEX_OF = {torch.float16: torch.complex32, torch.float32: torch.complex64, torch.float64: torch.complex128}


def _overlaps(a, b):
    return torch._C._overlaps(a, b)


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
        """Validate and normalise a coefficient sequence (rules of src/polytensors/_tensor.py:37-96)."""
        if isinstance(coeffs, PolyTensor):
            coeffs = coeffs.coeffs
        coeffs = tuple(coeffs)
        if degree is None and PolyTensor._well_formed(coeffs):
            return coeffs
        if not coeffs:
            raise ValueError("at least one coefficient is required")
        if degree is not None:
            if isinstance(degree, bool):
                raise TypeError("degree must be a nonnegative integer")
            degree = operator.index(degree)
            if degree < 0:
                raise ValueError("degree must be nonnegative")
        first = coeffs[0]
        base = first if isinstance(first, torch.Tensor) else torch.as_tensor(first)
        if not isinstance(first, torch.Tensor) and not (base.is_floating_point() or base.is_complex()):
            base = base.to(torch.get_default_dtype())
        tensors = []
        for c in coeffs:
            if isinstance(c, torch.Tensor):
                tensors.append(c)
            else:
                # Python numbers take the base's precision without a float32 round trip.
                tensors.append(torch.as_tensor(c, device=base.device,
                                               dtype=torch.promote_types(base.dtype, torch.as_tensor(c).dtype)))
        for c in tensors:
            if isinstance(c, PolyTensor):
                raise TypeError("nested PolyTensor coefficients are not supported")
            if c.layout != torch.strided:
                raise TypeError("coefficients must be dense strided tensors")
            if not (c.is_floating_point() or c.is_complex()):
                raise TypeError("tensor coefficients must have floating-point or complex dtype")
            if c.device != base.device:
                raise ValueError("all coefficients must be on the same device")
        common = tensors[0].dtype
        for c in tensors[1:]:
            common = torch.promote_types(common, c.dtype)
        real = torch.empty((), dtype=common).real.dtype
        complex_dirs = any(c.is_complex() for c in tensors[1:])
        tensors = [c.to(dtype=common if (c.is_complex() or (k > 0 and complex_dirs)) else real)
                   for k, c in enumerate(tensors)]
        if degree is not None:
            if degree < len(tensors) - 1:
                raise ValueError("degree must be at least the degree of coeffs")
            template = tensors[-1] if len(tensors) > 1 else tensors[0]
            tensors += [torch.zeros_like(template) for _ in range(degree + 1 - len(tensors))]
        shape = torch.broadcast_shapes(*(c.shape for c in tensors))
        tensors = [c if c.shape == shape else c.expand(shape).clone() for c in tensors]
        # Orders must be independently mutable: an in-place update of one order must not
        # write into another through shared storage.
        out = []
        for c in tensors:
            if any(_overlaps(c, prev) for prev in out):
                c = c.clone()
            out.append(c)
        return tuple(out)

    @staticmethod
    def _well_formed(coeffs):
        """Whether ``coeffs`` already satisfies every construction rule (the common case for
        rule outputs), so construction can skip normalisation."""
        if not coeffs:
            return False
        base = coeffs[0]
        if type(base) is not torch.Tensor or base.layout != torch.strided:
            return False
        dtype = base.dtype
        if not (dtype.is_floating_point or dtype.is_complex):
            return False
        higher = None
        for c in coeffs[1:]:
            if type(c) is not torch.Tensor or c.layout != torch.strided or c.shape != base.shape \
                    or c.device != base.device:
                return False
            if higher is None:
                higher = c.dtype
                if higher != dtype and _COMPLEX_OF.get(dtype) != higher:
                    return False
            elif c.dtype != higher:
                return False
        for i in range(1, len(coeffs)):
            for j in range(i):
                if _overlaps(coeffs[i], coeffs[j]):
                    return False
        return True

    def _set_coeffs(self, coeffs):
        self.coeffs = self._coerce_coeffs(coeffs)
        self.degree = len(self.coeffs) - 1

    @staticmethod
    def __new__(cls, coeffs, *, degree=None, requires_grad=False):
        coeffs = cls._coerce_coeffs(coeffs, degree)
        base = coeffs[0]
        out = torch.Tensor._make_wrapper_subclass(
            cls, base.shape, strides=base.stride(), storage_offset=base.storage_offset(),
            dtype=base.dtype, layout=base.layout, device=base.device, requires_grad=requires_grad)
        out.coeffs = coeffs
        out.degree = len(coeffs) - 1
        # Autograd may keep only the C++ TensorImpl of a saved wrapper; retention scopes
        # keep the Python object (and its coefficients) alive through backward.
        for refs in _state.retention_scopes.get():
            refs.append(out)
        return out

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
        try:
            yield
        finally:
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
        """Ordinary autograd graphs on the coefficient tensors (reference mode of the same
        name).  Not implemented by the polykern kernels: operations raise inside it."""
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

    def backward(self, gradient=None, retain_graph=None, create_graph=False, inputs=None):
        if gradient is None:
            if self.numel() != 1:
                raise RuntimeError("grad can be implicitly created only for scalar outputs")
            if self.is_complex():
                raise RuntimeError("an explicit gradient is required for a complex output")
            gradient = PolyTensor.constant(torch.ones_like(self.value), self.degree)
        elif not isinstance(gradient, PolyTensor):
            gradient = PolyTensor.constant(gradient, self.degree)
        torch.autograd.backward(self, gradient, retain_graph=retain_graph, create_graph=create_graph,
                                inputs=inputs)

    def __repr__(self):
        if not hasattr(self, "coeffs"):
            return f"PolyTensor(<uninitialized>, requires_grad={self.requires_grad})"
        return f"PolyTensor({self.coeffs}, requires_grad={self.requires_grad})"

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
        # value semantics (and native view tracking) while the rules run below autograd.
        with contextlib.ExitStack() as stack:
            for key in (torch._C.DispatchKey.Conjugate, torch._C.DispatchKey.Negative,
                        torch._C.DispatchKey.ADInplaceOrView):
                stack.enter_context(torch._C._SetExcludeDispatchKeyGuard(key, False))
            return dispatch(func, args, {} if kwargs is None else kwargs)
