"""Bind the polykern kernels to the reference's own ``PolyTensor`` (samuel-gunn/poly-tensors).

``install(polytensors)`` replaces the reference's gate functions for the hot path with calls into
``libpolykern``; the reference keeps its ``PolyTensor`` class, constructor rules, ``.coeffs`` /
``.value``, ``retain_wrappers()``, context managers and ``__torch_function__`` /
``__torch_dispatch__`` routing unchanged.  The sites, in the reference's source:

  * ``_plain.plain_polynomial_product`` (src/polytensors/_plain.py:118-128), which
    ``dispatch_range`` imports at every call (src/polytensors/_range_ops.py:24, :78-84):
    mm / bmm / matmul / addmm / linear (matrix=True, :160-176) -> pk_poly_gemm, and the
    elementwise Cauchy product of mul (matrix=False, :133-149) -> pk_series_map(MUL);
  * ``_fused_norm.eligible`` / ``rms_norm`` (src/polytensors/_fused_norm.py:11-21, :63-69),
    reached from ``maybe_decompose`` (src/polytensors/_decompositions.py:56-64) -> pk_rmsnorm_*;
  * ``_fused_cross_entropy.eligible`` / ``fused`` (src/polytensors/_fused_cross_entropy.py:131-170),
    reached from ``maybe_decompose`` (:65-79) and ``PolyTensor.cross_entropy``
    (src/polytensors/_tensor.py:255-269) -> pk_cross_entropy_*;
  * ``_fused_attention.eligible`` / ``attention`` (src/polytensors/_fused_attention.py:227-316),
    reached from ``maybe_decompose`` (:80-98) -> pk_flash_attn_fwd / score-epilogue products;
  * ``_fused_activation.maybe_activation`` (src/polytensors/_fused_activation.py:5-24), which
    ``plain_rule`` imports at every call (src/polytensors/_plain.py:280-290) -> pk_series_map
    (GELU / tanh / sigmoid and their backward rules).

Where the reference's degree-1 Triton gates accept degree 1 only, these accept every degree the
kernels take (<= 15).  Calls the kernels do not take (CPU tensors, mixed dtypes, shapes the
product does not cover) go to the function that was there before, so the reference's results are
unchanged there.  The reference's own switches keep their meaning: ``plain_range()`` (the
bound sites are plain-range rules), ``fused_attention(False)`` / ``fused_cross_entropy(False)``
and ``coefficient_autograd()`` (which keeps the general rules, as the reference's gates do).
"""

import contextlib

import torch

from . import _attention, _fused, _kernels as K, _lib, _state

_installed = {}


@contextlib.contextmanager
def _as(cls):
    token = _state.poly_class.set(cls)
    try:
        yield
    finally:
        _state.poly_class.reset(token)


def _real_float(t):
    return t.dtype in (torch.float32, torch.float64, torch.bfloat16, torch.float16)


# ------------------------------------------------------------------------------------------
# plain_polynomial_product (src/polytensors/_plain.py:118-128)

def _matrix_planes(A, B):
    """(a_planes, b_planes, reshape) for the shapes pk_poly_gemm takes, or None."""
    a, b = A[0], B[0]
    if a.dim() == 2 and b.dim() == 2:
        return A, B, None
    if a.dim() >= 3 and b.dim() == 2:
        lead, K_ = a.shape[:-1], a.shape[-1]
        return [x.reshape(-1, K_) for x in A], B, (*lead, b.shape[-1])
    if a.dim() >= 3 and a.dim() == b.dim() and a.shape[:-2] == b.shape[:-2]:
        lead = a.shape[:-2]
        return ([x.reshape(-1, *a.shape[-2:]) for x in A], [y.reshape(-1, *b.shape[-2:]) for y in B],
                (*lead, a.shape[-2], b.shape[-1]))
    return None


def _bound_product(original, PlainTensor):
    def plain_polynomial_product(left, right, *, matrix=False):
        A = [x.mantissa for x in left]
        B = [y.mantissa for y in right]
        planes = (*A, *B)
        if len(A) != len(B) or len(A) > _lib.PK_MAX_PLANES or not all(p.is_cuda for p in planes):
            return original(left, right, matrix=matrix)
        if matrix:
            if K.gemm_dtype(A, B) is None:
                return original(left, right, matrix=matrix)
            shaped = _matrix_planes(A, B)
            if shaped is None:
                return original(left, right, matrix=matrix)
            a, b, shape = shaped
            out = K.poly_matmul(a, b)
            if shape is not None:
                out = [c.reshape(shape) for c in out]
            return tuple(PlainTensor(c) for c in out)
        dtype = A[0].dtype
        if not _real_float(A[0]) or any(p.dtype != dtype for p in planes):
            return original(left, right, matrix=matrix)
        try:
            torch.broadcast_shapes(A[0].shape, B[0].shape)
        except RuntimeError:
            return original(left, right, matrix=matrix)
        return tuple(PlainTensor(c) for c in K.series_map("mul", len(A) - 1, A, B))

    plain_polynomial_product.__wrapped__ = original
    return plain_polynomial_product


# ------------------------------------------------------------------------------------------
# maybe_activation (src/polytensors/_fused_activation.py:5-24)

def _bound_activation(original, coefficient_autograd):
    def maybe_activation(X, kind, G=None):
        if coefficient_autograd.get():
            return None
        values = list(X) + ([] if G is None else list(G))
        if (len(X) > _lib.PK_MAX_PLANES or not all(c.is_cuda for c in values) or not _real_float(X[0])
                or any(c.dtype != X[0].dtype or c.shape != X[0].shape for c in values)):
            return original(X, kind, G)
        if G is None:
            return tuple(K.series_map(kind, len(X) - 1, list(X)))
        return tuple(K.series_map(kind + "_bwd", len(X) - 1, list(G), list(X)))

    maybe_activation.__wrapped__ = original
    return maybe_activation


# ------------------------------------------------------------------------------------------
# RMSNorm (src/polytensors/_fused_norm.py:11-21, :63-69)

def _bound_norm(module, ref):
    original_eligible, original_run = module.eligible, module.rms_norm

    def eligible(input, normalized_shape, eps):
        if not ref.plain_range_enabled() or ref.coefficient_autograd.get() or not isinstance(input, ref.cls):
            return original_eligible(input, normalized_shape, eps)
        if not all(c.is_cuda for c in input.coeffs):
            return original_eligible(input, normalized_shape, eps)
        with _as(ref.cls):
            return _fused.rms_norm_eligible(input, tuple(normalized_shape), None, eps) or \
                original_eligible(input, normalized_shape, eps)

    def rms_norm(input, normalized_shape, weight=None, eps=None):
        shape = tuple(normalized_shape)
        if not (isinstance(input, ref.cls) and all(c.is_cuda for c in input.coeffs)):
            return original_run(input, normalized_shape, weight, eps)
        with _as(ref.cls):
            if not _fused.rms_norm_eligible(input, shape, None, eps):
                return original_run(input, normalized_shape, weight, eps)
            fuse_weight = weight is not None and _fused.rms_norm_eligible(input, shape, weight, eps)
            if fuse_weight:
                return _fused.rms_norm(input, shape, weight, eps)
            out = _fused.rms_norm(input, shape, None, eps)
        return out if weight is None else out * weight

    eligible.__wrapped__, rms_norm.__wrapped__ = original_eligible, original_run
    return eligible, rms_norm


# ------------------------------------------------------------------------------------------
# cross entropy (src/polytensors/_fused_cross_entropy.py:131-170)

def _bound_cross_entropy(module, ref):
    original_eligible, original_fused = module.eligible, module.fused

    def eligible(input, target, weight, reduction, label_smoothing, softcap=None):
        if (module._enabled.get() and ref.plain_range_enabled() and not ref.coefficient_autograd.get()
                and isinstance(input, ref.cls)):
            with _as(ref.cls):
                if _fused.cross_entropy_eligible(input, target, weight, reduction, label_smoothing):
                    return True
        return original_eligible(input, target, weight, reduction, label_smoothing, softcap)

    def fused(input, target, ignore_index=-100, reduction="mean", softcap=None):
        with _as(ref.cls):
            if not _fused.cross_entropy_eligible(input, target, None, reduction, 0.0):
                return original_fused(input, target, ignore_index=ignore_index, reduction=reduction, softcap=softcap)
            return _fused.fused_cross_entropy(input, target, ignore_index=ignore_index, reduction=reduction,
                                              softcap=softcap)

    eligible.__wrapped__, fused.__wrapped__ = original_eligible, original_fused
    return eligible, fused


# ------------------------------------------------------------------------------------------
# attention (src/polytensors/_fused_attention.py:227-316)

def _bound_attention(module, ref):
    original_eligible, original_attention = module.eligible, module.attention

    def eligible(query, key, value, attn_mask, dropout_p, is_causal, enable_gqa):
        if module._enabled.get() and ref.plain_range_enabled() and not ref.coefficient_autograd.get():
            with _as(ref.cls):
                if _attention.eligible(query, key, value, attn_mask, dropout_p, is_causal, None, enable_gqa):
                    return True
        return original_eligible(query, key, value, attn_mask, dropout_p, is_causal, enable_gqa)

    def attention(query, key, value, attn_mask=None, is_causal=False, scale=None):
        with _as(ref.cls):
            if not _attention.eligible(query, key, value, attn_mask, 0.0, is_causal, scale, False):
                return original_attention(query, key, value, attn_mask=attn_mask, is_causal=is_causal, scale=scale)
            return _attention.attention(query, key, value, attn_mask=None, is_causal=is_causal, scale=scale)

    eligible.__wrapped__, attention.__wrapped__ = original_eligible, original_attention
    return eligible, attention


# ------------------------------------------------------------------------------------------

class _Reference:
    """The reference's class and switches, looked up once at install time."""

    def __init__(self, package):
        from importlib import import_module

        name = package.__name__
        self.tensor = import_module(f"{name}._tensor")
        self.plain = import_module(f"{name}._plain")
        self.cls = self.tensor.PolyTensor
        self.coefficient_autograd = self.tensor._coefficient_autograd_enabled
        self.plain_range_enabled = self.plain.plain_range_enabled
        self.norm = import_module(f"{name}._fused_norm")
        self.ce = import_module(f"{name}._fused_cross_entropy")
        self.attn = import_module(f"{name}._fused_attention")
        self.act = import_module(f"{name}._fused_activation")


def install(package):
    """Route the reference package's hot-path gates (``package`` is the imported
    ``polytensors`` module) to libpolykern.  Idempotent; ``uninstall`` restores them."""
    if package.__name__ in _installed:
        return
    _lib.load()   # fail loudly now if the library is missing, not inside a dispatch rule
    ref = _Reference(package)
    saved = []

    def put(module, name, value):
        saved.append((module, name, getattr(module, name)))
        setattr(module, name, value)

    put(ref.plain, "plain_polynomial_product",
        _bound_product(ref.plain.plain_polynomial_product, ref.plain.PlainTensor))
    put(ref.act, "maybe_activation", _bound_activation(ref.act.maybe_activation, ref.coefficient_autograd))
    eligible, run = _bound_norm(ref.norm, ref)
    put(ref.norm, "eligible", eligible)
    put(ref.norm, "rms_norm", run)
    eligible, run = _bound_cross_entropy(ref.ce, ref)
    put(ref.ce, "eligible", eligible)
    put(ref.ce, "fused", run)
    eligible, run = _bound_attention(ref.attn, ref)
    put(ref.attn, "eligible", eligible)
    put(ref.attn, "attention", run)
    _installed[package.__name__] = saved


def uninstall(package):
    """Put back the reference's own gate functions."""
    for module, name, value in reversed(_installed.pop(package.__name__, [])):
        setattr(module, name, value)


def installed(package):
    return package.__name__ in _installed


__all__ = ["install", "uninstall", "installed"]
