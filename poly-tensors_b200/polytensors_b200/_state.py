"""Context-local switches of the PolyTensor API (the reference's ContextVars)."""

import contextvars

retention_scopes = contextvars.ContextVar("polytensor_retention_scopes", default=())
plain_range = contextvars.ContextVar("polytensor_plain_range", default=False)
fused_attention = contextvars.ContextVar("polytensor_fused_attention", default=True)
fused_cross_entropy = contextvars.ContextVar("polytensor_fused_cross_entropy", default=True)
coefficient_autograd = contextvars.ContextVar("polytensor_coefficient_autograd", default=False)
# The PolyTensor class the fused operations build their results from: unset for this package's
# own class; the reference binding (refbind) sets the reference's class around its calls.
poly_class = contextvars.ContextVar("polytensor_class", default=None)


def poly_cls():
    cls = poly_class.get()
    if cls is None:
        from ._tensor import PolyTensor

        return PolyTensor
    return cls
