"""Context-local switches of the PolyTensor API (the reference's ContextVars)."""

import contextvars
import threading

import torch

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


# plain_range() blocks open anywhere in the process.  Backward of CUDA tensors runs on the autograd
# engine's device threads, where the ContextVars of the thread that called backward() are not set;
# an operation running inside a backward while a plain_range() block is open is taken to belong to
# it (a backward is run inside the context of its forward), so the gradient rules keep the forward's
# plain-range arithmetic.
_plain_open = 0
_plain_lock = threading.Lock()


def enter_plain():
    global _plain_open
    with _plain_lock:
        _plain_open += 1


def exit_plain():
    global _plain_open
    with _plain_lock:
        _plain_open -= 1


def plain_mode():
    """Whether series arithmetic here runs in plain range: inside plain_range() on this context, or
    inside a backward while a plain_range() block is open."""
    if plain_range.get():
        return True
    return _plain_open > 0 and torch._C._current_autograd_node() is not None
