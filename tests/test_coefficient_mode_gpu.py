"""PolyTensor.coefficient_autograd() through the kernels: output coefficients are ordinary tensors
whose gradients with respect to the input coefficients are the coefficient map's vector-Jacobian
products (the reference's src/polytensors/_tensor.py:290-323).

Checked two ways: against the reference's own test pattern (tests/test_fused_kernels.py:75-90:
the gradient of sum(out_1) with respect to the order-0 inputs equals order 1 of the wrapper
gradient series for G = (1, 0)), and against plain torch autograd through the CPU oracle, which
differentiates the coefficient map directly.  float64, tolerance 1e-10 per plane (1e-12 where the
two sides run the same kernels)."""

import pytest
import torch
import torch.nn.functional as F

from gpu_util import assert_close, poly, series
from oracle import polyref as ref

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-300)).item()


def test_coefficient_mode_matches_wrapper_autograd():
    from polytensors_b200 import PolyTensor

    shape = (1, 2, 96, 32)
    coefficients = [tuple(c.cuda().requires_grad_() for c in series(shape, 1, 40 + i)) for i in range(3)]
    q, k, v = (PolyTensor(c, requires_grad=False) for c in coefficients)
    with PolyTensor.coefficient_autograd(), PolyTensor.plain_range():
        out = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    assert out.coeffs[1].grad_fn is not None
    first = torch.autograd.grad(out.coeffs[1].sum(), [c[0] for c in coefficients])
    q2, k2, v2 = (PolyTensor(tuple(x.detach() for x in c), requires_grad=True) for c in coefficients)
    with PolyTensor.retain_wrappers(), PolyTensor.plain_range():
        out2 = F.scaled_dot_product_attention(q2, k2, v2, is_causal=True)
        out2.backward(PolyTensor.constant(torch.ones_like(out2.value), 1))
    for x, g in zip((q2, k2, v2), first):
        assert _rel(g, x.grad.coeffs[1]) < 1e-12
    assert _rel(out.coeffs[1].detach(), out2.coeffs[1].detach()) < 1e-12


def _oracle_grads(fn, inputs, weights):
    """d sum_k <W_k, out_k> / d(every input plane) by torch autograd through the oracle."""
    leaves = [[p.clone().requires_grad_() for p in s] for s in inputs]
    out = fn(*leaves)
    loss = sum((o * w).sum() for o, w in zip(out, weights))
    grads = torch.autograd.grad(loss, [p for s in leaves for p in s], allow_unused=True)
    return [o.detach() for o in out], [torch.zeros_like(p) if g is None else g
                                       for g, p in zip(grads, [p for s in leaves for p in s])]


def _coefficient_grads(fn, inputs, weights):
    from polytensors_b200 import PolyTensor

    leaves = [[p.cuda().requires_grad_() for p in s] for s in inputs]
    with PolyTensor.coefficient_autograd(), PolyTensor.plain_range():
        out = fn(*(PolyTensor(tuple(s), requires_grad=False) for s in leaves))
    loss = sum((o * w.cuda()).sum() for o, w in zip(out.coeffs, weights))
    grads = torch.autograd.grad(loss, [p for s in leaves for p in s], allow_unused=True)
    return [o.detach().cpu() for o in out.coeffs], [torch.zeros_like(p).cpu() if g is None else g.cpu()
                                                    for g, p in zip(grads, [p for s in leaves for p in s])]


@pytest.mark.parametrize("causal", [True, False])
def test_coefficient_mode_attention_against_oracle_autograd(causal):
    n, shape = 2, (1, 2, 80, 32)
    inputs = [series(shape, n, 50 + i) for i in range(3)]
    weights = series(shape, n, 59)
    fn_ref = lambda q, k, v: ref.attention(q, k, v, is_causal=causal)
    fn = lambda q, k, v: F.scaled_dot_product_attention(q, k, v, is_causal=causal)
    want_o, want_g = _oracle_grads(fn_ref, inputs, weights)
    got_o, got_g = _coefficient_grads(fn, inputs, weights)
    assert_close(got_o, want_o, 1e-10, "out")
    assert_close(got_g, want_g, 1e-10, "coefficient gradients")


def test_coefficient_mode_matmul_gelu_chain_against_oracle_autograd():
    n = 3
    X, W = series((24, 40), n, 61), series((40, 16), n, 62)
    weights = series((24, 16), n, 63)
    fn_ref = lambda x, w: ref.gelu(ref.poly_matmul(x, w))
    fn = lambda x, w: F.gelu(x @ w)
    want_o, want_g = _oracle_grads(fn_ref, [X, W], weights)
    got_o, got_g = _coefficient_grads(fn, [X, W], weights)
    assert_close(got_o, want_o, 1e-10, "out")
    assert_close(got_g, want_g, 1e-10, "coefficient gradients")


def test_coefficient_mode_without_grad_is_the_plain_result():
    from polytensors_b200 import PolyTensor

    X = series((8, 12), 2, 70)
    with PolyTensor.coefficient_autograd():
        got = torch.exp(poly(X))
    assert all(c.grad_fn is None for c in got.coeffs)
    assert_close([c.cpu() for c in got.coeffs], ref.series_exp(X), 1e-12, "exp")
