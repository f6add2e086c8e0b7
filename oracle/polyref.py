"""CPU oracle for the PolyTensor truncated-Taylor-series hot path.

TEST INFRASTRUCTURE ONLY.  This module is the checker that the CUDA kernels of
``polytensors_b200`` are compared against; only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg may import it.  The product never calls it.

It restates, on CPU PyTorch tensors, the plain-range algorithms of the reference
(samuel-gunn/poly-tensors, ``PolyTensor.plain_range()`` mode).  A series is a list of
coefficient tensors ``[c_0, ..., c_n]``.  Every function cites the reference code it
restates (paths inside that project).  The restatement is pinned against golden
vectors produced by the reference itself (``tests/golden/make_golden.py``).

Backward passes use the identity the reference documents for its fused kernels
(src/polytensors/_fused_attention.py:18-22, docs/api.md:148-153): for a truncated
series map y(t) = f(x(t)) of degree D, coefficient j of the gradient series
J(x(t))^T G(t) equals d/d x_{D-j} of sum_k <G_k, y_{D-k}>.  ``series_vjp`` evaluates
that with torch.autograd on the forward coefficient map.
"""

import math

import torch


# ----------------------------------------------------------------------------------
# Cauchy products and elementary recurrences

def cauchy(a, b, op=None):
    """Truncated product C_k = sum_{i<=k} a_i * b_{k-i}, accumulated left to right
    (src/polytensors/_plain.py:118-128 and :143-150)."""
    op = op or (lambda x, y: x * y)
    out = []
    for k in range(len(a)):
        total = op(a[0], b[k])
        for i in range(1, k + 1):
            total = total + op(a[i], b[k - i])
        out.append(total)
    return out


def _matmul_promoted(x, y):
    # Real base values may carry complex directions (src/polytensors/_plain.py:77-80).
    dtype = torch.promote_types(x.dtype, y.dtype)
    return torch.matmul(x.to(dtype), y.to(dtype))


def poly_matmul(A, B):
    """Polynomial matrix product (src/polytensors/_plain.py:118-128 with matrix=True,
    reached from src/polytensors/_range_ops.py:160-162)."""
    return cauchy(A, B, _matmul_promoted)


def series_exp(X):
    """exp along a series: Y_0 = exp(X_0), Y_k = sum_{i=1..k} (i/k) X_i Y_{k-i}
    (src/polytensors/_plain.py:153-159)."""
    Y = [torch.exp(X[0])]
    for k in range(1, len(X)):
        Y.append(sum((i / k) * X[i] * Y[k - i] for i in range(1, k + 1)))
    return Y


def series_log(X):
    """log along a series with normalised directions (src/polytensors/_plain.py:162-171)."""
    Y = [torch.log(X[0])]
    u = [None] + [x / X[0] for x in X[1:]]
    for k in range(1, len(X)):
        s = u[k]
        for i in range(1, k):
            s = s - (i / k) * Y[i] * u[k - i]
        Y.append(s)
    return Y


def series_rsqrt(X):
    """X^(-1/2) via 2 X Y' + X' Y = 0 (src/polytensors/_series.py:83-96)."""
    Y = [torch.rsqrt(X[0])]
    u = [None] + [x / X[0] for x in X[1:]]
    for k in range(1, len(X)):
        s = ((2 * k - 1) / (2 * k)) * u[1] * Y[k - 1]
        for i in range(2, k + 1):
            s = s + ((2 * k - i) / (2 * k)) * u[i] * Y[k - i]
        Y.append(-s)
    return Y


def series_quotient(A, B):
    """A / B (src/polytensors/_range_ops.py:86-93)."""
    out = []
    for k in range(len(A)):
        r = A[k]
        for i in range(1, k + 1):
            r = r - B[i] * out[k - i]
        out.append(r / B[0])
    return out


# ----------------------------------------------------------------------------------
# Activations (exact GELU, tanh, sigmoid) by Faa di Bruno composition

def _compose(derivs, X):
    """f(X(t)) from f^(j)(X_0), j = 0..D, using powers of h = X - X_0
    (src/polytensors/_plain.py:174-188)."""
    D = len(X) - 1
    if D == 0:
        return [derivs[0]]
    h = [torch.zeros_like(X[1])] + list(X[1:])
    out = [derivs[0]] + [None] * D
    power = h
    fact = 1.0
    for j in range(1, D + 1):
        fact *= j
        coef = derivs[j] / fact
        for k in range(j, D + 1):
            term = coef * power[k]
            out[k] = term if out[k] is None else out[k] + term
        if j < D:
            power = cauchy(power, h)
    return out


def _hermite_prob(x, count):
    """Probabilists' Hermite polynomials He_0..He_{count-1} (src/polytensors/_plain.py:191-196)."""
    vals = [torch.ones_like(x), x]
    for n in range(1, count - 1):
        vals.append(x * vals[n] - n * vals[n - 1])
    return vals[:count]


def gelu_derivatives(x, count, offset=0):
    """d^n/dx^n of x*Phi(x) for n = offset..offset+count-1 (src/polytensors/_plain.py:199-218)."""
    phi = torch.exp(-0.5 * x * x) / math.sqrt(2 * math.pi)
    Phi = 0.5 * (1 + torch.erf(x / math.sqrt(2)))
    he = _hermite_prob(x, offset + count + 1)

    def dPhi(m):
        if m == 0:
            return Phi
        return (-1.0 if (m - 1) % 2 else 1.0) * he[m - 1] * phi

    return [x * Phi if n == 0 else x * dPhi(n) + n * dPhi(n - 1) for n in range(offset, offset + count)]


def _output_poly_derivatives(y, count, offset, g):
    """Derivatives P_n(y) of f with f' = g(f) (src/polytensors/_plain.py:221-243)."""
    poly = [0.0, 1.0]
    polys = [poly]
    for _ in range(offset + count - 1):
        d = [i * c for i, c in enumerate(poly)][1:] or [0.0]
        prod = [0.0] * (len(d) + len(g) - 1)
        for i, a in enumerate(d):
            for j, b in enumerate(g):
                prod[i + j] += a * b
        poly = prod
        polys.append(poly)
    out = []
    for p in polys[offset:offset + count]:
        v = torch.zeros_like(y)
        for c in reversed(p):
            v = v * y + c
        out.append(v)
    return out


def activation(X, kind, derivative_order=0):
    """plain_activation (src/polytensors/_plain.py:246-259)."""
    D = len(X) - 1
    if kind == "gelu":
        d = gelu_derivatives(X[0], D + 1, derivative_order)
    elif kind == "tanh":
        d = _output_poly_derivatives(torch.tanh(X[0]), D + 1, derivative_order, [1.0, 0.0, -1.0])
    elif kind == "sigmoid":
        d = _output_poly_derivatives(torch.sigmoid(X[0]), D + 1, derivative_order, [0.0, 1.0, -1.0])
    else:
        raise ValueError(kind)
    return _compose(d, X)


def gelu(X):
    return activation(X, "gelu")


def gelu_backward(G, X):
    """aten.gelu_backward in plain range: G * gelu'(X) (src/polytensors/_plain.py:310-315)."""
    return cauchy(G, activation(X, "gelu", derivative_order=1))


# ----------------------------------------------------------------------------------
# Softmax family, cross entropy

def softmax_family(X, dim):
    """(softmax, log_softmax, logsumexp keepdim) series (src/polytensors/_plain.py:262-273)."""
    lse0 = torch.logsumexp(X[0], dim=dim, keepdim=True)
    centered = [X[0] - lse0] + list(X[1:])
    E = series_exp(centered)
    Z = [e.sum(dim=dim, keepdim=True) for e in E]
    log_z = series_log(Z)
    log_sm = [torch.log_softmax(X[0], dim=dim)] + [c - l for c, l in zip(centered[1:], log_z[1:])]
    sm = series_exp(log_sm)
    sm[0] = torch.softmax(X[0], dim=dim)
    return sm, log_sm, [lse0] + list(log_z[1:])


def log_softmax_backward(G, Y, dim):
    """_log_softmax_backward_data in plain range (src/polytensors/_plain.py:348-354)."""
    P = series_exp(Y)
    S = [g.sum(dim=dim, keepdim=True) for g in G]
    return [g - p for g, p in zip(G, cauchy(P, S))]


def softmax_backward(G, Y, dim):
    """_softmax_backward_data in plain range (src/polytensors/_plain.py:342-347)."""
    inner = [s.sum(dim=dim, keepdim=True) for s in cauchy(G, Y)]
    return cauchy(Y, [g - i for g, i in zip(G, inner)])


def cross_entropy(X, target, ignore_index=-100, reduction="mean"):
    """F.cross_entropy on (N, C) logits as PyTorch composes it in plain range:
    log_softmax series (src/polytensors/_plain.py:326-332) then per-plane NLL
    (src/polytensors/_dispatch.py:537-543).  Returns the loss series."""
    _, log_sm, _ = softmax_family(X, 1)
    valid = target != ignore_index
    safe = torch.where(valid, target, torch.zeros_like(target))
    picked = [-(ls.gather(1, safe[:, None])[:, 0]) for ls in log_sm]
    losses = [torch.where(valid, p, torch.zeros_like(p)) for p in picked]
    if reduction == "none":
        return losses
    if reduction == "sum":
        return [l.sum() for l in losses]
    count = valid.sum().to(losses[0].dtype)
    return [l.sum() / count for l in losses]


def cross_entropy_backward(X, target, G, ignore_index=-100, reduction="mean"):
    """Gradient series of cross_entropy w.r.t. the logits for the loss-gradient series G
    (scalars for 'mean'/'sum', per-row for 'none'): NLL backward scatters -G to the
    targets (src/polytensors/_dispatch.py:556-562), then _log_softmax_backward_data."""
    _, log_sm, _ = softmax_family(X, 1)
    N, C = X[0].shape
    valid = target != ignore_index
    safe = torch.where(valid, target, torch.zeros_like(target))
    if reduction == "mean":
        scale = 1.0 / valid.sum().to(X[0].dtype)
    else:
        scale = 1.0
    grads = []
    for g in G:
        g = torch.as_tensor(g, dtype=X[0].dtype)
        per_row = (g.expand(N) if g.dim() == 0 else g) * scale
        per_row = torch.where(valid, per_row, torch.zeros_like(per_row))
        gl = torch.zeros(N, C, dtype=X[0].dtype)
        gl.scatter_(1, safe[:, None], -per_row[:, None])
        grads.append(gl)
    return log_softmax_backward(grads, log_sm, 1)


# ----------------------------------------------------------------------------------
# RMSNorm and attention decompositions

def rms_norm(X, normalized_shape, weight=None, eps=None):
    """x * rsqrt(mean(x*x) + eps) * weight as series (src/polytensors/_decompositions.py:14-22).
    ``weight`` is a series or None; eps defaults to finfo(dtype).eps."""
    dims = tuple(range(-len(normalized_shape), 0))
    if eps is None:
        eps = torch.finfo(X[0].dtype).eps
    sq = cauchy(X, X)
    ms = [s.mean(dim=dims, keepdim=True) for s in sq]
    ms = [ms[0] + eps] + ms[1:]
    out = cauchy(X, series_rsqrt(ms))
    if weight is not None:
        out = cauchy(out, weight)
    return out


def attention(Q, K, V, is_causal=False, scale=None, attn_mask=None):
    """Reference SDPA decomposition (src/polytensors/_decompositions.py:28-43):
    softmax((Q*scale) @ K^T masked) @ V, all as series."""
    L, S = Q[0].shape[-2], K[0].shape[-2]
    scale = 1 / math.sqrt(Q[0].shape[-1]) if scale is None else scale
    scores = cauchy([q * scale for q in Q], [k.transpose(-2, -1) for k in K], _matmul_promoted)
    if is_causal:
        keep = torch.ones(L, S, dtype=torch.bool).tril(0)
        scores = [s.masked_fill(~keep, float("-inf")) if i == 0 else s.masked_fill(~keep, 0.0)
                  for i, s in enumerate(scores)]
    if attn_mask is not None:
        if attn_mask.dtype == torch.bool:
            scores = [s.masked_fill(~attn_mask, float("-inf")) if i == 0 else s.masked_fill(~attn_mask, 0.0)
                      for i, s in enumerate(scores)]
        else:
            scores = [scores[0] + attn_mask] + scores[1:]
    sm, _, _ = softmax_family(scores, -1)
    return cauchy(sm, V, _matmul_promoted)


# ----------------------------------------------------------------------------------
# Series vector-Jacobian products

def series_vjp(fn, inputs, grad_out):
    """Gradient series of ``fn`` at the input series ``inputs`` (a list of series) for the
    output-gradient series ``grad_out``; real coefficients only.

    Returns one gradient series per input, coefficient j being d/d x_{D-j} of
    sum_k <G_k, y_{D-k}> (the swapped-cotangent identity of the module docstring)."""
    leaves = [[c.detach().clone().requires_grad_(True) for c in X] for X in inputs]
    Y = fn(*leaves)
    D = len(Y) - 1
    objective = sum((grad_out[k] * Y[D - k]).sum() for k in range(D + 1))
    flat = [c for X in leaves for c in X]
    grads = torch.autograd.grad(objective, flat, allow_unused=True)
    out, pos = [], 0
    for X in leaves:
        g = [grads[pos + i] if grads[pos + i] is not None else torch.zeros_like(X[i]) for i in range(len(X))]
        pos += len(X)
        out.append([g[D - j] for j in range(D + 1)])
    return out


# ----------------------------------------------------------------------------------
# Comparison metrics used by the parity tests

def plane_errors(got, ref):
    """Per coefficient plane: max |got - ref| / max |ref| (the tolerance metric for float32)."""
    errs = []
    for g, r in zip(got, ref):
        g = g.detach().to("cpu", torch.complex128 if (g.is_complex() or r.is_complex()) else torch.float64)
        r = r.detach().to("cpu", g.dtype)
        denom = r.abs().max().item() if r.numel() else 0.0
        diff = (g - r).abs().max().item() if r.numel() else 0.0
        errs.append(diff / denom if denom > 0 else diff)
    return errs


def rel_errors(got, ref):
    """Per coefficient plane: max |got - ref| / max |ref| computed in float64/complex128
    (the relative metric used for float64 and complex128; identical formula)."""
    return plane_errors(got, ref)
