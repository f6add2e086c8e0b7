"""Series attention, ``scaled_dot_product_attention`` on PolyTensors.

Evaluates the reference definition (src/polytensors/_decompositions.py:28-43:
``softmax(scale * Q K^T, masked) V`` with every product a truncated Cauchy product) a
block of heads at a time, so the (L, S) score planes of only that block exist at once:

    scores = Q K^T                  pk_poly_gemm (all n+1 output planes in one launch)
    P      = softmax(scale*scores)  pk_attn_probs (causal mask in-kernel, series normaliser)
    O      = P V                    pk_poly_gemm

and the backward (the series form of the reference's bmm / softmax backward rules):

    dV = P^T dO,  dP = dO V^T,  dS = scale * P (*) (dP - sum_d dO (*) O),
    dQ = dS K,    dK = dS^T Q.

P is recomputed in backward from the saved inputs; only the per-row normaliser series
(n+1 values per query row) is kept from the forward.
"""

import math

import torch

from . import _kernels as K
from . import _lib
from . import _state

# Bytes of score planes (scores/probabilities and their gradient) alive per head block.
_BLOCK_BYTES = 4 << 30


def _poly_cls():
    from ._tensor import PolyTensor

    return PolyTensor


def _planes(x, degree):
    P = _poly_cls()
    if isinstance(x, P):
        return list(x.coeffs)
    return [x] + [torch.zeros_like(x) for _ in range(degree)]


def eligible(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None, enable_gqa=False):
    P = _poly_cls()
    if not _state.fused_attention.get() or _state.coefficient_autograd.get():
        return False
    if dropout_p != 0.0 or enable_gqa or attn_mask is not None:
        return False
    tensors = (query, key, value)
    if not all(isinstance(t, torch.Tensor) for t in tensors):
        return False
    polys = [t for t in tensors if isinstance(t, P)]
    if not polys:
        return False
    degree = polys[0].degree
    if any(p.degree != degree for p in polys) or degree >= _lib.PK_MAX_PLANES:
        return False
    if any(not isinstance(t, P) and t.requires_grad for t in tensors):
        return False
    planes = [c for t in tensors for c in _planes(t, degree)]
    dtype = planes[0].dtype
    if dtype not in (torch.float32, torch.float64, torch.bfloat16):
        return False
    if any(c.dtype != dtype or not c.is_cuda for c in planes):
        return False
    if query.ndim < 3 or key.shape[:-1] != value.shape[:-1] or query.shape[:-2] != key.shape[:-2]:
        return False
    return query.shape[-1] == key.shape[-1]


def _flat(planes, shape):
    return [p.expand(shape).reshape(-1, shape[-2], shape[-1]).contiguous() for p in planes]


def _block_heads(L, S, n_planes, esz, heads):
    per_head = 2 * n_planes * L * S * esz
    return max(1, min(heads, _BLOCK_BYTES // max(per_head, 1)))


def _probs(Sc, L, scale, causal):
    """Scores -> probabilities in place; returns the per-row normaliser statistics."""
    hb, _, S = Sc[0].shape
    rows = hb * L
    stats = torch.empty(rows, len(Sc), dtype=K.compute_dtype(Sc[0].dtype), device=Sc[0].device)
    ps, keep = _lib.pointer_array(Sc)
    status = _lib.load().pk_attn_probs(K.dtype_code(Sc[0].dtype), len(Sc) - 1, rows, S, L, ps, S, float(scale),
                                       1 if causal else 0, 0, ps, S, stats.data_ptr(),
                                       K._stream(Sc[0].device))
    _lib.check(status, "pk_attn_probs")
    return stats


def flash_eligible(Q, Kp, V):
    """Whether the single-kernel forward (pk_flash_attn_fwd) applies: bfloat16 planes, degree <= 3,
    head dim 64 or 128 for queries, keys and values alike."""
    D = Q[0].shape[-1]
    return (Q[0].dtype == torch.bfloat16 and len(Q) <= 4 and D in (64, 128)
            and Kp[0].shape[-1] == D and V[0].shape[-1] == D)


def flash_forward(Q, Kp, V, causal, scale):
    BH, L, D = Q[0].shape
    S = Kp[0].shape[1]
    O = [torch.empty_like(q) for q in Q]
    pq, k1 = _lib.pointer_array(Q)
    pk_, k2 = _lib.pointer_array(Kp)
    pv, k3 = _lib.pointer_array(V)
    po, k4 = _lib.pointer_array(O)
    status = _lib.load().pk_flash_attn_fwd(_lib.PK_BF16, len(Q) - 1, BH, L, S, D, pq, pk_, pv, po,
                                           1 if causal else 0, float(scale), K._stream(Q[0].device))
    _lib.check(status, "pk_flash_attn_fwd")
    return O


def forward_planes(Q, Kp, V, causal, scale):
    """O planes (BH, L, Dv) for flattened (BH, T, D) planes."""
    if flash_eligible(Q, Kp, V):
        return flash_forward(Q, Kp, V, causal, scale)
    BH, L, _ = Q[0].shape
    S = Kp[0].shape[1]
    hb = _block_heads(L, S, len(Q), Q[0].element_size(), BH)
    outs = [torch.empty(BH, L, V[0].shape[2], dtype=Q[0].dtype, device=Q[0].device) for _ in Q]
    for h0 in range(0, BH, hb):
        h1 = min(BH, h0 + hb)
        Sc = K.poly_matmul([q[h0:h1] for q in Q], [k[h0:h1].transpose(1, 2) for k in Kp])
        _probs(Sc, L, scale, causal)
        O = K.poly_matmul(Sc, [v[h0:h1] for v in V])
        for dst, src in zip(outs, O):
            dst[h0:h1].copy_(src)
    return outs


def backward_planes(Q, Kp, V, O, dO, causal, scale, need):
    BH, L, _ = Q[0].shape
    S = Kp[0].shape[1]
    D = len(Q) - 1
    # dsum[row] = sum_d dO (*) O, as a [rows][n+1] table
    prod = K.series_map("mul", D, dO, O)
    if prod[0].dtype in (torch.bfloat16, torch.float16):
        prod = [p.float() for p in prod]
    dsum = torch.stack(K.series_reduce(prod, BH * L, prod[0].shape[-1], 1), dim=-1)
    dsum = dsum.to(K.compute_dtype(Q[0].dtype)).contiguous()
    dQ = [torch.empty_like(q) for q in Q] if need[0] else None
    dK = [torch.empty_like(k) for k in Kp] if need[1] else None
    dV = [torch.empty_like(v) for v in V] if need[2] else None
    hb = _block_heads(L, S, len(Q), Q[0].element_size(), BH)
    code = K.dtype_code(Q[0].dtype)
    for h0 in range(0, BH, hb):
        h1 = min(BH, h0 + hb)
        sl = slice(h0, h1)
        Pr = K.poly_matmul([q[sl] for q in Q], [k[sl].transpose(1, 2) for k in Kp])
        _probs(Pr, L, scale, causal)
        if dV is not None:
            for dst, src in zip(dV, K.poly_matmul([p.transpose(1, 2) for p in Pr], [g[sl] for g in dO])):
                dst[sl].copy_(src)
        dP = K.poly_matmul([g[sl] for g in dO], [v[sl].transpose(1, 2) for v in V])
        rows = (h1 - h0) * L
        pp, k1 = _lib.pointer_array(Pr)
        pd, k2 = _lib.pointer_array(dP)
        status = _lib.load().pk_attn_dscores(code, D, rows, S, pp, S, pd, S, dsum[h0 * L:h1 * L].data_ptr(),
                                             float(scale), pd, S, K._stream(Q[0].device))
        _lib.check(status, "pk_attn_dscores")
        if dQ is not None:
            for dst, src in zip(dQ, K.poly_matmul(dP, [k[sl] for k in Kp])):
                dst[sl].copy_(src)
        if dK is not None:
            for dst, src in zip(dK, K.poly_matmul([d.transpose(1, 2) for d in dP], [q[sl] for q in Q])):
                dst[sl].copy_(src)
    return dQ, dK, dV


class _SeriesAttention(torch.autograd.Function):
    """Series attention on PolyTensors (wrapper autograd)."""

    @staticmethod
    def forward(ctx, query, key, value, causal, scale):
        P = _poly_cls()
        D = next(t for t in (query, key, value) if isinstance(t, P)).degree
        Q = _flat(_planes(query, D), query.shape)
        Kp = _flat(_planes(key, D), key.shape)
        V = _flat(_planes(value, D), value.shape)
        O = forward_planes(Q, Kp, V, causal, scale)
        ctx.saved = (Q, Kp, V, O)
        ctx.meta = (causal, scale, D, query.shape, key.shape, value.shape)
        ctx.poly = tuple(isinstance(t, P) for t in (query, key, value))
        out_shape = (*query.shape[:-1], value.shape[-1])
        return P(tuple(o.view(out_shape) for o in O))

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad):
        P = _poly_cls()
        Q, Kp, V, O = ctx.saved
        causal, scale, D, qs, ks, vs = ctx.meta
        dO = _flat(_planes(grad, D), (*qs[:-1], vs[-1]))
        need = tuple(p and n for p, n in zip(ctx.poly, ctx.needs_input_grad[:3]))
        dQ, dK, dV = backward_planes(Q, Kp, V, O, dO, causal, scale, need)
        grads = []
        for g, shape in ((dQ, qs), (dK, ks), (dV, vs)):
            grads.append(P(tuple(t.view(shape) for t in g)) if g is not None else None)
        return (*grads, None, None)


def attention(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None, enable_gqa=False):
    """scaled_dot_product_attention on PolyTensors (an eligible call, see ``eligible``)."""
    P = _poly_cls()
    scale = 1 / math.sqrt(query.shape[-1]) if scale is None else float(scale)
    if torch.is_grad_enabled() and any(isinstance(t, P) and t.requires_grad for t in (query, key, value)):
        return _SeriesAttention.apply(query, key, value, bool(is_causal), scale)
    with torch.no_grad():
        D = next(t for t in (query, key, value) if isinstance(t, P)).degree
        Q = _flat(_planes(query, D), query.shape)
        Kp = _flat(_planes(key, D), key.shape)
        V = _flat(_planes(value, D), value.shape)
        O = forward_planes(Q, Kp, V, bool(is_causal), scale)
        return P(tuple(o.view(*query.shape[:-1], value.shape[-1]) for o in O))
