"""Composite operations intercepted above autograd (``__torch_function__``).

Mirrors src/polytensors/_decompositions.py:52-99: ``rms_norm``, ``cross_entropy`` and
``scaled_dot_product_attention`` on PolyTensors.  Where the reference runs a degree-1
Triton kernel or decomposes into many series operations, these run one libpolykern
kernel per direction of the pass (any degree), wrapped in an ``autograd.Function``
whose backward is the series backward rule evaluated by a second kernel.
"""

import math

import torch
import torch.nn.functional as F

from . import _kernels as K
from . import _state


def _poly_cls():
    return _state.poly_cls()


def _planes(x, degree):
    P = _poly_cls()
    if isinstance(x, P):
        return list(x.coeffs)
    return [x] + [torch.zeros_like(x) for _ in range(degree)]


def _grad_planes(g, degree, P):
    """Incoming gradient: a PolyTensor, or an ordinary tensor meaning zero higher planes."""
    if isinstance(g, P):
        return list(g.coeffs)
    return [g] + [torch.zeros_like(g) for _ in range(degree)]


def _supported(planes):
    return all(p.is_cuda and p.dtype in (torch.float32, torch.float64, torch.bfloat16, torch.float16)
               for p in planes)


# ======================================================================================
# RMSNorm (src/polytensors/_decompositions.py:14-22, :56-64; src/polytensors/_fused_norm.py)

def _rms_norm_decomposed(input, normalized_shape, weight=None, eps=None):
    dims = tuple(range(-len(normalized_shape), 0))
    if eps is None:
        eps = torch.finfo(input.dtype).eps
    out = input * torch.rsqrt((input * input).mean(dim=dims, keepdim=True) + eps)
    if weight is not None:
        out = out * weight
    return out


class _SeriesRMSNorm(torch.autograd.Function):
    """y = x (*) rsqrt(mean(x (*) x) + eps) (*) w on PolyTensors (wrapper autograd)."""

    @staticmethod
    def forward(ctx, x, weight, shape, eps):
        P = _poly_cls()
        D = x.degree
        cols = math.prod(shape)
        W = _planes(weight, D) if weight is not None else None
        y, rstd = K.rmsnorm_fwd(list(x.coeffs), cols, W, eps)
        ctx.x_planes, ctx.w_planes, ctx.rstd = list(x.coeffs), W, rstd
        ctx.cols, ctx.shape, ctx.eps, ctx.degree = cols, shape, eps, D
        ctx.w_poly = isinstance(weight, P)
        ctx.w_shape = weight.shape if weight is not None else None
        ctx.cls = P
        return P(tuple(y))

    @staticmethod
    def backward(ctx, grad):
        P = ctx.cls
        G = _grad_planes(grad, ctx.degree, P)
        want_dw = ctx.w_planes is not None and ctx.needs_input_grad[1]
        if torch.is_grad_enabled():
            # Further reverse derivatives: differentiable series operations instead of the kernel.
            x = P(tuple(ctx.x_planes))
            g = P(tuple(G))
            dims = tuple(range(-len(ctx.shape), 0))
            w = P(tuple(ctx.w_planes)) if ctx.w_planes is not None else None
            gy = g * w if w is not None else g
            r = torch.rsqrt((x * x).mean(dim=dims, keepdim=True) + ctx.eps)
            dx = gy * r - x * r * r * r * (x * gy).mean(dim=dims, keepdim=True)
            dw = None
            if want_dw:
                lead = tuple(range(x.dim() - len(ctx.shape)))
                dw = (g * (x * r)).sum(dim=lead) if lead else g * (x * r)
            return dx, dw, None, None
        dx, dw = K.rmsnorm_bwd(ctx.x_planes, ctx.cols, ctx.w_planes, G, ctx.rstd, want_dw)
        dw_out = None
        if want_dw:
            dw = [t.view(ctx.w_shape) for t in dw]
            dw_out = P(tuple(dw)) if ctx.w_poly else dw[0]
        return P(tuple(dx)), dw_out, None, None


def rms_norm_eligible(input, shape, weight, eps):
    P = _poly_cls()
    if not isinstance(input, P) or _state.coefficient_autograd.get():
        return False
    if not shape or tuple(input.shape[-len(shape):]) != tuple(shape) or input.numel() == 0:
        return False
    if eps is not None and not isinstance(eps, (float, int)):
        return False
    planes = list(input.coeffs)
    if weight is not None:
        if tuple(weight.shape) != tuple(shape):
            return False
        if isinstance(weight, P):
            if weight.degree != input.degree:
                return False
            planes += list(weight.coeffs)
        else:
            planes.append(weight)
    return _supported(planes) and all(p.dtype == planes[0].dtype for p in planes) and input.degree < 16


def rms_norm(input, normalized_shape, weight=None, eps=None):
    shape = tuple(normalized_shape)
    eps = torch.finfo(input.dtype).eps if eps is None else float(eps)
    if torch.is_grad_enabled() and (input.requires_grad or (weight is not None and weight.requires_grad)):
        return _SeriesRMSNorm.apply(input, weight, shape, eps)
    with torch.no_grad():
        return _SeriesRMSNorm.forward(_NoCtx(), input, weight, shape, eps)


class _NoCtx:
    needs_input_grad = (False, False, False, False)


# ======================================================================================
# Cross entropy (src/polytensors/_decompositions.py:65-79; src/polytensors/_fused_cross_entropy.py)

class _SeriesCrossEntropy(torch.autograd.Function):
    """Per-row cross entropy of a PolyTensor of (N, C) logits (wrapper autograd)."""

    @staticmethod
    def forward(ctx, logits, target, ignore_index, softcap):
        P = _poly_cls()
        Z = list(logits.coeffs)
        loss, stats = K.cross_entropy_fwd(Z, target, ignore_index, softcap)
        ctx.z, ctx.target, ctx.stats = Z, target, stats
        ctx.ignore_index, ctx.softcap, ctx.degree = ignore_index, softcap, logits.degree
        ctx.cls = P
        return P(tuple(loss))

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad):
        P = ctx.cls
        G = _grad_planes(grad, ctx.degree, P)
        dz = K.cross_entropy_bwd(ctx.z, ctx.target, ctx.ignore_index, ctx.softcap, ctx.stats, G)
        return P(tuple(dz)), None, None, None


def cross_entropy_eligible(input, target, weight, reduction, label_smoothing):
    P = _poly_cls()
    if not _state.fused_cross_entropy.get() or _state.coefficient_autograd.get():
        return False
    if not isinstance(input, P) or input.ndim != 2 or input.degree >= 16:
        return False
    if isinstance(target, P) or not isinstance(target, torch.Tensor) or target.dtype != torch.int64:
        return False
    if target.shape != input.shape[:1] or weight is not None or label_smoothing != 0.0:
        return False
    if reduction not in ("none", "mean", "sum"):
        return False
    planes = list(input.coeffs)
    return _supported(planes) and all(p.dtype == planes[0].dtype for p in planes) and target.is_cuda


def fused_cross_entropy(input, target, ignore_index=-100, reduction="mean", softcap=None):
    if torch.is_grad_enabled() and input.requires_grad:
        losses = _SeriesCrossEntropy.apply(input, target, ignore_index, softcap)
    else:
        with torch.no_grad():
            loss, _ = K.cross_entropy_fwd(list(input.coeffs), target, ignore_index, softcap)
        losses = _poly_cls()(tuple(loss))
    if reduction == "none":
        return losses
    total = losses.sum()
    if reduction == "sum":
        return total
    count = (target != ignore_index).sum().to(losses.value.dtype)
    return total / count


def cross_entropy(logits, target, softcap=None, ignore_index=-100, reduction="mean"):
    """PolyTensor.cross_entropy: optional softcap applied inside the fused pass."""
    if cross_entropy_eligible(logits, target, None, reduction, 0.0):
        return fused_cross_entropy(logits, target, ignore_index=ignore_index, reduction=reduction, softcap=softcap)
    logits = logits.to(torch.promote_types(logits.dtype, torch.float32))
    if softcap is not None:
        logits = softcap * torch.tanh(logits / softcap)
    return F.cross_entropy(logits, target, ignore_index=ignore_index, reduction=reduction)


# ======================================================================================
# Linear + cross entropy with chunked logits (a fusion the reference does not have: its fused
# cross entropy, src/polytensors/_fused_cross_entropy.py:131-170, starts from materialised logits)

_LOGITS_CHUNK_BYTES = 1 << 30


class _LinearCrossEntropy(torch.autograd.Function):
    """Per-row cross entropy of ``h W^T`` (series) over row chunks: at most one chunk of logit
    planes exists at a time, in forward and in backward (which recomputes each chunk's logits)."""

    @staticmethod
    def forward(ctx, h, weight, target, ignore_index, softcap, chunk):
        P = _poly_cls()
        D = h.degree
        H = [x.reshape(-1, x.shape[-1]) for x in h.coeffs]
        W = _planes(weight, D)
        R, V = H[0].shape[0], W[0].shape[0]
        cdt = K.compute_dtype(H[0].dtype)
        losses = [torch.empty(R, dtype=cdt, device=H[0].device) for _ in H]
        stats = torch.empty(R, D + 1, dtype=cdt, device=H[0].device)
        t = target.reshape(-1)
        for r0 in range(0, R, chunk):
            r1 = min(R, r0 + chunk)
            z = K.poly_matmul([x[r0:r1] for x in H], [w.t() for w in W])
            loss, st = K.cross_entropy_fwd(z, t[r0:r1], ignore_index, softcap)
            for dst, src in zip(losses, loss):
                dst[r0:r1].copy_(src)
            stats[r0:r1].copy_(st)
            del z
        ctx.H, ctx.W, ctx.target, ctx.stats = H, W, t, stats
        ctx.meta = (ignore_index, softcap, chunk, D, h.shape, isinstance(weight, P), weight.shape, P)
        return P(tuple(losses))

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad):
        ignore_index, softcap, chunk, D, h_shape, w_poly, w_shape, P = ctx.meta
        H, W, t, stats = ctx.H, ctx.W, ctx.target, ctx.stats
        G = _grad_planes(grad, D, P)
        R = H[0].shape[0]
        need_h, need_w = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        dH = [torch.empty_like(x) for x in H] if need_h else None
        dW = [torch.empty(w_shape, dtype=W[0].dtype, device=W[0].device) for _ in W] if need_w else None
        for r0 in range(0, R, chunk):
            r1 = min(R, r0 + chunk)
            Hc = [x[r0:r1] for x in H]
            z = K.poly_matmul(Hc, [w.t() for w in W])
            dz = K.cross_entropy_bwd(z, t[r0:r1], ignore_index, softcap, stats[r0:r1],
                                     [g.expand(R)[r0:r1] for g in G])
            del z
            if need_h:
                K.poly_matmul(dz, W, out=[x[r0:r1] for x in dH])
            if need_w:
                K.poly_matmul([d.t() for d in dz], Hc, out=dW, accumulate=r0 > 0)
        gh = P(tuple(x.view(h_shape) for x in dH)) if need_h else None
        gw = (P(tuple(dW)) if w_poly else dW[0]) if need_w else None
        return gh, gw, None, None, None, None


def linear_cross_entropy_eligible(h, weight, target):
    P = _poly_cls()
    if not isinstance(h, P) or _state.coefficient_autograd.get() or h.degree >= 16 or h.dim() < 1:
        return False
    if isinstance(target, P) or not isinstance(target, torch.Tensor) or target.dtype != torch.int64:
        return False
    if isinstance(weight, P) and weight.degree != h.degree:
        return False
    if weight.dim() != 2 or weight.shape[1] != h.shape[-1] or target.numel() * h.shape[-1] != h.numel():
        return False
    planes = list(h.coeffs) + _planes(weight, h.degree)
    return (_supported(planes) and all(p.dtype == planes[0].dtype for p in planes)
            and planes[0].dtype in (torch.float32, torch.float64) and target.is_cuda)


def linear_cross_entropy(h, weight, target, ignore_index=-100, reduction="mean", softcap=None, chunk_rows=None):
    """Cross entropy of the logits ``h @ weight.T`` (optionally capped as ``softcap * tanh(z / softcap)``)
    without forming all of them: rows go through the linear and the streaming cross-entropy
    kernel in chunks (``chunk_rows``, default: logit planes of at most 1 GiB per chunk), and the
    backward recomputes each chunk's logits.  Same result as
    ``F.cross_entropy(F.linear(h, weight), target, ...)`` on a PolyTensor ``h`` of shape (..., d)
    with targets of shape (...); ``weight`` (V, d) is a PolyTensor of the same degree or an
    ordinary tensor (zero higher coefficients).  reduction: "mean", "sum" or "none"."""
    if reduction not in ("none", "mean", "sum"):
        raise ValueError(f"unsupported reduction {reduction!r}")
    if not linear_cross_entropy_eligible(h, weight, target):
        raise NotImplementedError("linear_cross_entropy: needs a CUDA PolyTensor input (float32 or float64) and "
                                  "int64 targets with one target per row")
    V = weight.shape[0]
    rows = target.numel()
    if chunk_rows is None:
        per_row = (h.degree + 1) * V * h.coeffs[0].element_size()
        chunk_rows = max(128, min(rows, _LOGITS_CHUNK_BYTES // max(per_row, 1)) // 128 * 128)
    chunk_rows = max(1, int(chunk_rows))
    if torch.is_grad_enabled() and (h.requires_grad or weight.requires_grad):
        losses = _LinearCrossEntropy.apply(h, weight, target, int(ignore_index), softcap, chunk_rows)
    else:
        with torch.no_grad():
            losses = _LinearCrossEntropy.forward(_NoCtxLCE(), h, weight, target, int(ignore_index), softcap,
                                                 chunk_rows)
    if reduction == "none":
        return losses
    total = losses.sum()
    if reduction == "sum":
        return total
    count = (target != ignore_index).sum().to(losses.value.dtype)
    return total / count


class _NoCtxLCE:
    needs_input_grad = (False, False, False, False, False, False)


# ======================================================================================
# Attention (src/polytensors/_decompositions.py:28-43, :80-98)

def attention_decomposed(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None,
                         enable_gqa=False):
    """The reference definition of scaled_dot_product_attention in series operations."""
    if dropout_p != 0.0 or enable_gqa:
        raise NotImplementedError("PolyTensor attention supports dropout_p=0 without GQA")
    L, S = query.size(-2), key.size(-2)
    scale = 1 / math.sqrt(query.size(-1)) if scale is None else scale
    scores = (query * scale) @ key.transpose(-2, -1)
    if is_causal:
        keep = torch.ones(L, S, dtype=torch.bool, device=scores.device).tril(diagonal=0)
        scores = scores.masked_fill(~keep, float("-inf"))
    if attn_mask is not None:
        if attn_mask.dtype == torch.bool:
            scores = scores.masked_fill(~attn_mask, float("-inf"))
        else:
            scores = scores + attn_mask
    return torch.softmax(scores, dim=-1) @ value


# ======================================================================================

_RMS_NORM = frozenset((F.rms_norm, torch.rms_norm))
_CROSS_ENTROPY = frozenset((F.cross_entropy,))
_ATTENTION = frozenset((F.scaled_dot_product_attention,))
_CE_ARGS = ("input", "target", "weight", "size_average", "ignore_index", "reduce", "reduction", "label_smoothing")
_SDPA_ARGS = ("query", "key", "value", "attn_mask", "dropout_p", "is_causal", "scale", "enable_gqa")


def maybe_fused(function, args, kwargs):
    """Result of the fused / decomposed rule, or NotImplemented to continue normally."""
    P = _poly_cls()
    if function in _RMS_NORM:
        bound = dict(zip(("input", "normalized_shape", "weight", "eps"), args))
        bound.update(kwargs)
        if not any(isinstance(bound.get(k), P) for k in ("input", "weight")):
            return NotImplemented
        shape = tuple(bound["normalized_shape"])
        if rms_norm_eligible(bound["input"], shape, bound.get("weight"), bound.get("eps")):
            return rms_norm(bound["input"], shape, bound.get("weight"), bound.get("eps"))
        return _rms_norm_decomposed(bound["input"], shape, bound.get("weight"), bound.get("eps"))
    if function in _CROSS_ENTROPY:
        bound = dict(zip(_CE_ARGS, args))
        bound.update(kwargs)
        if bound.get("size_average") is not None or bound.get("reduce") is not None:
            return NotImplemented
        if not cross_entropy_eligible(bound.get("input"), bound.get("target"), bound.get("weight"),
                                      bound.get("reduction", "mean"), bound.get("label_smoothing", 0.0)):
            return NotImplemented
        loss = fused_cross_entropy(bound["input"], bound["target"], ignore_index=bound.get("ignore_index", -100),
                                   reduction=bound.get("reduction", "mean"))
        return loss if loss.dtype == bound["input"].dtype else loss.to(bound["input"].dtype)
    if function in _ATTENTION:
        bound = dict(zip(_SDPA_ARGS, args))
        bound.update(kwargs)
        if not any(isinstance(v, P) for v in bound.values()):
            return NotImplemented
        from . import _attention

        if _attention.eligible(**bound):
            return _attention.attention(**bound)
        return attention_decomposed(**bound)
    return NotImplemented
