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
(n+1 values per query row) is kept from the forward.  bfloat16 planes (degree <= 3) use the
single-kernel forward (pk_flash_attn_fwd) and a backward over all queries of a block of heads
with the softmax in the score products' epilogue (pk_attn_probs_gemm / pk_attn_dscores_gemm)
and banded gradient products (pk_poly_gemm_banded).  Other dtypes tile the queries under a causal
mask, so that their row-wise softmax passes and products skip the masked half; float32
planes with head dimension 64 (degree <= 3) run the same single-kernel forward and score-epilogue
backward on bf16 hi/lo plane pairs (products as hi*hi + hi*lo + lo*hi, fp32 accumulation); other
float32 shapes tile the queries with Q, K, V, dO split once into hi/lo pairs and probabilities and
score gradients written as pairs by the row kernels, so every product reads its operands in place.
"""

import math

import torch

from . import _kernels as K
from . import _lib
from . import _state

# Bytes of score planes (scores/probabilities and their gradient) alive per head block.
_BLOCK_BYTES = 4 << 30
# The bf16 backward keeps the probability and score-gradient planes of ALL queries of a head
# block (no query tiling; the causal products skip the masked half instead), so it gets more.
_FUSED_BLOCK_BYTES = 16 << 30


def _poly_cls():
    return _state.poly_cls()


def _planes(x, degree, P=None):
    P = P or _poly_cls()
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
    if dtype not in (torch.float32, torch.float64, torch.bfloat16, torch.float16):
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


def _probs(Sc, q_len, scale, causal, shift=0):
    """Scores -> probabilities in place; returns the per-row normaliser statistics.  Row r of
    each matrix is query shift + (r % q_len)."""
    hb, Lq, S = Sc[0].shape
    rows = hb * Lq
    stats = torch.empty(rows, len(Sc), dtype=K.compute_dtype(Sc[0].dtype), device=Sc[0].device)
    ps, keep = _lib.pointer_array(Sc)
    status = _lib.load().pk_attn_probs(K.dtype_code(Sc[0].dtype), len(Sc) - 1, rows, S, q_len, ps, S, float(scale),
                                       1 if causal else 0, shift, ps, S, stats.data_ptr(),
                                       K._stream(Sc[0].device))
    _lib.check(status, "pk_attn_probs")
    return stats


def flash_eligible(Q, Kp, V):
    """Whether the single-kernel forward (pk_flash_attn_fwd) applies: bfloat16 planes, degree <= 3,
    head dim 64 or 128 for queries, keys and values alike."""
    D = Q[0].shape[-1]
    return (Q[0].dtype == torch.bfloat16 and len(Q) <= 4 and D in (64, 128)
            and Kp[0].shape[-1] == D and V[0].shape[-1] == D)


def flash_forward(Q, Kp, V, causal, scale, stats=None):
    """O planes; ``stats`` (optional, float32 (BH, L, n+1)) receives each query row's softmax
    normaliser series."""
    BH, L, D = Q[0].shape
    S = Kp[0].shape[1]
    O = [torch.empty_like(q) for q in Q]
    pq, k1 = _lib.pointer_array(Q)
    pk_, k2 = _lib.pointer_array(Kp)
    pv, k3 = _lib.pointer_array(V)
    po, k4 = _lib.pointer_array(O)
    status = _lib.load().pk_flash_attn_fwd(_lib.PK_BF16, len(Q) - 1, BH, L, S, D, pq, pk_, pv, po,
                                           1 if causal else 0, float(scale),
                                           stats.data_ptr() if stats is not None else None, K._stream(Q[0].device))
    _lib.check(status, "pk_flash_attn_fwd")
    return O


def f32_split_eligible(Q, Kp, V):
    """Whether float32 attention runs on the split kernels: float32 planes, degree <= 3, head
    dimension 64 for queries, keys and values.  Q, K, V (and dO) are split once into bf16 hi/lo
    plane pairs; the single-kernel forward and the score-epilogue products evaluate every product
    as hi*hi + hi*lo + lo*hi with fp32 accumulation, and the probability / score-gradient planes
    come out already split, so the gradient products read them in place (pk_poly_gemm_hilo)."""
    return (Q[0].dtype == torch.float32 and len(Q) <= 4 and Q[0].shape[-1] == 64
            and Kp[0].shape[-1] == 64 and V[0].shape[-1] == 64)


def _flash_f32(Q, Kp, V, causal, scale, stats=None):
    """pk_flash_attn_fwd on float32 planes given as hi/lo pairs; float32 O planes."""
    BH, L, D = Q[0].shape
    S = Kp[0].shape[1]
    Qh, Kh, Vh = (K.split_hilo(X) for X in (Q, Kp, V))
    O = [torch.empty_like(q) for q in Q]
    pq, k1 = _lib.pointer_array(Qh)
    pk_, k2 = _lib.pointer_array(Kh)
    pv, k3 = _lib.pointer_array(Vh)
    po, k4 = _lib.pointer_array(O)
    status = _lib.load().pk_flash_attn_fwd(_lib.PK_F32, len(Q) - 1, BH, L, S, D, pq, pk_, pv, po,
                                           1 if causal else 0, float(scale),
                                           stats.data_ptr() if stats is not None else None, K._stream(Q[0].device))
    _lib.check(status, "pk_flash_attn_fwd")
    return O


def fused_backward_eligible(Q, Kp, V):
    """Whether the backward builds probabilities and score gradients in the epilogue of their
    products (pk_attn_probs_gemm / pk_attn_dscores_gemm): bfloat16 planes, degree <= 3, head
    dimensions multiples of 8 up to 128 (the flattened planes are contiguous, so every slice is
    aligned)."""
    return (Q[0].dtype == torch.bfloat16 and len(Q) <= 4 and Q[0].shape[-1] % 8 == 0
            and V[0].shape[-1] % 8 == 0 and Q[0].shape[-1] <= 128 and V[0].shape[-1] <= 128)


def _query_tiles(L, S, causal):
    """(start, stop, keys) per query tile: with a causal mask, query tile t only meets the keys up
    to its last query, so tiling the queries skips most of the masked half of the scores."""
    if not causal or L < 512:
        return [(0, L, S)]
    tiles = min(8, L // 256)
    size = -(-L // tiles)
    return [(q0, min(L, q0 + size), min(S, min(L, q0 + size))) for q0 in range(0, L, size)]


def forward_planes(Q, Kp, V, causal, scale, stats=None):
    """O planes (BH, L, Dv) for flattened (BH, T, D) planes; ``stats`` (optional, (BH, L, n+1) in
    the compute dtype) receives each query row's softmax normaliser series."""
    if flash_eligible(Q, Kp, V):
        return flash_forward(Q, Kp, V, causal, scale, stats)
    if f32_split_eligible(Q, Kp, V):
        return _flash_f32(Q, Kp, V, causal, scale, stats)
    if tiled_f32_eligible(Q, Kp, V):
        return _forward_f32_tiled(Q, Kp, V, causal, scale, stats)
    BH, L, _ = Q[0].shape
    S = Kp[0].shape[1]
    hb = _block_heads(L, S, len(Q), Q[0].element_size(), BH)
    outs = [torch.empty(BH, L, V[0].shape[2], dtype=Q[0].dtype, device=Q[0].device) for _ in Q]
    for h0 in range(0, BH, hb):
        h1 = min(BH, h0 + hb)
        for q0, q1, kend in _query_tiles(L, S, causal):
            Sc = K.poly_matmul([q[h0:h1, q0:q1] for q in Q], [k[h0:h1, :kend].transpose(1, 2) for k in Kp])
            st = _probs(Sc, q1 - q0, scale, causal, q0)
            if stats is not None:
                stats[h0:h1, q0:q1].copy_(st.view(h1 - h0, q1 - q0, -1))
            O = K.poly_matmul(Sc, [v[h0:h1, :kend] for v in V])
            for dst, src in zip(outs, O):
                dst[h0:h1, q0:q1].copy_(src)
    return outs


def _score_gemm(name, A, B, out, rows, scale, causal, shift, probs=None, split=False):
    """pk_attn_probs_gemm / pk_attn_dscores_gemm on (hb, M, K) x (hb, K, N) bf16 plane views;
    ``rows``: float32 (hb, M, n+1) view (statistics or dsum) with unit inner strides.  ``causal``:
    False, True, or 2 (causal; tiles lying wholly more than 192 keys past the admissible region are
    left unwritten, for consumers that only read near it).  ``split``: float32 attention, every plane
    list (A, B, out, probs) holding bf16 hi/lo pairs [hi_0, lo_0, hi_1, ...]."""
    code = _lib.PK_F32 if split else _lib.PK_BF16
    degree = len(A) // (2 if split else 1) - 1
    hb, M, Kd = A[0].shape
    N = B[0].shape[2]
    pa, k1 = _lib.pointer_array(A)
    pb, k2 = _lib.pointer_array(B)
    po, k3 = _lib.pointer_array(out)
    a_s, b_s, o_s = A[0].stride(), B[0].stride(), out[0].stride()
    lib = _lib.load()
    stream = K._stream(A[0].device)
    if name == "probs":
        status = lib.pk_attn_probs_gemm(code, degree, hb, M, N, Kd, pa, *a_s, pb, *b_s, po, o_s[0], o_s[1],
                                        rows.data_ptr(), rows.stride(0), float(scale), int(causal), shift,
                                        stream)
    else:
        pp, k4 = _lib.pointer_array(probs)
        p_s = probs[0].stride()
        status = lib.pk_attn_dscores_gemm(code, degree, hb, M, N, Kd, pa, *a_s, pb, *b_s, pp, p_s[0],
                                          p_s[1], rows.data_ptr(), rows.stride(0), float(scale),
                                          int(causal), shift, po, o_s[0], o_s[1], stream)
    _lib.check(status, f"pk_attn_{name}_gemm")
    return out


def _fused_backward(Q, Kp, V, dO, dsum, stats, causal, scale, dQ, dK, dV):
    """bf16 backward over all queries of a head block at a time: probabilities and score gradients
    from the score-epilogue products, then the three gradient products, banded under a causal
    mask (dV = P^T dO and dK = dS^T Q need keys <= queries, k >= m; dQ = dS K needs k <= m), so
    the masked half of the score planes is neither multiplied nor re-read."""
    BH, L, _ = Q[0].shape
    S = Kp[0].shape[1]
    NP = len(Q)
    per_head = 2 * NP * L * S * Q[0].element_size()
    hb = max(1, min(BH, _FUSED_BLOCK_BYTES // max(per_head, 1)))
    lower, upper = (1, 2) if causal else (0, 0)
    # the banded products read the score planes only near the diagonal (k-block rounding), so the
    # score kernels leave the zeros of tiles far above it unwritten
    mode = 2 if causal else 0
    for h0 in range(0, BH, hb):
        hs = slice(h0, min(BH, h0 + hb))
        hbn = hs.stop - hs.start
        Pr = [torch.empty(hbn, L, S, dtype=Q[0].dtype, device=Q[0].device) for _ in Q]
        _score_gemm("probs", [q[hs] for q in Q], [k[hs].transpose(1, 2) for k in Kp], Pr, stats[hs], scale,
                    mode, 0)
        if dV is not None:
            K.poly_matmul([p.transpose(1, 2) for p in Pr], [g[hs] for g in dO], out=[t[hs] for t in dV], band=lower)
        dS = [torch.empty_like(p) for p in Pr]
        _score_gemm("dscores", [g[hs] for g in dO], [v[hs].transpose(1, 2) for v in V], dS, dsum[hs], scale,
                    mode, 0, probs=Pr)
        del Pr
        if dQ is not None:
            K.poly_matmul(dS, [k[hs] for k in Kp], out=[t[hs] for t in dQ], band=upper)
        if dK is not None:
            K.poly_matmul([d.transpose(1, 2) for d in dS], [q[hs] for q in Q], out=[t[hs] for t in dK], band=lower)


def _fused_backward_f32(Q, Kp, V, dO, dsum, stats, causal, scale, dQ, dK, dV):
    """float32 backward (D = 64, degree <= 3) on the split kernels: the structure of the bf16
    backward, with Q, K, V, dO split once into hi/lo pairs, probabilities and score gradients
    written as hi/lo pairs by the score-epilogue products, and the banded gradient products
    reading those pairs in place (pk_poly_gemm_hilo)."""
    BH, L, _ = Q[0].shape
    S = Kp[0].shape[1]
    NP = len(Q)
    per_head = 2 * 2 * NP * L * S * 2   # probability and score-gradient hi/lo pairs, bf16
    hb = max(1, min(BH, _FUSED_BLOCK_BYTES // max(per_head, 1)))
    lower, upper = (1, 2) if causal else (0, 0)
    mode = 2 if causal else 0
    Qh, Kh, Vh, dOh = (K.split_hilo(X) for X in (Q, Kp, V, dO))
    for h0 in range(0, BH, hb):
        hs = slice(h0, min(BH, h0 + hb))
        hbn = hs.stop - hs.start
        # rows padded to a multiple of 8 keys: the gradient products read these planes in place,
        # which needs 16-byte row pitches
        Sp = -(-S // 8) * 8
        Pr = [torch.empty(hbn, L, Sp, dtype=torch.bfloat16, device=Q[0].device)[..., :S] for _ in range(2 * NP)]
        _score_gemm("probs", [q[hs] for q in Qh], [k[hs].transpose(1, 2) for k in Kh], Pr, stats[hs], scale,
                    mode, 0, split=True)
        if dV is not None:
            K.poly_matmul_hilo([p.transpose(1, 2) for p in Pr], True, [g[hs] for g in dOh], True,
                               out=[t[hs] for t in dV], band=lower)
        # the split score gradient is written key-major (coalesced stores): dSt[b][key][query]
        Lp = -(-L // 8) * 8
        dSt = [torch.empty(hbn, S, Lp, dtype=torch.bfloat16, device=Q[0].device)[..., :L] for _ in range(2 * NP)]
        _score_gemm("dscores", [g[hs] for g in dOh], [v[hs].transpose(1, 2) for v in Vh], dSt, dsum[hs], scale,
                    mode, 0, probs=Pr, split=True)
        del Pr
        if dQ is not None:
            K.poly_matmul_hilo([d.transpose(1, 2) for d in dSt], True, [k[hs] for k in Kh], True,
                               out=[t[hs] for t in dQ], band=upper)
        if dK is not None:
            K.poly_matmul_hilo(dSt, True, [q[hs] for q in Qh], True, out=[t[hs] for t in dK], band=lower)


def tiled_f32_eligible(Q, Kp, V):
    """Whether float32 attention outside the split kernels (head dimension other than 64, degree
    up to 7) runs on hi/lo operands: Q, K, V (and dO) split once into bf16 pairs, probabilities and
    score gradients written as pairs by the row kernels (pk_attn_probs_hilo /
    pk_attn_dscores_hilo), every product reading its operands in place (pk_poly_gemm_hilo), so no
    score tile is staged again.  Head dimensions must keep 16-byte row pitches for the pairs."""
    return (Q[0].dtype == torch.float32 and len(Q) <= 8 and Q[0].shape[-1] % 8 == 0
            and Kp[0].shape[-1] % 8 == 0 and V[0].shape[-1] % 8 == 0)


def _tile_heads(tiles, n_planes, heads):
    """Heads per block for the tiled float32 path: a query tile holds float32 scores (reused for
    dP) and two hi/lo pair sets (probabilities, score gradient), 12 bytes per score per plane."""
    per_head = 12 * n_planes * max((q1 - q0) * kend for q0, q1, kend in tiles)
    return max(1, min(heads, _BLOCK_BYTES // max(per_head, 1)))


def _hilo_scores(hb, rows, cols, n_planes, device):
    """2 n_planes bf16 planes (hb, rows, cols) with rows padded to a multiple of 8 columns (16-byte
    pitches for the products that read them in place)."""
    cp = -(-cols // 8) * 8
    return [torch.empty(hb, rows, cp, dtype=torch.bfloat16, device=device)[..., :cols] for _ in range(2 * n_planes)]


def _probs_hilo(Sc, Pr, q_len, scale, causal, shift):
    """float32 scores -> probabilities as hi/lo pairs (pk_attn_probs_hilo); returns the row statistics."""
    hb, Lq, S = Sc[0].shape
    rows = hb * Lq
    stats = torch.empty(rows, len(Sc), dtype=torch.float32, device=Sc[0].device)
    ps, k1 = _lib.pointer_array(Sc)
    pp, k2 = _lib.pointer_array(Pr)
    status = _lib.load().pk_attn_probs_hilo(len(Sc) - 1, rows, S, q_len, ps, Sc[0].stride(1), float(scale),
                                            1 if causal else 0, shift, pp, Pr[0].stride(1), stats.data_ptr(),
                                            K._stream(Sc[0].device))
    _lib.check(status, "pk_attn_probs_hilo")
    return stats


def _forward_f32_tiled(Q, Kp, V, causal, scale, stats=None):
    """float32 forward per block of heads and causal query tile on hi/lo operands: scores
    Q Kᵀ (float32), probabilities as hi/lo pairs, O = P V banded to the admissible keys."""
    BH, L, _ = Q[0].shape
    S = Kp[0].shape[1]
    NP = len(Q)
    Qh, Kh, Vh = (K.split_hilo(X) for X in (Q, Kp, V))
    tiles = _query_tiles(L, S, causal)
    hb = _tile_heads(tiles, NP, BH)
    outs = [torch.empty(BH, L, V[0].shape[2], dtype=torch.float32, device=Q[0].device) for _ in Q]
    for h0 in range(0, BH, hb):
        hs = slice(h0, min(BH, h0 + hb))
        for q0, q1, kend in tiles:
            qs = slice(q0, q1)
            Sc = K.poly_matmul_hilo([q[hs, qs] for q in Qh], True, [k[hs, :kend].transpose(1, 2) for k in Kh], True)
            Pr = _hilo_scores(hs.stop - hs.start, q1 - q0, kend, NP, Q[0].device)
            st = _probs_hilo(Sc, Pr, q1 - q0, scale, causal, q0)
            del Sc
            if stats is not None:
                stats[hs, qs].copy_(st.view(hs.stop - hs.start, q1 - q0, -1))
            K.poly_matmul_hilo(Pr, True, [v[hs, :kend] for v in Vh], True, out=[o[hs, qs] for o in outs],
                               band=2 if causal else 0, band_offset=q0 if causal else 0)
    return outs


def _backward_f32_tiled(Q, Kp, V, dO, dsum, causal, scale, dQ, dK, dV):
    """float32 backward per block of heads and causal query tile on hi/lo operands: probabilities
    recomputed as hi/lo pairs, dP = dO Vᵀ (float32), the score gradient as hi/lo pairs, and the
    three gradient products banded to the admissible keys."""
    BH, L, _ = Q[0].shape
    S = Kp[0].shape[1]
    NP = len(Q)
    Qh, Kh, Vh, dOh = (K.split_hilo(X) for X in (Q, Kp, V, dO))
    tiles = _query_tiles(L, S, causal)
    hb = _tile_heads(tiles, NP, BH)
    for h0 in range(0, BH, hb):
        hs = slice(h0, min(BH, h0 + hb))
        hbn = hs.stop - hs.start
        for t in (dK or []) + (dV or []):
            t[hs].zero_()
        for q0, q1, kend in tiles:
            qs, ks = slice(q0, q1), slice(0, kend)
            lower = dict(band=1, band_offset=-q0) if causal else {}
            upper = dict(band=2, band_offset=q0) if causal else {}
            Sc = K.poly_matmul_hilo([q[hs, qs] for q in Qh], True, [k[hs, ks].transpose(1, 2) for k in Kh], True)
            Pr = _hilo_scores(hbn, q1 - q0, kend, NP, Q[0].device)
            _probs_hilo(Sc, Pr, q1 - q0, scale, causal, q0)
            if dV is not None:
                K.poly_matmul_hilo([p.transpose(1, 2) for p in Pr], True, [g[hs, qs] for g in dOh], True,
                                   out=[t[hs, ks] for t in dV], accumulate=True, **lower)
            dP = K.poly_matmul_hilo([g[hs, qs] for g in dOh], True, [v[hs, ks].transpose(1, 2) for v in Vh], True,
                                    out=Sc)
            dS = _hilo_scores(hbn, q1 - q0, kend, NP, Q[0].device)
            ds_rows = dsum[hs, qs].contiguous()
            pp, k1 = _lib.pointer_array(Pr)
            pd, k2 = _lib.pointer_array(dP)
            po, k3 = _lib.pointer_array(dS)
            status = _lib.load().pk_attn_dscores_hilo(NP - 1, hbn * (q1 - q0), kend, pp, Pr[0].stride(1), pd,
                                                      dP[0].stride(1), ds_rows.data_ptr(), float(scale), po,
                                                      dS[0].stride(1), K._stream(Q[0].device))
            _lib.check(status, "pk_attn_dscores_hilo")
            del Pr, Sc, dP
            if dQ is not None:
                K.poly_matmul_hilo(dS, True, [k[hs, ks] for k in Kh], True, out=[t[hs, qs] for t in dQ], **upper)
            if dK is not None:
                K.poly_matmul_hilo([d.transpose(1, 2) for d in dS], True, [q[hs, qs] for q in Qh], True,
                                   out=[t[hs, ks] for t in dK], accumulate=True, **lower)


def backward_planes(Q, Kp, V, O, dO, causal, scale, need, stats=None):
    BH, L, _ = Q[0].shape
    S = Kp[0].shape[1]
    D = len(Q) - 1
    # dsum[row] = sum_d dO (*) O, as a [rows][n+1] table (one fused row kernel)
    dsum = K.attn_dsum(dO, O).view(BH, L, D + 1)
    dQ = [torch.empty_like(q) for q in Q] if need[0] else None
    dK = [torch.empty_like(k) for k in Kp] if need[1] else None
    dV = [torch.empty_like(v) for v in V] if need[2] else None
    hb = _block_heads(L, S, len(Q), Q[0].element_size(), BH)
    code = K.dtype_code(Q[0].dtype)
    tiles = _query_tiles(L, S, causal)
    fused = stats is not None and fused_backward_eligible(Q, Kp, V)
    if fused:
        _fused_backward(Q, Kp, V, dO, dsum, stats, causal, scale, dQ, dK, dV)
        return dQ, dK, dV
    if stats is not None and f32_split_eligible(Q, Kp, V):
        _fused_backward_f32(Q, Kp, V, dO, dsum, stats, causal, scale, dQ, dK, dV)
        return dQ, dK, dV
    if tiled_f32_eligible(Q, Kp, V):
        _backward_f32_tiled(Q, Kp, V, dO, dsum, causal, scale, dQ, dK, dV)
        return dQ, dK, dV
    for h0 in range(0, BH, hb):
        h1 = min(BH, h0 + hb)
        hs = slice(h0, h1)
        if dK is not None:
            for t in dK:
                t[hs].zero_()
        if dV is not None:
            for t in dV:
                t[hs].zero_()
        for q0, q1, kend in tiles:
            qs, ks = slice(q0, q1), slice(0, kend)
            Pr = K.poly_matmul([q[hs, qs] for q in Q], [k[hs, ks].transpose(1, 2) for k in Kp])
            _probs(Pr, q1 - q0, scale, causal, q0)
            if dV is not None:
                K.poly_matmul([p.transpose(1, 2) for p in Pr], [g[hs, qs] for g in dO],
                              out=[t[hs, ks] for t in dV], accumulate=True)
            dS = K.poly_matmul([g[hs, qs] for g in dO], [v[hs, ks].transpose(1, 2) for v in V])
            rows = (h1 - h0) * (q1 - q0)
            ds_rows = dsum[hs, qs].contiguous()
            pp, k1 = _lib.pointer_array(Pr)
            pd, k2 = _lib.pointer_array(dS)
            status = _lib.load().pk_attn_dscores(code, D, rows, kend, pp, kend, pd, kend, ds_rows.data_ptr(),
                                                 float(scale), pd, kend, K._stream(Q[0].device))
            _lib.check(status, "pk_attn_dscores")
            del Pr
            if dQ is not None:
                K.poly_matmul(dS, [k[hs, ks] for k in Kp], out=[t[hs, qs] for t in dQ])
            if dK is not None:
                K.poly_matmul([d.transpose(1, 2) for d in dS], [q[hs, qs] for q in Q],
                              out=[t[hs, ks] for t in dK], accumulate=True)
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
        stats = None
        if fused_backward_eligible(Q, Kp, V) or f32_split_eligible(Q, Kp, V):
            stats = torch.empty(*Q[0].shape[:2], len(Q), dtype=torch.float32, device=Q[0].device)
        O = forward_planes(Q, Kp, V, causal, scale, stats)
        ctx.saved = (Q, Kp, V, O, stats)
        ctx.meta = (causal, scale, D, query.shape, key.shape, value.shape)
        ctx.poly = tuple(isinstance(t, P) for t in (query, key, value))
        ctx.cls = P
        out_shape = (*query.shape[:-1], value.shape[-1])
        return P(tuple(o.view(out_shape) for o in O))

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad):
        P = ctx.cls
        Q, Kp, V, O, stats = ctx.saved
        causal, scale, D, qs, ks, vs = ctx.meta
        dO = _flat(_planes(grad, D, P), (*qs[:-1], vs[-1]))
        need = tuple(p and n for p, n in zip(ctx.poly, ctx.needs_input_grad[:3]))
        dQ, dK, dV = backward_planes(Q, Kp, V, O, dO, causal, scale, need, stats)
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
