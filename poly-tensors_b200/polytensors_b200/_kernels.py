"""Tensor-level wrappers around the libpolykern C ABI.

Each function takes coefficient planes as CUDA tensors, allocates outputs (and any
workspace) with the PyTorch caching allocator, and enqueues the kernel on the current
CUDA stream.  Unsupported inputs raise ``NotImplementedError``; there is no CPU or
eager-PyTorch fallback.
"""

import torch

from . import _lib

_DTYPE_CODE = {torch.float32: _lib.PK_F32, torch.float64: _lib.PK_F64,
               torch.bfloat16: _lib.PK_BF16, torch.float16: _lib.PK_F16}


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(tensors, what):
    for t in tensors:
        if not t.is_cuda:
            raise NotImplementedError(f"{what}: the polykern kernels need CUDA tensors (no CPU path)")


def _uniform(planes):
    """Planes sharing one stride pattern (the C ABI takes one set of strides per operand)."""
    strides = planes[0].stride()
    if all(p.stride() == strides for p in planes):
        return list(planes)
    return [p.contiguous() for p in planes]


def _complex_from(planes):
    for k, p in enumerate(planes):
        if p.is_complex():
            return k
    return len(planes)


def gemm_dtype(a_planes, b_planes):
    """(dtype code, a_complex_from, b_complex_from, output dtypes) or None if unsupported."""
    P = len(a_planes)
    base = a_planes[0].dtype
    if any(p.dtype != base for p in (*a_planes, *b_planes)):
        # real float64 base with complex128 directions on either operand
        ok = all(p.dtype in (torch.float64, torch.complex128) for p in (*a_planes, *b_planes))
        if not ok or a_planes[0].dtype != torch.float64 or b_planes[0].dtype != torch.float64:
            return None
        acf, bcf = _complex_from(a_planes), _complex_from(b_planes)
        if any(p.dtype != torch.complex128 for p in a_planes[acf:]) or \
           any(p.dtype != torch.complex128 for p in b_planes[bcf:]):
            return None
        outs = [torch.complex128 if (k >= acf or k >= bcf) else torch.float64 for k in range(P)]
        return _lib.PK_C128, acf, bcf, outs
    if base not in _DTYPE_CODE:
        return None
    return _DTYPE_CODE[base], P, P, [base] * P


def poly_matmul(a_planes, b_planes):
    """C_k = sum_{i+j=k} A_i @ B_j for planes of shape (M, K) x (K, N) or (B, M, K) x (B, K, N).

    Mirrors plain_polynomial_product(matrix=True) (src/polytensors/_plain.py:118-128)
    including real-base / complex-direction promotion (src/polytensors/_plain.py:77-80).
    """
    P = len(a_planes)
    if P != len(b_planes) or P == 0:
        raise ValueError("poly_matmul: operands must have the same number of planes")
    if P > _lib.PK_MAX_PLANES:
        raise NotImplementedError(f"poly_matmul: degree {P - 1} exceeds the kernel limit {_lib.PK_MAX_PLANES - 1}")
    _require_cuda((*a_planes, *b_planes), "poly_matmul")
    spec = gemm_dtype(a_planes, b_planes)
    if spec is None:
        raise NotImplementedError(f"poly_matmul: unsupported plane dtypes "
                                  f"{[p.dtype for p in a_planes]} x {[p.dtype for p in b_planes]}")
    code, acf, bcf, out_dtypes = spec
    a_planes, b_planes = _uniform(a_planes), _uniform(b_planes)
    a0, b0 = a_planes[0], b_planes[0]
    if a0.dim() != b0.dim() or a0.dim() not in (2, 3):
        raise NotImplementedError("poly_matmul: expected 2-D or batched 3-D planes")
    batched = a0.dim() == 3
    if batched:
        batch, M, K = a0.shape
        if b0.shape[0] != batch:
            raise ValueError("poly_matmul: batch sizes differ")
        N = b0.shape[2]
        a_bs, a_rs, a_cs = a0.stride()
        b_bs, b_rs, b_cs = b0.stride()
    else:
        batch, (M, K), N = 1, a0.shape, b0.shape[1]
        a_bs, (a_rs, a_cs) = 0, a0.stride()
        b_bs, (b_rs, b_cs) = 0, b0.stride()
    if b0.shape[-2] != K:
        raise ValueError(f"poly_matmul: inner dimensions differ ({K} vs {b0.shape[-2]})")
    shape = (batch, M, N) if batched else (M, N)
    outs = [torch.empty(shape, dtype=dt, device=a0.device) for dt in out_dtypes]
    c_bs, c_rs = (M * N, N)
    lib = _lib.load()
    degree = P - 1
    ws_bytes = lib.pk_poly_gemm_workspace_size(code, degree, batch, M, N, K, acf, bcf)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=a0.device)
    pa, ka = _lib.pointer_array(a_planes)
    pb, kb = _lib.pointer_array(b_planes)
    pc, kc = _lib.pointer_array(outs)
    status = lib.pk_poly_gemm(code, degree, batch, M, N, K,
                              pa, a_bs, a_rs, a_cs, pb, b_bs, b_rs, b_cs, pc, c_bs, c_rs,
                              acf, bcf, ws.data_ptr(), ws.numel(), _stream(a0.device))
    _lib.check(status, "pk_poly_gemm")
    return outs
