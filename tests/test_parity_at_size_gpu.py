"""Parity at the configurations' own sizes (configs[1-3] of the benchmark), against the CPU
oracle in float64.

Accumulation error grows with the reduction length, so the small-shape parity tests do not
cover the benchmark shapes.  Where the full oracle would take minutes on the host, the check
is row-sampled: a seeded random set of rows of A (or of the query/batch rows) through the
oracle, compared with the same rows of the GPU result; every row of the product depends on all
of B and all of K, so the sample sees the full reduction.  Tolerances (per coefficient plane,
max|gpu - oracle| / max|oracle|): float32 1e-4, float64 / complex128 1e-10 (the north-star
bounds); bf16 storage 2e-2 for attention outputs and 5e-2 for gradients (the reference's own
bf16 bounds, tests/test_fused_kernels.py:64-72).  float64 also gets an elementwise relative
check on the entries that are not small against the plane's largest (|ref| >= 1e-2 max|ref|),
bound 1e-9: the per-plane metric alone would let a relative error hide in small entries.
"""

import math

import pytest
import torch
import torch.nn.functional as F

from gpu_util import assert_close
from oracle import polyref as ref

pytestmark = pytest.mark.gpu


def cuda_series(shape, n, seed, dtype, complex_from=None):
    """Planes generated on the device (seeded): plane k ~ N(0,1)/k!, complex from ``complex_from``."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    out = []
    for k in range(n + 1):
        if complex_from is not None and k >= complex_from:
            re = torch.randn(*shape, generator=g, device="cuda", dtype=torch.float64)
            im = torch.randn(*shape, generator=g, device="cuda", dtype=torch.float64)
            out.append(torch.complex(re, im) / math.factorial(k))
        else:
            out.append((torch.randn(*shape, generator=g, device="cuda", dtype=torch.float32)
                        / math.factorial(k)).to(dtype))
    return out


def sample_rows(M, rows, seed):
    return torch.randperm(M, generator=torch.Generator().manual_seed(seed))[:rows].sort().values


def elementwise_rel(got, want, floor=1e-2):
    """Largest |got - want| / |want| over the entries with |want| >= floor * max|want|, all planes."""
    worst = 0.0
    for g, w in zip(got, want):
        dt = torch.complex128 if (w.is_complex() or g.is_complex()) else torch.float64
        g, w = g.to(dt), w.to(dt)
        big = w.abs() >= floor * w.abs().max()
        if big.any():
            worst = max(worst, ((g - w).abs()[big] / w.abs()[big]).max().item())
    return worst


def check_product(M, n, dtype, tol, rows, complex_from=None, seed=0):
    from polytensors_b200 import _kernels as K

    A = cuda_series((M, M), n, 100 + seed, dtype, complex_from)
    B = cuda_series((M, M), n, 200 + seed, dtype, complex_from)
    C = K.poly_matmul(A, B)
    idx = sample_rows(M, rows, seed)
    cidx = idx.cuda()
    got = [c[cidx].cpu() for c in C]
    del C
    up = torch.complex128 if complex_from is not None else torch.float64
    Ah = [a[cidx].cpu().to(up if a.is_complex() else torch.float64) for a in A]
    Bh = [b.cpu().to(up if b.is_complex() else torch.float64) for b in B]
    del A, B
    torch.cuda.empty_cache()
    want = ref.poly_matmul(Ah, Bh)
    errs = assert_close(got, want, tol, f"{dtype} M=N=K={M} degree {n}")
    print(f"product {dtype} M=N=K={M} degree {n}: plane errors {errs}")
    if dtype == torch.float64:
        rel = elementwise_rel(got, want)
        print(f"  elementwise relative error (entries >= 1e-2 max): {rel}")
        assert rel <= 1e-9
    return errs


@pytest.mark.parametrize("M,n", [(8192, 4), (4096, 2), (8192, 2), (4096, 8), (8192, 8)])
def test_float32_product_at_config_size(M, n):
    """configs[1] float32: the benchmark configuration (8192^3, degree 4), degrees 2 and 8."""
    check_product(M, n, torch.float32, 1e-4, rows=32)


@pytest.mark.parametrize("M,n", [(1024, 2), (1024, 4), (1024, 8), (4096, 2), (4096, 4), (4096, 8), (8192, 2),
                                 (8192, 4)])
def test_float64_product_at_config_size(M, n):
    """configs[1] float64 on the DMMA path."""
    check_product(M, n, torch.float64, 1e-10, rows=64)


@pytest.mark.parametrize("n", [2, 4, 8])
def test_complex_directions_product_at_config_size(n):
    """configs[1] complex128 directions at 4096: real float64 base, complex128 planes k >= 1."""
    check_product(4096, n, torch.float64, 1e-10, rows=64, complex_from=1)


# ----------------------------------------------------------------------------------------
# configs[3] attention: one head at the sequence length of the benchmark

def _host(planes):
    return [p.detach().float().cpu().double() for p in planes]


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-4), (torch.bfloat16, 2e-2)])
def test_attention_forward_at_config_length(dtype, tol):
    """(1, 1, 4096, 128), degree 3, causal, scale 1/sqrt(128): forward through the API."""
    from polytensors_b200 import PolyTensor

    n, shape = 3, (1, 1, 4096, 128)
    Q, Kp, V = (cuda_series(shape, n, s, dtype) for s in (11, 12, 13))
    with torch.no_grad(), PolyTensor.plain_range():
        o = F.scaled_dot_product_attention(*(PolyTensor(tuple(X)) for X in (Q, Kp, V)), is_causal=True)
    want = ref.attention(_host(Q), _host(Kp), _host(V), is_causal=True)
    print(f"attention forward {dtype} L=4096:", assert_close([c.float().cpu() for c in o.coeffs], want, tol, "o"))


@pytest.mark.parametrize("dtype,tol_o,tol_g", [(torch.float32, 1e-4, 1e-4), (torch.bfloat16, 2e-2, 5e-2)])
def test_attention_backward_at_1024(dtype, tol_o, tol_g):
    """(1, 1, 1024, 128), degree 3, causal: forward and backward through the API."""
    from polytensors_b200 import PolyTensor

    n, shape = 3, (1, 1, 1024, 128)
    Q, Kp, V, G = (cuda_series(shape, n, s, dtype) for s in (21, 22, 23, 24))
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        q, k, v = (PolyTensor(tuple(X), requires_grad=True) for X in (Q, Kp, V))
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        o.backward(PolyTensor(tuple(G)))
    fn = lambda a, b, c: ref.attention(a, b, c, is_causal=True)   # noqa: E731
    host = [_host(X) for X in (Q, Kp, V, G)]
    print(f"attention {dtype} L=1024 o:", assert_close([c.float().cpu() for c in o.coeffs], fn(*host[:3]), tol_o, "o"))
    want = ref.series_vjp(fn, host[:3], host[3])
    for name, t, w in (("dq", q, want[0]), ("dk", k, want[1]), ("dv", v, want[2])):
        print(f"  {name}:", assert_close([c.float().cpu() for c in t.grad.coeffs], w, tol_g, name))


def test_attention_f32_training_shape_forward_backward():
    """configs[4]'s attention: float32, head dimension 64, sequence 1024, degree 3, causal, on
    12 heads, forward and backward (the split kernels) against the float64 oracle."""
    from polytensors_b200 import PolyTensor

    n, shape = 3, (1, 12, 1024, 64)
    Q, Kp, V, G = (cuda_series(shape, n, s, torch.float32) for s in (41, 42, 43, 44))
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        q, k, v = (PolyTensor(tuple(X), requires_grad=True) for X in (Q, Kp, V))
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        o.backward(PolyTensor(tuple(G)))
    fn = lambda a, b, c: ref.attention(a, b, c, is_causal=True)   # noqa: E731
    host = [_host(X) for X in (Q, Kp, V, G)]
    print("attention f32 D=64 L=1024 o:", assert_close([c.cpu() for c in o.coeffs], fn(*host[:3]), 1e-4, "o"))
    want = ref.series_vjp(fn, host[:3], host[3])
    for name, t, w in (("dq", q, want[0]), ("dk", k, want[1]), ("dv", v, want[2])):
        print(f"  {name}:", assert_close([c.cpu() for c in t.grad.coeffs], w, 1e-4, name))


# ----------------------------------------------------------------------------------------
# RMSNorm -> GELU -> linear(32000) -> cross entropy, width 4096, degree 4

def test_norm_gelu_linear_ce_chain_at_config_width():
    """256 rows of the configs[2] chain (hidden 4096, vocabulary 32000, degree 4, float32),
    forward and backward through the API, against the oracle's series backward in float64.

    The per-row loss planes (reduction 'none') are checked at 1e-4 of their plane max-norm.  The
    mean loss is a scalar per plane whose value can be far smaller than its terms (the mean of
    256 row losses of both signs), so its error is measured against the same per-row max-norm:
    the scale of the numbers being averaged."""
    from polytensors_b200 import PolyTensor

    n, R, H, V = 4, 256, 4096, 32000
    X = cuda_series((R, H), n, 31, torch.float32)
    g = torch.Generator().manual_seed(32)
    w0 = 1 + 0.02 * torch.randn(H, generator=g)
    W0 = 0.02 * torch.randn(V, H, generator=g)
    target = torch.randint(0, V, (R,), generator=g)
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        x = PolyTensor(tuple(X), requires_grad=True)
        w = PolyTensor((w0.cuda(),), degree=n, requires_grad=True)
        W = PolyTensor((W0.cuda(),), degree=n, requires_grad=True)
        logits = F.linear(F.gelu(F.rms_norm(x, (H,), w)), W)
        rows = F.cross_entropy(logits, target.cuda(), reduction="none")
        loss = F.cross_entropy(logits, target.cuda())
        loss.backward()

    def chain(xs, ws, wl, reduction="mean"):
        h = ref.gelu(ref.rms_norm(xs, (H,), ws))
        return ref.cross_entropy(ref.cauchy(h, [t.t() for t in wl], lambda a, b: a @ b), target, reduction=reduction)

    zeros = lambda t: [t.double()] + [torch.zeros_like(t, dtype=torch.float64) for _ in range(n)]   # noqa: E731
    inputs = [_host(X), zeros(w0), zeros(W0)]
    want_rows = chain(*inputs, reduction="none")
    print("chain row losses:", assert_close([c.detach().cpu() for c in rows.coeffs], want_rows, 1e-4, "row losses"))
    want = chain(*inputs)
    for k, (got_k, want_k, rk) in enumerate(zip(loss.coeffs, want, want_rows)):
        err = abs(got_k.item() - want_k.item()) / rk.abs().max().item()
        print(f"  mean loss plane {k}: error / max row loss = {err:.3g}")
        assert err <= 1e-4, (k, err)
    seed = [torch.tensor(1.0, dtype=torch.float64)] + [torch.tensor(0.0, dtype=torch.float64)] * n
    grads = ref.series_vjp(chain, inputs, seed)
    for name, t, wt in (("dx", x, grads[0]), ("dw", w, grads[1]), ("dW", W, grads[2])):
        print(f"  {name}:", assert_close([c.cpu() for c in t.grad.coeffs], wt, 1e-4, name))
