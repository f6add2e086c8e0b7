"""Degree-1 parity at the gates of the reference's Triton kernels.

The reference accelerates degree 1 only, with these gates (which this library's kernels cover at
every degree): attention with head dims 16/32/64/128 for float16, bfloat16 and float32 and
16/32/64 for float64 (src/polytensors/_fused_attention.py:200-201, 227-256); cross entropy on
(N, C) float16 / bfloat16 / float32 logits with softcap, ignore_index and none/mean/sum
(src/polytensors/_fused_cross_entropy.py:131-147); RMSNorm up to 8192 elements per row in float16,
bfloat16, float32 and float64 (src/polytensors/_fused_norm.py:11-21); GELU / tanh / sigmoid in the
same four dtypes (src/polytensors/_fused_activation.py:5-24).  Every case here is compared with the
float64 oracle of the reference's plain-range rules on the same dtype-rounded inputs.

Tolerances (max |got - want| / plane max-norm): float64 1e-10 (gradients 1e-9), float32 1e-4,
float16 storage 1e-2, bfloat16 storage 3e-2."""

import pytest
import torch
import torch.nn.functional as F

from gpu_util import assert_close, coeffs, poly, series
from oracle import polyref as ref

pytestmark = pytest.mark.gpu

TOL = {torch.float64: 1e-10, torch.float32: 1e-4, torch.float16: 1e-2, torch.bfloat16: 3e-2}


def _d(planes):
    return [p.double() for p in planes]


ATTN_CASES = [(dt, D) for dt in (torch.float16, torch.bfloat16, torch.float32) for D in (16, 32, 64, 128)] + \
             [(torch.float64, D) for D in (16, 32, 64)]


@pytest.mark.parametrize("dtype,D", ATTN_CASES)
def test_attention_degree1_head_dims(dtype, D):
    from polytensors_b200 import PolyTensor

    causal = D in (16, 64)
    shape = (1, 2, 80, D)
    Q, Kp, V, G = (series(shape, 1, s, dtype) for s in (81, 82, 83, 84))
    fn = lambda q, k, v: ref.attention(q, k, v, is_causal=causal)
    ins = [_d(X) for X in (Q, Kp, V)]
    want_o = fn(*ins)
    want = ref.series_vjp(fn, ins, _d(G))
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        q, k, v = (poly(X, requires_grad=True) for X in (Q, Kp, V))
        o = F.scaled_dot_product_attention(q, k, v, is_causal=causal)
        o.backward(poly(G))
    tol = TOL[dtype]
    assert_close(coeffs(o), want_o, tol, "o")
    for name, t, w in (("dq", q, want[0]), ("dk", k, want[1]), ("dv", v, want[2])):
        assert_close(coeffs(t.grad), w, tol * (10 if dtype == torch.float64 else 1), name)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("reduction", ["none", "mean", "sum"])
def test_cross_entropy_degree1_softcap_strided(dtype, reduction):
    """Strided rows (a column slice of wider planes), softcap 30, ignore_index rows."""
    from polytensors_b200 import PolyTensor

    N, C, cap = 64, 1000, 30.0
    wide = series((N, C + 24), 1, 91, dtype)
    X = [w[:, 8:8 + C] for w in wide]
    target = torch.randint(0, C, (N,), generator=torch.Generator().manual_seed(92))
    target[::9] = -100
    X64 = _d(X)
    capped = lambda Xs: [cap * t for t in ref.activation([p / cap for p in Xs], "tanh")]
    fn = lambda Xs: ref.cross_entropy(capped(Xs), target, reduction=reduction)
    want = fn(X64)
    shape = tuple(want[0].shape)
    G = series(shape, 1, 93, torch.float64) if shape else [torch.tensor(1.25, dtype=torch.float64),
                                                            torch.tensor(-0.5, dtype=torch.float64)]
    want_dx = ref.series_vjp(fn, [X64], G)[0]
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        x = PolyTensor(tuple(w.cuda()[:, 8:8 + C] for w in wide), requires_grad=True)
        ce = PolyTensor.cross_entropy(x, target.cuda(), softcap=cap, reduction=reduction)
        ce.backward(poly(G))
    assert_close(coeffs(ce), want, 1e-4, "loss (float32 accumulation)")
    assert_close(coeffs(x.grad), want_dx, {torch.float16: 2e-3, torch.bfloat16: 2e-2, torch.float32: 1e-4}[dtype],
                 "dx")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32, torch.float64])
@pytest.mark.parametrize("cols", [8192, 100])
def test_rmsnorm_degree1_widths(dtype, cols):
    from polytensors_b200 import PolyTensor

    X = series((6, cols), 1, 101, dtype)
    W = [(1 + 0.02 * torch.randn(cols, generator=torch.Generator().manual_seed(102), dtype=torch.float64)).to(dtype),
         torch.zeros(cols, dtype=dtype)]
    G = series((6, cols), 1, 103, dtype)
    fn = lambda x, w: ref.rms_norm(x, (cols,), w)
    ins = [_d(X), _d(W)]
    want = fn(*ins)
    want_g = ref.series_vjp(fn, ins, _d(G))
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        x, w = poly(X, requires_grad=True), poly(W, requires_grad=True)
        y = F.rms_norm(x, (cols,), w)
        y.backward(poly(G))
    tol = TOL[dtype]
    assert_close(coeffs(y), want, tol, "y")
    assert_close(coeffs(x.grad), want_g[0], tol * (10 if dtype == torch.float64 else 1), "dx")
    assert_close(coeffs(w.grad), want_g[1], tol * (10 if dtype == torch.float64 else 1), "dw")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32, torch.float64])
@pytest.mark.parametrize("kind", ["gelu", "tanh", "sigmoid"])
def test_activations_degree1(dtype, kind):
    from polytensors_b200 import PolyTensor

    X, G = series((3000,), 1, 111, dtype), series((3000,), 1, 112, dtype)
    fn = lambda x: ref.gelu(x) if kind == "gelu" else ref.activation(x, kind)
    want = fn(_d(X))
    want_dx = ref.series_vjp(fn, [_d(X)], _d(G))[0]
    op = {"gelu": F.gelu, "tanh": torch.tanh, "sigmoid": torch.sigmoid}[kind]
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        x = poly(X, requires_grad=True)
        y = op(x)
        y.backward(poly(G))
    tol = TOL[dtype]
    assert_close(coeffs(y), want, tol, "y")
    assert_close(coeffs(x.grad), want_dx, tol * (10 if dtype == torch.float64 else 1), "dx")
