"""Parity of the series kernels, reached through the PolyTensor API, with the reference's
own outputs (golden vectors) and the CPU oracle.

Tolerances, per coefficient plane (max |got - want| / max |want|): float64 1e-10,
float32 1e-4."""

import pytest
import torch
import torch.nn.functional as F

from gpu_util import assert_close, coeffs, cuda, poly, series
from oracle import polyref as ref

pytestmark = pytest.mark.gpu

F64, F32 = 1e-10, 1e-4


def test_elementwise_series_ops_golden(golden):
    from polytensors_b200 import PolyTensor

    g = golden("series_ops_f64_n5")
    x, xp, y, yp = (poly(g[k]) for k in ("X", "Xp", "Y", "Yp"))
    with PolyTensor.plain_range():
        got = {
            "mul": x * y, "div": x / yp, "add": x + 2.5 * y, "exp": torch.exp(x), "log": torch.log(xp),
            "rsqrt": torch.rsqrt(xp), "tanh": torch.tanh(x), "sigmoid": torch.sigmoid(x), "gelu": F.gelu(x),
            "softmax": torch.softmax(x, dim=-1), "log_softmax": torch.log_softmax(x, dim=-1),
            "sum1": x.sum(dim=1), "mean0": x.mean(dim=0), "square": x.square(),
        }
    for key, value in got.items():
        assert_close(coeffs(value), g[key], F64, key)


@pytest.mark.parametrize("precision", ["f64", "f32"])
def test_complex_direction_series_ops_golden(golden, precision):
    """Elementwise rules, sums and products on a real base with complex directions
    (pk_series_map_complex) against the reference's own results: plane dtypes as the reference
    gives them (real base, complex directions) and values within 1e-10 (float64 / complex128) or
    1e-4 (float32 / complex64 inputs)."""
    from polytensors_b200 import PolyTensor

    g = golden("series_ops_c128_n3")
    tol = F64 if precision == "f64" else F32

    def dev(planes):
        if precision == "f32":
            planes = [p.to(torch.complex64 if p.is_complex() else torch.float32) for p in planes]
        return poly(planes)

    x, xp, y, yp, r = (dev(g[k]) for k in ("X", "Xp", "Y", "Yp", "R"))
    with PolyTensor.plain_range():
        got = {
            "mul": x * y, "mul_real": x * r, "div": x / yp, "add": x + 2.5 * y, "sub_real": r - x,
            "scale_complex": x * (0.5 - 1.5j), "exp": torch.exp(x), "log": torch.log(xp), "sqrt": torch.sqrt(xp),
            "rsqrt": torch.rsqrt(xp), "reciprocal": torch.reciprocal(xp), "tanh": torch.tanh(x),
            "sigmoid": torch.sigmoid(x), "gelu": F.gelu(x), "square": x.square(), "sum1": x.sum(dim=1),
            "mean0": x.mean(dim=0),
        }
    for key, value in got.items():
        want = g[key]
        assert [c.is_complex() for c in value.coeffs] == [c.is_complex() for c in want], key
        assert_close([c.to(torch.complex128) for c in coeffs(value)], [c.to(torch.complex128) for c in want],
                     tol, key)


def test_complex_directions_embedding_and_inplace_rules():
    """Row gathers and their backward move complex planes as (re, im) pairs; an in-place update of a
    real series with a complex one raises like the reference."""
    from polytensors_b200 import PolyTensor

    gen = torch.Generator().manual_seed(3)
    base = torch.randn(10, 6, generator=gen, dtype=torch.float64)
    dirs = [torch.complex(torch.randn(10, 6, generator=gen, dtype=torch.float64),
                          torch.randn(10, 6, generator=gen, dtype=torch.float64)) for _ in range(2)]
    w = PolyTensor(tuple(t.cuda() for t in [base] + dirs), requires_grad=True)
    idx = torch.tensor([[1, 4, 4], [9, 0, 2]], device="cuda")
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        e = F.embedding(idx, w)
        for got, plane in zip(e.coeffs, w.coeffs):
            assert got.dtype == plane.dtype and torch.equal(got, plane.detach()[idx])
        e.sum().backward()
    counts = torch.zeros(10, dtype=torch.float64, device="cuda").index_add_(0, idx.reshape(-1),
                                                                           torch.ones(6, dtype=torch.float64,
                                                                                      device="cuda"))
    assert torch.equal(w.grad.coeffs[0], counts[:, None].expand(10, 6))
    real = PolyTensor(tuple(torch.ones(10, 6, dtype=torch.float64, device="cuda") for _ in range(3)))
    with PolyTensor.plain_range(), pytest.raises(RuntimeError, match="complex"):
        real.add_(PolyTensor(tuple(t.cuda() for t in [base] + dirs)))


@pytest.mark.parametrize("n", [1, 3, 8])
def test_elementwise_f32_against_oracle(n):
    from polytensors_b200 import PolyTensor

    X = series((64, 257), n, 1, torch.float32)
    Y = series((64, 257), n, 2, torch.float32)
    Yp = [Y[0].abs() + 0.5] + Y[1:]
    X64, Y64, Yp64 = ([p.double() for p in s] for s in (X, Y, Yp))
    with PolyTensor.plain_range():
        x, y, yp = poly(X), poly(Y), poly(Yp)
        checks = [
            (x * y, ref.cauchy(X64, Y64)), (x / yp, ref.series_quotient(X64, Yp64)),
            (torch.exp(x), ref.series_exp(X64)), (torch.tanh(x), ref.activation(X64, "tanh")),
            (torch.sigmoid(x), ref.activation(X64, "sigmoid")), (F.gelu(x), ref.gelu(X64)),
            (torch.rsqrt(yp), ref.series_rsqrt(Yp64)), (torch.log(yp), ref.series_log(Yp64)),
            (x.sum(dim=0), [p.sum(dim=0) for p in X64]), (x.mean(), [p.mean() for p in X64]),
            (torch.softmax(x, dim=0), ref.softmax_family(X64, 0)[0]),
            (x ** 3, ref.cauchy(ref.cauchy(X64, X64), X64)),
            (1 - 0.5 * x, [1 - 0.5 * X64[0]] + [-0.5 * p for p in X64[1:]]),
        ]
    for i, (got, want) in enumerate(checks):
        assert_close(coeffs(got), want, F32, f"check {i}")


def test_broadcast_and_inplace_sgd_update():
    from polytensors_b200 import PolyTensor

    X = series((8, 5), 3, 3, torch.float32)
    b = series((5,), 3, 4, torch.float32)
    with PolyTensor.plain_range():
        x, bias = poly(X), poly(b)
        assert_close(coeffs(x + bias), [p + q for p, q in zip(X, b)], 1e-6)
        w = poly(X)
        g = poly(series((8, 5), 3, 5, torch.float32))
        planes_before = [p.data_ptr() for p in w.coeffs]
        w.add_(g, alpha=-0.1)
        assert [p.data_ptr() for p in w.coeffs] == planes_before
        G = series((8, 5), 3, 5, torch.float32)
        assert_close(coeffs(w), [p - 0.1 * q for p, q in zip(X, G)], 1e-6)


def test_matmul_backward_golden(golden):
    from polytensors_b200 import PolyTensor

    for name in ("matmul_f64_n2", "bmm_f64_n3"):
        g = golden(name)
        with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
            a, b = poly(g["A"], requires_grad=True), poly(g["B"], requires_grad=True)
            c = a @ b
            c.backward(poly(g["G"]))
            assert_close(coeffs(c), g["C"], F64, name)
            assert_close(coeffs(a.grad), g["dA"], F64, name + " dA")
            assert_close(coeffs(b.grad), g["dB"], F64, name + " dB")


@pytest.mark.parametrize("name,tol", [("rmsnorm_f64_n3", F64), ("rmsnorm_f32_n3", F32)])
def test_rmsnorm_golden(golden, name, tol):
    from polytensors_b200 import PolyTensor

    g = golden(name)
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        x, w = poly(g["X"], requires_grad=True), poly(g["W"], requires_grad=True)
        y = F.rms_norm(x, (32,), w)
        y.backward(poly(g["G"]))
        assert_close(coeffs(y), g["Y"], tol, "y")
        assert_close(coeffs(x.grad), g["dX"], tol * 10, "dx")
        assert_close(coeffs(w.grad), g["dW"], tol * 10, "dw")


def test_rmsnorm_f32_config_width():
    from polytensors_b200 import PolyTensor

    n, H = 4, 4096
    X = series((64, H), n, 6, torch.float32)
    w0 = 1 + 0.02 * torch.randn(H, generator=torch.Generator().manual_seed(7))
    W = [w0] + [torch.zeros(H) for _ in range(n)]
    G = series((64, H), n, 8, torch.float32)
    X64, W64, G64 = ([p.double() for p in s] for s in (X, W, G))
    fn = lambda Xs, Ws: ref.rms_norm(Xs, (H,), Ws)
    want_y = fn(X64, W64)
    want_dx, want_dw = ref.series_vjp(fn, [X64, W64], G64)
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        x, w = poly(X, requires_grad=True), poly(W, requires_grad=True)
        y = F.rms_norm(x, (H,), w)
        y.backward(poly(G))
    assert_close(coeffs(y), want_y, F32, "y")
    assert_close(coeffs(x.grad), want_dx, F32, "dx")
    assert_close(coeffs(w.grad), want_dw, F32, "dw")


@pytest.mark.parametrize("dtype,n,cols,weight", [
    (torch.float32, 4, 4096, "series"), (torch.float32, 5, 2048, "plain"), (torch.float32, 3, 8192, "none"),
    (torch.bfloat16, 4, 4096, "series"), (torch.float16, 2, 1024, "plain"),
    (torch.float32, 1, 4096, "none"), (torch.float32, 1, 4096, "series"), (torch.float32, 0, 1000, "plain"),
    (torch.bfloat16, 1, 2048, "series"), (torch.float32, 1, 1001, "series")])
def test_rmsnorm_backward_many_rows(dtype, n, cols, weight):
    """More rows than clusters fit on the GPU at once (each cluster streams a run of rows), rows
    strided inside a wider buffer, a weight series with non-zero directions, a plain weight, none."""
    from polytensors_b200 import PolyTensor

    rows, tol = 1000, {torch.float32: F32, torch.bfloat16: 2e-2, torch.float16: 2e-3}[dtype]
    X = series((rows, cols + 64), n, 21, dtype)
    G = series((rows, cols), n, 22, dtype)
    gw = torch.Generator().manual_seed(23)
    W = [(1 + 0.1 * torch.randn(cols, generator=gw, dtype=torch.float64)).to(dtype)]
    W += [(0.1 * torch.randn(cols, generator=gw, dtype=torch.float64) / (k + 1)).to(dtype) if weight == "series"
          else torch.zeros(cols, dtype=dtype) for k in range(n)]
    d64 = lambda s: [p.double() for p in s]
    X64 = [p[:, :cols].double() for p in X]
    eps = torch.finfo(dtype).eps  # F.rms_norm's default for these planes
    fn = ((lambda x, w: ref.rms_norm(x, (cols,), w, eps)) if weight != "none"
          else (lambda x: ref.rms_norm(x, (cols,), None, eps)))
    ins = [X64] + ([d64(W)] if weight != "none" else [])
    want_y = fn(*ins)
    want_g = ref.series_vjp(fn, ins, d64(G))
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        x = PolyTensor(tuple(p.cuda()[:, :cols] for p in X), requires_grad=True)
        if weight == "series":
            w = poly(W, requires_grad=True)
        elif weight == "plain":
            w = W[0].cuda()
        else:
            w = None
        y = F.rms_norm(x, (cols,), w)
        y.backward(poly(G))
    assert_close(coeffs(y), want_y, tol, "y")
    assert_close(coeffs(x.grad), want_g[0], tol, "dx")
    if weight == "series":
        assert_close(coeffs(w.grad), want_g[1], tol, "dw")


def test_gelu_golden(golden):
    from polytensors_b200 import PolyTensor

    g = golden("gelu_f64_n4")
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        x = poly(g["X"], requires_grad=True)
        y = F.gelu(x)
        y.backward(poly(g["G"]))
    assert_close(coeffs(y), g["Y"], F64)
    assert_close(coeffs(x.grad), g["dX"], F64)


def test_cross_entropy_golden(golden):
    from polytensors_b200 import PolyTensor

    g = golden("ce_f64_n4")
    n = len(g["X"]) - 1
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        Z = PolyTensor((torch.tensor(0.0, dtype=torch.float64, device="cuda"), 1.0), degree=n)
        x = poly(g["X"], requires_grad=True)
        ce = F.cross_entropy(x, g["target"].cuda())
        loss = ce * (1 - 0.5 * Z)
        loss.backward()
    assert_close(coeffs(ce), g["CE"], F64, "ce")
    assert_close(coeffs(loss), g["loss"], F64, "loss")
    assert_close(coeffs(x.grad), g["dX"], F64, "dx")
    g = golden("ce_none_f64_n4")
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        x = poly(g["X"], requires_grad=True)
        per_row = F.cross_entropy(x, g["target"].cuda(), reduction="none")
        per_row.backward(poly(g["G"]))
    assert_close(coeffs(per_row), g["CE"], F64, "ce none")
    assert_close(coeffs(x.grad), g["dX"], F64, "dx none")


def test_cross_entropy_unfused_path_matches(golden):
    from polytensors_b200 import PolyTensor

    g = golden("ce_f64_n4")
    with PolyTensor.plain_range(), PolyTensor.fused_cross_entropy(False), PolyTensor.retain_wrappers():
        x = poly(g["X"], requires_grad=True)
        ce = F.cross_entropy(x, g["target"].cuda())
        ce.backward()
    assert_close(coeffs(ce), g["CE"], F64, "ce")
    lam = [torch.tensor(1.0, dtype=torch.float64)] + [torch.tensor(0.0, dtype=torch.float64)] * (len(g["X"]) - 1)
    want = ref.cross_entropy_backward(g["X"], g["target"], lam)
    assert_close(coeffs(x.grad), want, F64, "dx")


def test_cross_entropy_f32_vocab_and_softcap():
    from polytensors_b200 import PolyTensor

    n, N, C = 4, 96, 32000
    X = series((N, C), n, 9, torch.float32)
    target = torch.randint(0, C, (N,), generator=torch.Generator().manual_seed(10))
    target[::7] = -100
    X64 = [p.double() for p in X]
    want = ref.cross_entropy(X64, target)
    lam = [torch.tensor(1.0, dtype=torch.float64)] + [torch.tensor(0.0, dtype=torch.float64)] * n
    want_dx = ref.cross_entropy_backward(X64, target, lam)
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        x = poly(X, requires_grad=True)
        ce = F.cross_entropy(x, target.cuda())
        ce.backward()
    assert_close(coeffs(ce), want, F32, "ce")
    assert_close(coeffs(x.grad), want_dx, F32, "dx")
    # softcap: the cap is a series tanh applied before the loss
    cap = 30.0
    capped = [cap * t for t in ref.activation([p / cap for p in X64], "tanh")]
    want = ref.cross_entropy(capped, target, reduction="sum")
    fn = lambda Xs: ref.cross_entropy([cap * t for t in ref.activation([p / cap for p in Xs], "tanh")], target,
                                      reduction="sum")
    want_dx = ref.series_vjp(fn, [X64], lam)[0]
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        x = poly(X, requires_grad=True)
        ce = PolyTensor.cross_entropy(x, target.cuda(), softcap=cap, reduction="sum")
        ce.backward()
    assert_close(coeffs(ce), want, F32, "softcap ce")
    assert_close(coeffs(x.grad), want_dx, F32, "softcap dx")


@pytest.mark.parametrize("name,kw", [("attn_causal_f64_n3", dict(is_causal=True)),
                                     ("attn_full_f64_n3", dict(scale=0.3))])
def test_attention_golden(golden, name, kw):
    from polytensors_b200 import PolyTensor

    g = golden(name)
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        q, k, v = (poly(g[key], requires_grad=True) for key in ("Q", "K", "V"))
        o = F.scaled_dot_product_attention(q, k, v, **kw)
        o.backward(poly(g["G"]))
    assert_close(coeffs(o), g["O"], F64, "o")
    assert_close(coeffs(q.grad), g["dQ"], 1e-9, "dq")
    assert_close(coeffs(k.grad), g["dK"], 1e-9, "dk")
    assert_close(coeffs(v.grad), g["dV"], 1e-9, "dv")


def test_embedding_forward_backward():
    from polytensors_b200 import PolyTensor

    n, V, d = 3, 50, 16
    W = series((V, d), n, 11, torch.float32)
    ids = torch.randint(0, V, (4, 7), generator=torch.Generator().manual_seed(12))
    G = series((4, 7, d), n, 13, torch.float32)
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        w = poly(W, requires_grad=True)
        e = F.embedding(ids.cuda(), w)
        e.backward(poly(G))
    assert_close(coeffs(e), [p[ids] for p in W], 1e-7)
    want = [torch.zeros(V, d).index_add_(0, ids.reshape(-1), g.reshape(-1, d)) for g in G]
    assert_close(coeffs(w.grad), want, 1e-6)


@pytest.mark.parametrize("dtype,tol,causal", [(torch.float32, F32, True), (torch.float32, F32, False),
                                              (torch.float64, F64, True), (torch.bfloat16, 3e-2, True)])
def test_attention_against_oracle(dtype, tol, causal):
    from polytensors_b200 import PolyTensor

    n, shape = 3, (2, 3, 200, 64)
    Q, Kp, V, G = (series(shape, n, s, dtype) for s in (21, 22, 23, 24))
    ref64 = [[p.double() for p in s] for s in (Q, Kp, V, G)]
    fn = lambda q, k, v: ref.attention(q, k, v, is_causal=causal)
    want_o = fn(*ref64[:3])
    want = ref.series_vjp(fn, ref64[:3], ref64[3])
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        q, k, v = (poly(s, requires_grad=True) for s in (Q, Kp, V))
        o = F.scaled_dot_product_attention(q, k, v, is_causal=causal)
        o.backward(poly(G))
    assert_close(coeffs(o), want_o, tol, "o")
    for name, t, w in (("dq", q, want[0]), ("dk", k, want[1]), ("dv", v, want[2])):
        assert_close(coeffs(t.grad), w, tol * (10 if dtype == torch.float64 else 1), name)


def test_attention_fused_and_decomposed_paths_agree():
    from polytensors_b200 import PolyTensor

    n, shape = 2, (1, 2, 96, 32)
    Q, Kp, V = (series(shape, n, s, torch.float64) for s in (31, 32, 33))
    outs = []
    for enabled in (True, False):
        with PolyTensor.plain_range(), PolyTensor.fused_attention(enabled):
            outs.append(coeffs(F.scaled_dot_product_attention(poly(Q), poly(Kp), poly(V), is_causal=True)))
    assert_close(outs[0], outs[1], F64)


@pytest.mark.parametrize("n,shape,causal", [(3, (2, 3, 300, 128), True), (3, (1, 2, 256, 64), False),
                                            (1, (2, 2, 130, 64), True), (2, (1, 1, 64, 128), True),
                                            (0, (1, 2, 200, 128), False)])
def test_flash_forward_bf16_against_oracle(n, shape, causal):
    """The single-kernel bf16 forward (pk_flash_attn_fwd) against the float64 oracle of the reference
    decomposition on the same bf16-rounded inputs; tolerance 3e-2 of the plane max-norm."""
    from polytensors_b200 import PolyTensor, _attention

    Q, Kp, V = (series(shape, n, s, torch.bfloat16) for s in (41, 42, 43))
    flat = [_attention._flat([p.cuda() for p in X], shape) for X in (Q, Kp, V)]
    assert _attention.flash_eligible(*flat)
    got = _attention.flash_forward(*flat, causal, 1 / shape[-1] ** 0.5)
    want = ref.attention(*[[p.double() for p in X] for X in (Q, Kp, V)], is_causal=causal)
    assert_close([g.view(shape).float() for g in got], want, 3e-2)
    with PolyTensor.plain_range():
        o = F.scaled_dot_product_attention(poly(Q), poly(Kp), poly(V), is_causal=causal)
    assert_close(coeffs(o), want, 3e-2, "through the API")


@pytest.mark.parametrize("dtype,tol", [(torch.float32, F32), (torch.float64, F64), (torch.bfloat16, 3e-2)])
def test_causal_query_tiled_attention_against_oracle(dtype, tol):
    """L >= 512 with a causal mask runs the head-blocked path in query tiles that only meet their
    admissible key prefix (forward and backward)."""
    from polytensors_b200 import PolyTensor

    n, shape = 2, (1, 2, 640, 32)
    Q, Kp, V, G = (series(shape, n, s, dtype) for s in (51, 52, 53, 54))
    ref64 = [[p.double() for p in s] for s in (Q, Kp, V, G)]
    fn = lambda q, k, v: ref.attention(q, k, v, is_causal=True)
    want_o = fn(*ref64[:3])
    want = ref.series_vjp(fn, ref64[:3], ref64[3])
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        q, k, v = (poly(s, requires_grad=True) for s in (Q, Kp, V))
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        o.backward(poly(G))
    assert_close(coeffs(o), want_o, tol, "o")
    for name, t, w in (("dq", q, want[0]), ("dk", k, want[1]), ("dv", v, want[2])):
        assert_close(coeffs(t.grad), w, tol * (10 if dtype == torch.float64 else 1), name)


@pytest.mark.parametrize("n,shape,causal", [(3, (1, 2, 130, 64), False), (2, (2, 1, 200, 128), True),
                                            (1, (1, 3, 96, 64), True), (0, (1, 2, 77, 64), False),
                                            (3, (1, 1, 600, 64), True)])
def test_bf16_backward_with_score_epilogues(n, shape, causal):
    """bf16 backward through pk_attn_probs_gemm / pk_attn_dscores_gemm (probabilities rebuilt from
    the forward's row statistics in the product's epilogue; score gradient likewise), against the
    float64 oracle of the reference decomposition on the same bf16-rounded inputs; tolerance 3e-2
    of the plane max-norm, as for the other bf16 attention paths."""
    from polytensors_b200 import PolyTensor, _attention

    Q, Kp, V, G = (series(shape, n, s, torch.bfloat16) for s in (61, 62, 63, 64))
    flat = [_attention._flat([p.cuda() for p in X], shape) for X in (Q, Kp, V)]
    assert _attention.fused_backward_eligible(*flat)
    ref64 = [[p.double() for p in s] for s in (Q, Kp, V, G)]
    fn = lambda q, k, v: ref.attention(q, k, v, is_causal=causal)
    want_o = fn(*ref64[:3])
    want = ref.series_vjp(fn, ref64[:3], ref64[3])
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        q, k, v = (poly(s, requires_grad=True) for s in (Q, Kp, V))
        o = F.scaled_dot_product_attention(q, k, v, is_causal=causal)
        o.backward(poly(G))
    assert_close(coeffs(o), want_o, 3e-2, "o")
    for name, t, w in (("dq", q, want[0]), ("dk", k, want[1]), ("dv", v, want[2])):
        assert_close(coeffs(t.grad), w, 3e-2, name)


def test_far_masked_score_tiles_left_unwritten():
    """causal == 2: the score kernels leave the 64-key tiles lying wholly more than 192 keys past the
    causal boundary of their 128-row tile unwritten, and write every other entry exactly as
    causal == 1 does (zeros included)."""
    from polytensors_b200 import _attention

    n, shape, scale = 3, (1, 2, 1000, 64), 1 / 64 ** 0.5
    Q, Kp = (series(shape, n, s, torch.bfloat16) for s in (81, 82))
    flat = [_attention._flat([p.cuda() for p in X], shape) for X in (Q, Kp)]
    BH, L = flat[0][0].shape[:2]
    V = [torch.zeros_like(q) for q in flat[0]]
    stats = torch.empty(BH, L, n + 1, dtype=torch.float32, device="cuda")
    _attention.flash_forward(flat[0], flat[1], V, True, scale, stats)
    outs = {}
    for mode in (1, 2):
        P = [torch.full((BH, L, L), float("nan"), dtype=torch.bfloat16, device="cuda") for _ in range(n + 1)]
        _attention._score_gemm("probs", flat[0], [k.transpose(1, 2) for k in flat[1]], P, stats, scale, mode, 0)
        outs[mode] = P
    rows = torch.arange(L, device="cuda")
    last_row = torch.clamp(rows // 128 * 128 + 127, max=L - 1)
    far = (rows // 64 * 64)[None, :] > last_row[:, None] + 192
    assert far.any()
    for a, b in zip(outs[1], outs[2]):
        assert not torch.isnan(a).any()
        assert torch.isnan(b[:, far]).all()
        assert torch.equal(b[:, ~far], a[:, ~far])


@pytest.mark.parametrize("shape", [(1, 2, 1000, 64), (2, 2, 700, 128)])
def test_attention_backward_reads_only_written_memory(shape, monkeypatch):
    """Every buffer the attention code allocates starts as NaN, so a read of anything left
    unwritten (the far score tiles above all) would reach the gradients."""
    from polytensors_b200 import PolyTensor, _attention

    real = _attention.torch

    class Poisoned:
        def __getattr__(self, name):
            return getattr(real, name)

        @staticmethod
        def empty(*args, **kw):
            t = real.empty(*args, **kw)
            return t.fill_(float("nan")) if t.is_floating_point() else t

        @staticmethod
        def empty_like(x, *args, **kw):
            t = real.empty_like(x, *args, **kw)
            return t.fill_(float("nan")) if t.is_floating_point() else t

    monkeypatch.setattr(_attention, "torch", Poisoned())
    n = 3
    Q, Kp, V, G = (series(shape, n, s, torch.bfloat16) for s in (91, 92, 93, 94))
    ref64 = [[p.double() for p in s] for s in (Q, Kp, V, G)]
    fn = lambda q, k, v: ref.attention(q, k, v, is_causal=True)
    want = ref.series_vjp(fn, ref64[:3], ref64[3])
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        q, k, v = (poly(s, requires_grad=True) for s in (Q, Kp, V))
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        o.backward(poly(G))
    for name, t, w in (("dq", q, want[0]), ("dk", k, want[1]), ("dv", v, want[2])):
        assert all(torch.isfinite(c).all() for c in coeffs(t.grad)), name
        assert_close(coeffs(t.grad), w, 3e-2, name)


def test_flash_forward_row_statistics():
    """pk_flash_attn_fwd's optional row statistics equal those of pk_attn_probs on the same scores."""
    from polytensors_b200 import _attention, _kernels

    n, shape = 3, (1, 2, 300, 128)
    Q, Kp, V = (series(shape, n, s, torch.bfloat16) for s in (71, 72, 73))
    flat = [_attention._flat([p.cuda() for p in X], shape) for X in (Q, Kp, V)]
    BH, L = flat[0][0].shape[:2]
    stats = torch.empty(BH, L, n + 1, dtype=torch.float32, device="cuda")
    _attention.flash_forward(*flat, True, 1 / 128 ** 0.5, stats)
    Sc = _kernels.poly_matmul([p.float() for p in flat[0]], [k.float().transpose(1, 2) for k in flat[1]])
    want = _attention._probs(Sc, L, 1 / 128 ** 0.5, True).view(BH, L, n + 1)
    torch.testing.assert_close(stats, want, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("n,shape,causal", [(3, (1, 2, 256, 64), True), (3, (2, 2, 600, 64), True),
                                            (2, (1, 3, 200, 64), False), (1, (1, 2, 130, 64), True),
                                            (0, (1, 2, 77, 64), False), (3, (1, 1, 1024, 64), True)])
def test_f32_split_attention_against_oracle(n, shape, causal):
    """float32 attention with head dimension 64 on the split kernels (single-kernel forward,
    score-epilogue backward and hi/lo gradient products), forward and backward against the float64
    oracle of the reference decomposition; tolerance 1e-4 of the plane max-norm."""
    from polytensors_b200 import PolyTensor, _lib

    Q, Kp, V, G = (series(shape, n, s, torch.float32) for s in (81, 82, 83, 84))
    ref64 = [[p.double() for p in s] for s in (Q, Kp, V, G)]
    fn = lambda q, k, v: ref.attention(q, k, v, is_causal=causal)   # noqa: E731
    want_o = fn(*ref64[:3])
    want = ref.series_vjp(fn, ref64[:3], ref64[3])
    for nm in ("flash_attn_fwd", "attn_probs_gemm", "attn_dscores_gemm"):
        _lib.profile_query(nm)
    _lib.profile_enable(True)
    try:
        with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
            q, k, v = (poly(s, requires_grad=True) for s in (Q, Kp, V))
            o = F.scaled_dot_product_attention(q, k, v, is_causal=causal)
            o.backward(poly(G))
        torch.cuda.synchronize()
    finally:
        _lib.profile_enable(False)
    for nm in ("flash_attn_fwd", "attn_probs_gemm", "attn_dscores_gemm"):
        assert _lib.profile_query(nm)[1] > 0, f"{nm} did not run"
    assert_close(coeffs(o), want_o, F32, "o")
    for name, t, w in (("dq", q, want[0]), ("dk", k, want[1]), ("dv", v, want[2])):
        assert_close(coeffs(t.grad), w, F32, name)


@pytest.mark.parametrize("n,shape,causal", [(3, (1, 2, 600, 128), True), (3, (2, 2, 77, 128), False),
                                            (5, (1, 2, 300, 96), True), (4, (1, 3, 520, 64), True),
                                            (7, (1, 1, 130, 32), False)])
def test_f32_tiled_hilo_attention_against_oracle(n, shape, causal):
    """float32 attention outside the split kernels (head dimension other than 64, or degree above
    3) on the tiled path with hi/lo operands: the probability and score-gradient pairs come from
    pk_attn_probs_hilo / pk_attn_dscores_hilo and every product reads its operands in place
    (ragged key counts exercise the padded pair pitches).  Forward and backward against the
    float64 oracle; tolerance 1e-4 of the plane max-norm."""
    from polytensors_b200 import PolyTensor, _attention, _lib

    Q, Kp, V, G = (series(shape, n, s, torch.float32) for s in (91, 92, 93, 94))
    ref64 = [[p.double() for p in s] for s in (Q, Kp, V, G)]
    fn = lambda q, k, v: ref.attention(q, k, v, is_causal=causal)   # noqa: E731
    want_o = fn(*ref64[:3])
    want = ref.series_vjp(fn, ref64[:3], ref64[3])
    flat = [p.cuda().reshape(-1, *shape[-2:]) for p in Q]
    assert _attention.tiled_f32_eligible(flat, flat, flat) and not _attention.f32_split_eligible(flat, flat, flat)
    for nm in ("attn_probs", "attn_dscores", "flash_attn_fwd"):
        _lib.profile_query(nm)
    _lib.profile_enable(True)
    try:
        with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
            q, k, v = (poly(s, requires_grad=True) for s in (Q, Kp, V))
            o = F.scaled_dot_product_attention(q, k, v, is_causal=causal)
            o.backward(poly(G))
        torch.cuda.synchronize()
    finally:
        _lib.profile_enable(False)
    assert _lib.profile_query("attn_probs")[1] > 0 and _lib.profile_query("attn_dscores")[1] > 0
    assert _lib.profile_query("flash_attn_fwd")[1] == 0
    assert_close(coeffs(o), want_o, F32, "o")
    for name, t, w in (("dq", q, want[0]), ("dk", k, want[1]), ("dv", v, want[2])):
        assert_close(coeffs(t.grad), w, F32, name)


@pytest.mark.parametrize("reduction,softcap,dtype,chunk", [("mean", None, torch.float32, 64),
                                                           ("sum", 30.0, torch.float32, 100),
                                                           ("none", None, torch.float64, 50),
                                                           ("mean", None, torch.float32, None)])
def test_linear_cross_entropy_matches_the_unfused_chain(reduction, softcap, dtype, chunk):
    """PolyTensor.linear_cross_entropy (row chunks of the series linear streamed into the
    cross-entropy kernel, logits recomputed in backward) against F.linear + cross entropy through
    the API and, without softcap, against the float64 oracle: loss and the gradients of the input
    and of a weight with nonzero higher coefficients; rows with ignore_index included."""
    from polytensors_b200 import PolyTensor

    n, R, d, V = 3, 300, 96, 1000
    tol = F32 if dtype == torch.float32 else F64
    X = series((R, d), n, 91, dtype)
    W = [w * 0.1 for w in series((V, d), n, 92, dtype)]
    g = torch.Generator().manual_seed(93)
    target = torch.randint(0, V, (R,), generator=g)
    target[::17] = -100
    Gr = series((R,), n, 94, dtype) if reduction == "none" else None

    def run(fused):
        with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
            h, w = poly(X, requires_grad=True), poly(W, requires_grad=True)
            if fused:
                loss = PolyTensor.linear_cross_entropy(h, w, target.cuda(), reduction=reduction, softcap=softcap,
                                                       chunk_rows=chunk)
            else:
                loss = PolyTensor.cross_entropy(F.linear(h, w), target.cuda(), reduction=reduction, softcap=softcap)
            loss.backward(poly(Gr) if Gr is not None else None)
            return coeffs(loss), coeffs(h.grad), coeffs(w.grad)

    got, want = run(True), run(False)
    for a, b, what in zip(got, want, ("loss", "dh", "dW")):
        assert_close(a, b, tol, what)
    if softcap is None:
        fn = lambda x, w: ref.cross_entropy(ref.cauchy(x, [t.t() for t in w], lambda a, b: a @ b), target,
                                            reduction=reduction)   # noqa: E731
        ref64 = [[p.double() for p in X], [p.double() for p in W]]
        out = fn(*ref64)
        seed = [p.double() for p in Gr] if Gr is not None else \
            [torch.tensor(1.0, dtype=torch.float64)] + [torch.tensor(0.0, dtype=torch.float64)] * n
        grads = ref.series_vjp(fn, ref64, seed)
        if reduction == "none":
            assert_close(got[0], out, tol, "loss vs oracle")
        assert_close(got[1], grads[0], tol, "dh vs oracle")
        assert_close(got[2], grads[1], tol, "dW vs oracle")


def test_linear_cross_entropy_keeps_one_logit_chunk():
    """Peak device memory of the fused form stays below one full set of logit planes."""
    from polytensors_b200 import PolyTensor

    n, R, d, V = 3, 4096, 256, 32000
    X = [x.cuda() for x in series((R, d), n, 95, torch.float32)]
    W = torch.randn(V, d, device="cuda") * 0.02
    target = torch.randint(0, V, (R,), device="cuda")
    logits_bytes = (n + 1) * R * V * 4
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        h = PolyTensor(tuple(X), requires_grad=True)
        loss = PolyTensor.linear_cross_entropy(h, W, target, chunk_rows=512)
        loss.backward()
    torch.cuda.synchronize()
    peak = torch.cuda.max_memory_allocated() - base
    assert peak < logits_bytes / 2, (peak, logits_bytes)
    assert torch.isfinite(h.grad.coeffs[0]).all()
