"""Pin the CPU oracle (oracle/polyref.py) against golden vectors produced by the
reference implementation itself (tests/golden/make_golden.py)."""

import math

import pytest
import torch

from oracle import polyref as ref


def assert_series_close(got, want, tol):
    errs = ref.plane_errors(got, want)
    assert len(got) == len(want)
    assert max(errs) <= tol, errs


@pytest.mark.parametrize("name", ["matmul_f64_n2", "matmul_f64_n4", "bmm_f64_n3"])
def test_matmul_forward_backward_f64(golden, name):
    g = golden(name)
    assert_series_close(ref.poly_matmul(g["A"], g["B"]), g["C"], 1e-13)
    dA, dB = ref.series_vjp(ref.poly_matmul, [g["A"], g["B"]], g["G"])
    assert_series_close(dA, g["dA"], 1e-13)
    assert_series_close(dB, g["dB"], 1e-13)


def test_matmul_f32(golden):
    g = golden("matmul_f32_n4")
    assert_series_close(ref.poly_matmul(g["A"], g["B"]), g["C"], 1e-6)
    A64 = [a.double() for a in g["A"]]
    B64 = [b.double() for b in g["B"]]
    assert_series_close(ref.poly_matmul(A64, B64), g["C"], 1e-6)


def test_matmul_complex_directions(golden):
    g = golden("matmul_c128_n2")
    C = ref.poly_matmul(g["A"], g["B"])
    assert C[0].dtype == torch.float64 and C[1].dtype == torch.complex128
    assert_series_close(C, g["C"], 1e-13)


@pytest.mark.parametrize("name,tol", [("rmsnorm_f64_n3", 1e-12), ("rmsnorm_f32_n3", 2e-6)])
def test_rmsnorm(golden, name, tol):
    g = golden(name)
    fn = lambda X, W: ref.rms_norm(X, (32,), W)
    assert_series_close(fn(g["X"], g["W"]), g["Y"], tol)
    dX, dW = ref.series_vjp(fn, [g["X"], g["W"]], g["G"])
    assert_series_close(dX, g["dX"], tol * 10)
    assert_series_close(dW, g["dW"], tol * 10)


def test_gelu(golden):
    g = golden("gelu_f64_n4")
    assert_series_close(ref.gelu(g["X"]), g["Y"], 1e-13)
    assert_series_close(ref.series_vjp(ref.gelu, [g["X"]], g["G"])[0], g["dX"], 1e-12)
    # the explicit plain-range backward rule agrees with the identity
    D = len(g["X"]) - 1
    assert_series_close(ref.gelu_backward(g["G"], g["X"]), g["dX"], 1e-12)


def test_cross_entropy(golden):
    g = golden("ce_f64_n4")
    ce = ref.cross_entropy(g["X"], g["target"])
    assert_series_close(ce, g["CE"], 1e-13)
    n = len(g["X"]) - 1
    lam = [torch.tensor(1.0, dtype=torch.float64), torch.tensor(-0.5, dtype=torch.float64)] + \
          [torch.tensor(0.0, dtype=torch.float64)] * (n - 1)
    assert_series_close(ref.cauchy(ce, lam), g["loss"], 1e-13)
    # d loss / d logits: the loss-gradient series seeding is (1, 0, ...) times (1 - 0.5 Z)
    dX = ref.cross_entropy_backward(g["X"], g["target"], lam)
    assert_series_close(dX, g["dX"], 1e-12)


def test_cross_entropy_none(golden):
    g = golden("ce_none_f64_n4")
    assert_series_close(ref.cross_entropy(g["X"], g["target"], reduction="none"), g["CE"], 1e-13)
    dX = ref.cross_entropy_backward(g["X"], g["target"], g["G"], reduction="none")
    assert_series_close(dX, g["dX"], 1e-12)
    fn = lambda X: ref.cross_entropy(X, g["target"], reduction="none")
    assert_series_close(ref.series_vjp(fn, [g["X"]], g["G"])[0], g["dX"], 1e-12)


@pytest.mark.parametrize("name,kw", [("attn_causal_f64_n3", dict(is_causal=True)),
                                     ("attn_full_f64_n3", dict(scale=0.3))])
def test_attention(golden, name, kw):
    g = golden(name)
    fn = lambda Q, K, V: ref.attention(Q, K, V, **kw)
    assert_series_close(fn(g["Q"], g["K"], g["V"]), g["O"], 1e-12)
    dQ, dK, dV = ref.series_vjp(fn, [g["Q"], g["K"], g["V"]], g["G"])
    assert_series_close(dQ, g["dQ"], 1e-11)
    assert_series_close(dK, g["dK"], 1e-11)
    assert_series_close(dV, g["dV"], 1e-11)


def test_series_ops(golden):
    g = golden("series_ops_f64_n5")
    X, Xp, Y, Yp = g["X"], g["Xp"], g["Y"], g["Yp"]
    checks = {
        "mul": ref.cauchy(X, Y),
        "div": ref.series_quotient(X, Yp),
        "add": [x + 2.5 * y for x, y in zip(X, Y)],
        "exp": ref.series_exp(X),
        "log": ref.series_log(Xp),
        "rsqrt": ref.series_rsqrt(Xp),
        "tanh": ref.activation(X, "tanh"),
        "sigmoid": ref.activation(X, "sigmoid"),
        "gelu": ref.gelu(X),
        "softmax": ref.softmax_family(X, -1)[0],
        "log_softmax": ref.softmax_family(X, -1)[1],
        "sum1": [x.sum(dim=1) for x in X],
        "mean0": [x.mean(dim=0) for x in X],
        "square": ref.cauchy(X, X),
    }
    for key, got in checks.items():
        assert_series_close(got, g[key], 1e-12)


def test_series_ops_complex_directions(golden):
    """The oracle's series rules on a real base with complex128 directions against the reference's
    own results (tests/golden/series_ops_c128_n3.pt): plane dtypes and values."""
    g = golden("series_ops_c128_n3")
    X, Xp, Y, Yp, R = g["X"], g["Xp"], g["Y"], g["Yp"], g["R"]
    checks = {
        "mul": ref.cauchy(X, Y), "mul_real": ref.cauchy(X, R), "div": ref.series_quotient(X, Yp),
        "add": [x + 2.5 * y for x, y in zip(X, Y)], "sub_real": [r - x for r, x in zip(R, X)],
        "scale_complex": [x * (0.5 - 1.5j) for x in X], "exp": ref.series_exp(X), "log": ref.series_log(Xp),
        "rsqrt": ref.series_rsqrt(Xp), "reciprocal": ref.series_quotient([torch.ones_like(Xp[0])] +
                                                                        [torch.zeros_like(t) for t in Xp[1:]], Xp),
        "tanh": ref.activation(X, "tanh"), "sigmoid": ref.activation(X, "sigmoid"), "gelu": ref.gelu(X),
        "square": ref.cauchy(X, X), "sum1": [x.sum(dim=1) for x in X], "mean0": [x.mean(dim=0) for x in X],
    }
    for key, got in checks.items():
        assert_series_close(got, g[key], 1e-12)
    assert g["mul"][0].dtype == torch.float64 and all(c.dtype == torch.complex128 for c in g["mul"][1:])


def test_bench_readme_fit_oracle_matches_the_reference_run(golden):
    """bench.py's configs[0] CPU leg (the README fit through the oracle) reproduces the reference's
    own README run (tests/golden/readme_fit_plain.pt): the seeded data follow the README's draws."""
    import bench

    g = golden("readme_fit_plain")
    data = bench.readme_fit_data()
    assert torch.equal(data[0], g["X"]) and torch.equal(data[3], g["Y_prime"])
    for dtype in (torch.float32, torch.float64):   # the fixture is the reference's float32 run
        w, c = bench.oracle_readme_fit(data, dtype)
        assert max(ref.plane_errors(w, g["w"])) <= 1e-5, dtype
        assert max(ref.plane_errors(c, g["c"])) <= 1e-5, dtype


def test_series_rules_and_backward_rules(golden):
    """sqrt, reciprocal, an integer power and the backward rules of tanh, sigmoid, GELU, softmax
    and log-softmax against the reference's own plain-range run (tests/golden/
    series_rules_bwd_f64_n4.pt: y.backward(G) for every rule)."""
    g = golden("series_rules_bwd_f64_n4")
    X, Xp, G = g["X"], g["Xp"], g["G"]
    one = [torch.ones_like(Xp[0])] + [torch.zeros_like(t) for t in Xp[1:]]
    sm, lsm, _ = ref.softmax_family(X, -1)
    checks = {
        "sqrt": ref.series_exp([0.5 * t for t in ref.series_log(Xp)]),
        "reciprocal": ref.series_quotient(one, Xp),
        "cube": ref.cauchy(ref.cauchy(X, X), X),
        "d_tanh": ref.cauchy(G, ref.activation(X, "tanh", derivative_order=1)),
        "d_sigmoid": ref.cauchy(G, ref.activation(X, "sigmoid", derivative_order=1)),
        "d_gelu": ref.gelu_backward(G, X),
        "d_softmax": ref.softmax_backward(G, sm, -1),
        "d_log_softmax": ref.log_softmax_backward(G, lsm, -1),
    }
    for key, got in checks.items():
        assert_series_close(got, g[key], 1e-12)


def test_softcap_cross_entropy_sum_and_embedding(golden):
    """PolyTensor.cross_entropy with a softcap and reduction 'sum', and F.embedding with
    padding_idx, forward and backward, against the reference's own plain-range run
    (tests/golden/ce_softcap_embedding_f64_n3.pt)."""
    g = golden("ce_softcap_embedding_f64_n3")
    X, target, G, W, idx, GE = g["X"], g["target"], g["G"], g["W"], g["idx"], g["GE"]
    cap = 5.0

    def capped_loss(Xs):
        capped = [cap * t for t in ref.activation([p / cap for p in Xs], "tanh")]
        return ref.cross_entropy(capped, target, reduction="sum")

    assert_series_close(capped_loss(X), g["softcap_sum"], 1e-12)
    assert_series_close(ref.series_vjp(capped_loss, [X], G)[0], g["d_softcap_sum"], 1e-12)
    assert_series_close([w[idx] for w in W], g["embedding"], 1e-12)
    want = []
    for ge in GE:
        d = torch.zeros_like(W[0]).index_add_(0, idx.reshape(-1), ge.reshape(-1, W[0].shape[1]))
        d[0] = 0.0   # padding_idx rows get no gradient
        want.append(d)
    assert_series_close(want, g["d_embedding"], 1e-12)
