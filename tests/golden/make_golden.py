"""Generate golden input/output vectors from the reference implementation itself.

Runs samuel-gunn/poly-tensors (imported from the ``src`` directory of a local checkout,
named by the ``POLYTENSORS_REFERENCE`` environment variable) on small seeded inputs, in
``PolyTensor.plain_range()`` mode unless a case says otherwise, and saves inputs and
outputs to ``tests/golden/*.pt``.  The reference is not needed afterwards: the CPU
tests pin the oracle (``oracle/polyref.py``) against these files and the GPU tests
compare the CUDA kernels against both.

    POLYTENSORS_REFERENCE=<checkout>/src python tests/golden/make_golden.py
"""

import math
import os
import pathlib
import sys

import torch
import torch.nn.functional as F

HERE = pathlib.Path(__file__).resolve().parent
REF = os.environ.get("POLYTENSORS_REFERENCE")
if not REF:
    sys.exit("set POLYTENSORS_REFERENCE to the reference checkout's src directory")
sys.path.insert(0, REF)
from polytensors import PolyTensor  # noqa: E402  (the reference)


def series(shape, n, seed, dtype=torch.float64, complex_from=None):
    g = torch.Generator().manual_seed(seed)
    out = []
    for k in range(n + 1):
        x = torch.randn(*shape, generator=g, dtype=torch.float64) / math.factorial(k)
        if complex_from is not None and k >= complex_from:
            y = torch.randn(*shape, generator=g, dtype=torch.float64) / math.factorial(k)
            x = torch.complex(x, y)
        out.append(x.to(dtype) if not x.is_complex() else x)
    return out


def coeffs(p):
    return [c.detach().clone() for c in p.coeffs]


def grads_of(*polys):
    return [coeffs(p.grad) for p in polys]


def save(name, **data):
    torch.save(data, HERE / f"{name}.pt")
    print("wrote", name)


def case_matmul(name, shape_a, shape_b, n, dtype, seed, backward=True):
    A, B = series(shape_a, n, seed, dtype), series(shape_b, n, seed + 1, dtype)
    out_shape = shape_a[:-1] + shape_b[-1:]
    G = series(out_shape, n, seed + 2, dtype)
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        a = PolyTensor(A, requires_grad=backward)
        b = PolyTensor(B, requires_grad=backward)
        c = a @ b
        data = dict(A=A, B=B, C=coeffs(c))
        if backward:
            c.backward(PolyTensor(G))
            data.update(G=G, dA=coeffs(a.grad), dB=coeffs(b.grad))
    save(name, **data)


def case_matmul_complex():
    A = series((12, 20), 2, 40, complex_from=1)
    B = series((20, 9), 2, 41, complex_from=1)
    with PolyTensor.plain_range():
        c = PolyTensor(A) @ PolyTensor(B)
    save("matmul_c128_n2", A=A, B=B, C=coeffs(c))


def case_rmsnorm(dtype, name):
    n = 3
    X = series((6, 32), n, 50, dtype)
    w = 1 + 0.02 * torch.randn(32, generator=torch.Generator().manual_seed(51), dtype=torch.float64)
    W = [w.to(dtype)] + [torch.zeros(32, dtype=dtype) for _ in range(n)]
    G = series((6, 32), n, 52, dtype)
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        x = PolyTensor(X, requires_grad=True)
        wp = PolyTensor(W, requires_grad=True)
        y = F.rms_norm(x, (32,), wp)
        y.backward(PolyTensor(G))
        save(name, X=X, W=W, G=G, Y=coeffs(y), dX=coeffs(x.grad), dW=coeffs(wp.grad))


def case_gelu():
    n = 4
    X = series((7, 9), n, 60)
    G = series((7, 9), n, 61)
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        x = PolyTensor(X, requires_grad=True)
        y = F.gelu(x)
        y.backward(PolyTensor(G))
        save("gelu_f64_n4", X=X, G=G, Y=coeffs(y), dX=coeffs(x.grad))


def case_cross_entropy():
    n = 4
    X = series((8, 50), n, 70)
    target = torch.randint(0, 50, (8,), generator=torch.Generator().manual_seed(71))
    target[3] = -100
    Z = PolyTensor((0, 1), degree=n)
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        x = PolyTensor(X, requires_grad=True)
        ce = F.cross_entropy(x, target)
        loss = ce * (1 - 0.5 * Z)
        loss.backward()
        save("ce_f64_n4", X=X, target=target, CE=coeffs(ce), loss=coeffs(loss), dX=coeffs(x.grad))
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        x = PolyTensor(X, requires_grad=True)
        per_row = F.cross_entropy(x, target, reduction="none")
        G = series((8,), n, 72)
        per_row.backward(PolyTensor(G))
        save("ce_none_f64_n4", X=X, target=target, G=G, CE=coeffs(per_row), dX=coeffs(x.grad))


def case_cross_entropy_softcap_and_embedding():
    """PolyTensor.cross_entropy with a softcap (the public API, src/polytensors/_tensor.py:255-269)
    and reduction 'sum', and F.embedding with padding_idx, forward and backward in plain range,
    degree 3."""
    n = 3
    X = series((6, 40), n, 140)
    target = torch.randint(0, 40, (6,), generator=torch.Generator().manual_seed(141))
    target[2] = -100
    G = [t.reshape(()) for t in series((1,), n, 142)]
    W = series((10, 4), n, 143)
    idx = torch.tensor([[1, 0, 3], [0, 9, 1]])
    GE = series((2, 3, 4), n, 144)
    out = {}
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        x = PolyTensor(X, requires_grad=True)
        loss = PolyTensor.cross_entropy(x, target, softcap=5.0, reduction="sum")
        loss.backward(PolyTensor(G))
        out["softcap_sum"], out["d_softcap_sum"] = coeffs(loss), coeffs(x.grad)
        w = PolyTensor(W, requires_grad=True)
        e = F.embedding(idx, w, padding_idx=0)
        e.backward(PolyTensor(GE))
        out["embedding"], out["d_embedding"] = coeffs(e), coeffs(w.grad)
    save("ce_softcap_embedding_f64_n3", X=X, target=target, G=G, W=W, idx=idx, GE=GE, **out)


def case_attention():
    n = 3
    shape = (1, 2, 9, 4)
    Q, K, V = (series(shape, n, s) for s in (80, 81, 82))
    G = series(shape, n, 83)
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        q, k, v = (PolyTensor(c, requires_grad=True) for c in (Q, K, V))
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        o.backward(PolyTensor(G))
        save("attn_causal_f64_n3", Q=Q, K=K, V=V, G=G, O=coeffs(o), dQ=coeffs(q.grad), dK=coeffs(k.grad),
             dV=coeffs(v.grad))
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        q, k, v = (PolyTensor(c, requires_grad=True) for c in (Q, K, V))
        o = F.scaled_dot_product_attention(q, k, v, scale=0.3)
        o.backward(PolyTensor(G))
        save("attn_full_f64_n3", Q=Q, K=K, V=V, G=G, O=coeffs(o), dQ=coeffs(q.grad), dK=coeffs(k.grad),
             dV=coeffs(v.grad))


def case_series_ops():
    n = 5
    X = series((4, 6), n, 90)
    Xp = [X[0].abs() + 0.5] + X[1:]
    Y = series((4, 6), n, 91)
    Yp = [Y[0].abs() + 0.5] + Y[1:]
    out = {}
    with PolyTensor.plain_range():
        x, xp, y, yp = PolyTensor(X), PolyTensor(Xp), PolyTensor(Y), PolyTensor(Yp)
        out["mul"] = coeffs(x * y)
        out["div"] = coeffs(x / yp)
        out["add"] = coeffs(x + 2.5 * y)
        out["exp"] = coeffs(torch.exp(x))
        out["log"] = coeffs(torch.log(xp))
        out["rsqrt"] = coeffs(torch.rsqrt(xp))
        out["tanh"] = coeffs(torch.tanh(x))
        out["sigmoid"] = coeffs(torch.sigmoid(x))
        out["gelu"] = coeffs(F.gelu(x))
        out["softmax"] = coeffs(torch.softmax(x, dim=-1))
        out["log_softmax"] = coeffs(torch.log_softmax(x, dim=-1))
        out["sum1"] = coeffs(x.sum(dim=1))
        out["mean0"] = coeffs(x.mean(dim=0))
        out["square"] = coeffs(x.square())
    save("series_ops_f64_n5", X=X, Xp=Xp, Y=Y, Yp=Yp, **out)


def case_series_rules_backward():
    """Forward rules the series_ops case leaves out (sqrt, reciprocal, an integer power) and the
    backward rules of tanh, sigmoid, GELU, softmax and log-softmax (y.backward(G) in plain range),
    degree 4."""
    n = 4
    X = series((5, 7), n, 130)
    Xp = [X[0].abs() + 0.5] + X[1:]
    G = series((5, 7), n, 131)
    out = {}
    with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
        x, xp = PolyTensor(X), PolyTensor(Xp)
        out["sqrt"] = coeffs(torch.sqrt(xp))
        out["reciprocal"] = coeffs(torch.reciprocal(xp))
        out["cube"] = coeffs(x ** 3)
        rules = (("tanh", torch.tanh), ("sigmoid", torch.sigmoid), ("gelu", F.gelu),
                 ("softmax", lambda t: torch.softmax(t, dim=-1)), ("log_softmax", lambda t: torch.log_softmax(t, dim=-1)))
        for name, fn in rules:
            xg = PolyTensor(X, requires_grad=True)
            fn(xg).backward(PolyTensor(G))
            out[f"d_{name}"] = coeffs(xg.grad)
    save("series_rules_bwd_f64_n4", X=X, Xp=Xp, G=G, **out)


def case_series_ops_complex():
    """Elementwise rules on a real base with complex128 directions (the constructor's model for a
    float64 base and complex directions), degree 3, in plain range."""
    n = 3
    X = series((4, 6), n, 95, complex_from=1)
    Xp = [X[0].abs() + 0.5] + X[1:]
    Y = series((4, 6), n, 96, complex_from=1)
    Yp = [Y[0].abs() + 0.5] + Y[1:]
    R = series((4, 6), n, 97)                     # a real series
    out = {}
    with PolyTensor.plain_range():
        x, xp, y, yp, r = PolyTensor(X), PolyTensor(Xp), PolyTensor(Y), PolyTensor(Yp), PolyTensor(R)
        out["mul"] = coeffs(x * y)
        out["mul_real"] = coeffs(x * r)
        out["div"] = coeffs(x / yp)
        out["add"] = coeffs(x + 2.5 * y)
        out["sub_real"] = coeffs(r - x)
        out["scale_complex"] = coeffs(x * (0.5 - 1.5j))
        out["exp"] = coeffs(torch.exp(x))
        out["log"] = coeffs(torch.log(xp))
        out["sqrt"] = coeffs(torch.sqrt(xp))
        out["rsqrt"] = coeffs(torch.rsqrt(xp))
        out["reciprocal"] = coeffs(torch.reciprocal(xp))
        out["tanh"] = coeffs(torch.tanh(x))
        out["sigmoid"] = coeffs(torch.sigmoid(x))
        out["gelu"] = coeffs(F.gelu(x))
        out["square"] = coeffs(x.square())
        out["sum1"] = coeffs(x.sum(dim=1))
        out["mean0"] = coeffs(x.mean(dim=0))
    save("series_ops_c128_n3", X=X, Xp=Xp, Y=Y, Yp=Yp, R=R, **out)


def case_default_mode_range():
    """Default (extended-range) mode with float32 values beyond float32's range: the reference keeps
    hidden mantissa/exponent coefficients, so intermediates that overflow or underflow in the public
    tensors come back finite.  Degree 3."""
    n = 3
    g = torch.Generator().manual_seed(120)
    big = [torch.randn(4, 5, generator=g) * 1e30 for _ in range(n + 1)]
    small = [torch.randn(4, 5, generator=g) * 1e-30 for _ in range(n + 1)]
    W = [torch.randn(5, 3, generator=g) * 1e25 for _ in range(n + 1)]
    Wt = [torch.randn(3, 5, generator=g) * 1e25 for _ in range(n + 1)]
    x, s, w, wt = PolyTensor(big), PolyTensor(small), PolyTensor(W), PolyTensor(Wt)
    out = {}
    y = x * x
    out["square_public"] = coeffs(y)
    out["square_back"] = coeffs(y / x)
    out["square_back_t"] = coeffs(y.t() / x.t())
    out["tiny_back"] = coeffs((s * s) / s)
    out["sub"] = coeffs((y - 0.5 * y) / x)
    out["rsub_back"] = coeffs((1.0 - y) / x)
    out["matmul_scaled"] = coeffs((x @ w) * 1e-35)
    out["linear_scaled"] = coeffs(F.linear(x, wt) * 1e-35)
    out["sum_scaled"] = coeffs((x * x).sum(dim=1) * 1e-35)
    out["mean_scaled"] = coeffs((x * x).mean() * 1e-35)
    out["reciprocal_back"] = coeffs(torch.reciprocal(y) * 1e30 * 1e30)
    z = x * 1.0
    z.mul_(x)
    z.div_(x)
    out["inplace_back"] = coeffs(z)
    # exp of a base around 100: exp(100) ~ 2.7e43 overflows float32's public coefficients
    E = [torch.full((4, 5), 100.0) + torch.randn(4, 5, generator=g)] + [torch.randn(4, 5, generator=g) / (k + 1)
                                                                          for k in range(n)]
    e = torch.exp(PolyTensor(E))
    out["exp_public"] = coeffs(e)
    out["exp_scaled"] = coeffs(e * 1e-30)
    save("default_mode_range_f32_n3", X=big, S=small, W=W, Wt=Wt, E=E, **out)


def case_readme_fit(plain):
    """README linear-regression fit (README.md:44-68), seed 0, 10 SGD steps."""
    torch.manual_seed(0)
    Z = PolyTensor((0, 1), degree=5)
    n, d, noise_std = 64, 3, 0.1
    A, b = torch.randn(d), torch.randn(())
    X = torch.randn(n, d)
    E = noise_std * torch.randn(n)
    Y = X @ A + b + E
    X_prime = torch.randn(n, d)
    Y_prime = (d + 1 + noise_std ** 2) ** 0.5 * torch.randn(n)
    w = (torch.zeros(d) + 0 * Z).requires_grad_()
    c = (torch.zeros(()) + 0 * Z).requires_grad_()
    opt = torch.optim.SGD([w, c], lr=0.1, foreach=False)
    batches = []
    ctx = PolyTensor.plain_range() if plain else torch.enable_grad()
    with ctx:
        for _ in range(10):
            i, j = torch.randint(n, (16,)), torch.randint(n, (16,))
            batches.append((i.clone(), j.clone()))
            opt.zero_grad(set_to_none=True)
            with PolyTensor.retain_wrappers():
                signal_loss = (X[i] @ w + c - Y[i]).square().mean()
                noise_loss = (X_prime[j] @ w + c - Y_prime[j]).square().mean()
                loss = (signal_loss + (1 - Z) * noise_loss) / 2
                loss.backward()
                opt.step()
    save("readme_fit_plain" if plain else "readme_fit_default", X=X, Y=Y, X_prime=X_prime, Y_prime=Y_prime,
         batches=batches, w=coeffs(w), c=coeffs(c))


def tiny_transformer_config():
    return dict(layers=2, d=16, heads=2, mlp=64, vocab=50, seq=8, batch=2, degree=3, steps=3, lr=0.1, lam=0.5)


def case_tiny_transformer(dtype=torch.float32, name="tiny_transformer_f32_n3"):
    """A reduced decoder step loop in the layout of the benchmark transformer: RMSNorm, separate
    q/k/v linears, causal SDPA, GELU MLP, untied head, loss CE*(1 - lam*Z), SGD(foreach=False).
    The float64 run starts from the float32 initial values and serves as the accuracy yardstick
    for float32 results (small coefficients of the loss lose many digits to float32 rounding)."""
    cfg = tiny_transformer_config()
    n, d, H, V, T, Bt = cfg["degree"], cfg["d"], cfg["heads"], cfg["vocab"], cfg["seq"], cfg["batch"]
    g = torch.Generator().manual_seed(100)
    init = {}

    def param(name, *shape, ones=False):
        base = torch.ones(*shape) if ones else 0.02 * torch.randn(*shape, generator=g)
        init[name] = base.clone()
        return torch.nn.Parameter(PolyTensor((base.to(dtype),), degree=n))

    P = {"emb": param("emb", V, d)}
    for l in range(cfg["layers"]):
        for nm, shape in (("n1", (d,)), ("n2", (d,))):
            P[f"{nm}.{l}"] = param(f"{nm}.{l}", *shape, ones=True)
        for nm in ("wq", "wk", "wv", "wo"):
            P[f"{nm}.{l}"] = param(f"{nm}.{l}", d, d)
        P[f"w1.{l}"] = param(f"w1.{l}", cfg["mlp"], d)
        P[f"w2.{l}"] = param(f"w2.{l}", d, cfg["mlp"])
    P["nf"] = param("nf", d, ones=True)
    P["head"] = param("head", V, d)
    ids = torch.randint(0, V, (cfg["steps"], Bt, T + 1), generator=g)
    Z = PolyTensor((0, 1), degree=n)
    opt = torch.optim.SGD(list(P.values()), lr=cfg["lr"], foreach=False)
    losses = []
    with PolyTensor.plain_range():
        for step in range(cfg["steps"]):
            opt.zero_grad(set_to_none=True)
            with PolyTensor.retain_wrappers():
                inp, tgt = ids[step, :, :-1], ids[step, :, 1:]
                x = F.embedding(inp, P["emb"])
                for l in range(cfg["layers"]):
                    h = F.rms_norm(x, (d,), P[f"n1.{l}"])
                    q, k, v = (F.linear(h, P[f"{nm}.{l}"]).view(Bt, T, H, d // H).transpose(1, 2)
                               for nm in ("wq", "wk", "wv"))
                    a = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(Bt, T, d)
                    x = x + F.linear(a, P[f"wo.{l}"])
                    h = F.rms_norm(x, (d,), P[f"n2.{l}"])
                    x = x + F.linear(F.gelu(F.linear(h, P[f"w1.{l}"])), P[f"w2.{l}"])
                logits = F.linear(F.rms_norm(x, (d,), P["nf"]), P["head"])
                loss = F.cross_entropy(logits.reshape(-1, V), tgt.reshape(-1)) * (1 - cfg["lam"] * Z)
                loss.backward()
                opt.step()
                losses.append(coeffs(loss))
    save(name, config=cfg, init=init, ids=ids, losses=losses, final={k: coeffs(p) for k, p in P.items()})


if __name__ == "__main__":
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    case_matmul("matmul_f64_n2", (24, 40), (40, 16), 2, torch.float64, 1)
    case_matmul("matmul_f64_n4", (17, 33), (33, 29), 4, torch.float64, 11)
    case_matmul("matmul_f32_n4", (24, 40), (40, 16), 4, torch.float32, 21)
    case_matmul("bmm_f64_n3", (3, 8, 12), (3, 12, 10), 3, torch.float64, 31)
    case_matmul_complex()
    case_rmsnorm(torch.float64, "rmsnorm_f64_n3")
    case_rmsnorm(torch.float32, "rmsnorm_f32_n3")
    case_gelu()
    case_cross_entropy()
    case_cross_entropy_softcap_and_embedding()
    case_attention()
    case_series_ops()
    case_series_ops_complex()
    case_series_rules_backward()
    case_default_mode_range()
    case_readme_fit(plain=False)
    case_readme_fit(plain=True)
    case_tiny_transformer()
    case_tiny_transformer(torch.float64, "tiny_transformer_f64_n3")
