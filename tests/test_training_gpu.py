"""End-to-end training through the PolyTensor API on the GPU, against trajectories the
reference produced (tests/golden): the README linear-regression fit and a reduced
decoder-only transformer (RMSNorm, causal attention, GELU MLP, CE*(1 - lambda Z), SGD)."""

import pytest
import torch
import torch.nn.functional as F

from gpu_util import assert_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["readme_fit_plain", "readme_fit_default"])
def test_readme_fit(golden, name):
    from polytensors_b200 import PolyTensor

    g = golden(name)
    dev = "cuda"
    Z = PolyTensor((torch.tensor(0.0, device=dev), 1.0), degree=5)
    X, Y, Xp, Yp = (g[k].to(dev) for k in ("X", "Y", "X_prime", "Y_prime"))
    d = X.shape[1]
    w = (torch.zeros(d, device=dev) + 0 * Z).requires_grad_()
    c = (torch.zeros((), device=dev) + 0 * Z).requires_grad_()
    opt = torch.optim.SGD([w, c], lr=0.1, foreach=False)
    with PolyTensor.plain_range():
        for i, j in g["batches"]:
            i, j = i.to(dev), j.to(dev)
            opt.zero_grad(set_to_none=True)
            with PolyTensor.retain_wrappers():
                signal_loss = (X[i] @ w + c - Y[i]).square().mean()
                noise_loss = (Xp[j] @ w + c - Yp[j]).square().mean()
                loss = (signal_loss + (1 - Z) * noise_loss) / 2
                loss.backward()
                opt.step()
    assert_close([p.detach().cpu() for p in w.coeffs], g["w"], 1e-4, "w")
    assert_close([p.detach().cpu() for p in c.coeffs], g["c"], 1e-4, "c")


def run_tiny_transformer(g, device="cuda"):
    from polytensors_b200 import PolyTensor

    cfg, init = g["config"], g["init"]
    n, d, H, V, T, Bt = cfg["degree"], cfg["d"], cfg["heads"], cfg["vocab"], cfg["seq"], cfg["batch"]
    P = {k: torch.nn.Parameter(PolyTensor((v.to(device),), degree=n)) for k, v in init.items()}
    Z = PolyTensor((torch.tensor(0.0, device=device), 1.0), degree=n)
    opt = torch.optim.SGD(list(P.values()), lr=cfg["lr"], foreach=False)
    ids = g["ids"].to(device)
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
                losses.append([c.detach().cpu() for c in loss.coeffs])
    return P, losses


def _as_accurate(got, ref32, ref64, what):
    """Per plane: |got - ref64| <= max(1e-4 * max|ref64|, 3 * |ref32 - ref64|), i.e. the float32
    GPU result is within the float32 tolerance of the float64 reference, or at least as accurate
    (within 3x) as the reference's own float32 result."""
    for k, (g, a, b) in enumerate(zip(got, ref32, ref64)):
        g, a, b = g.double(), a.double(), b.double()
        err = (g - b).abs().max().item()
        ref_err = (a - b).abs().max().item()
        scale = b.abs().max().item()
        assert err <= max(1e-4 * scale, 3 * ref_err), (what, k, err, ref_err, scale)


def test_tiny_transformer_matches_reference(golden):
    g32, g64 = golden("tiny_transformer_f32_n3"), golden("tiny_transformer_f64_n3")
    P, losses = run_tiny_transformer(g32)
    for step, got in enumerate(losses):
        _as_accurate(got, g32["losses"][step], g64["losses"][step], f"loss step {step}")
    for name in g32["final"]:
        got = [c.detach().cpu() for c in P[name].coeffs]
        _as_accurate(got, g32["final"][name], g64["final"][name], name)
