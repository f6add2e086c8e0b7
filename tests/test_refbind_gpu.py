"""The reference's own PolyTensor (samuel-gunn/poly-tensors, from baseline/_ref) running on CUDA
through libpolykern after polytensors_b200.refbind.install: a @ b, linear, the elementwise
product, F.gelu, F.rms_norm, F.cross_entropy and scaled_dot_product_attention inside
plain_range(), forward and backward, launch pk:: kernels (the library's launch counter moves)
and match the reference's own results on the CPU for the same inputs.  Degree 3 (beyond the
reference's degree-1 Triton gates); float32 within 1e-4 of the plane max-norm, float64 1e-10."""

import pytest
import torch
import torch.nn.functional as F

from gpu_util import assert_close
from refpkg import reference_package

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref():
    pkg = reference_package()
    from polytensors_b200 import refbind

    refbind.install(pkg)
    yield pkg
    refbind.uninstall(pkg)


def series(shape, seed, dtype, n=3):
    g = torch.Generator().manual_seed(seed)
    return tuple((torch.randn(*shape, generator=g, dtype=torch.float64) / (k + 1)).to(dtype) for k in range(n + 1))


def launches(fn):
    from polytensors_b200 import _lib

    before = _lib.launch_count()
    out = fn()
    torch.cuda.synchronize()
    return out, _lib.launch_count() - before


def run(P, device, fn, inputs, grads=True):
    """fn(*PolyTensors) on `device`; returns (output coeffs, input gradient coeffs)."""
    leaves = [P(tuple(c.to(device) for c in x), requires_grad=grads) for x in inputs]
    with P.plain_range(), P.retain_wrappers():
        out = fn(*leaves)
        coeffs = [c.detach().cpu() for c in out.coeffs]
        gr = []
        if grads:
            out.sum().backward() if out.numel() > 1 else out.backward()
            gr = [[c.detach().cpu() for c in t.grad.coeffs] for t in leaves]
    return coeffs, gr


CASES = {
    "matmul": (lambda a, b: a @ b, [((96, 80), 1), ((80, 72), 2)]),
    "linear": (lambda x, w: F.linear(x, w), [((2, 40, 64), 3), ((48, 64), 4)]),
    "mul": (lambda a, b: a * b, [((33, 17), 5), ((33, 17), 6)]),
    "gelu": (lambda x: F.gelu(x), [((50, 64), 7)]),
    "rms_norm": (lambda x, w: F.rms_norm(x, (64,), w), [((40, 64), 8), ((64,), 9)]),
    "sdpa": (lambda q, k, v: F.scaled_dot_product_attention(q, k, v, is_causal=True),
             [((1, 2, 96, 64), 10), ((1, 2, 96, 64), 11), ((1, 2, 96, 64), 12)]),
}


@pytest.mark.parametrize("name", sorted(CASES))
@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-4), (torch.float64, 1e-10)])
def test_reference_ops_run_on_polykern(ref, name, dtype, tol):
    fn, specs = CASES[name]
    inputs = [series(shape, seed, dtype) for shape, seed in specs]
    (got, got_g), count = launches(lambda: run(ref.PolyTensor, "cuda", fn, inputs))
    assert count > 0, f"{name}: no pk:: kernel launched"
    want, want_g = run(ref.PolyTensor, "cpu", fn, [tuple(c.double() for c in x) for x in inputs])
    assert_close(got, want, tol, name)
    for i, (g, w) in enumerate(zip(got_g, want_g)):
        assert_close(g, w, tol * 10, f"{name} grad {i}")


def test_reference_cross_entropy_runs_on_polykern(ref):
    P = ref.PolyTensor
    g = torch.Generator().manual_seed(13)
    target = torch.randint(0, 500, (64,), generator=g)
    inputs = [series((64, 500), 14, torch.float32)]
    fn_cuda = lambda z: F.cross_entropy(z, target.cuda())   # noqa: E731
    (got, got_g), count = launches(lambda: run(P, "cuda", fn_cuda, inputs))
    assert count > 0
    want, want_g = run(P, "cpu", lambda z: F.cross_entropy(z, target), [tuple(c.double() for c in inputs[0])])
    assert_close(got, want, 1e-4, "loss")
    assert_close(got_g[0], want_g[0], 1e-4, "dlogits")
    # the public softcapped form (src/polytensors/_tensor.py:255-269) goes through the same gate
    z = P(tuple(c.cuda() for c in inputs[0]))
    with P.plain_range():
        capped, count = launches(lambda: P.cross_entropy(z, target.cuda(), softcap=30.0))
    zc = P(tuple(c.double() for c in inputs[0]))
    with P.plain_range():
        want_c = P.cross_entropy(zc, target, softcap=30.0)
    assert count > 0
    assert_close([c.cpu() for c in capped.coeffs], list(want_c.coeffs), 1e-4, "softcap")
