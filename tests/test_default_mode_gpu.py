"""Default (extended-range) mode on the kernels against the reference's own default-mode run.

Outside PolyTensor.plain_range() the reference keeps a hidden mantissa / exponent copy of every
coefficient (src/polytensors/_scaled.py, _range.py, _range_ops.py), so intermediates that leave
float32's range in the public tensors come back finite.  tests/golden/default_mode_range_f32_n3.pt
holds that run (values around 1e30 and 1e-30, products around 1e60 and 1e55); here the same chain
runs on pk_scaled_* kernels.  Finite public coefficients agree within 1e-5 of the plane max-norm;
overflowed ones are infinite in the same places with the same signs."""

import pytest
import torch
import torch.nn.functional as F

from oracle import polyref as ref

pytestmark = pytest.mark.gpu


def _cuda(planes):
    from polytensors_b200 import PolyTensor

    return PolyTensor(tuple(p.cuda() for p in planes))


def _same(got, want, tol, what):
    got = [g.detach().cpu() for g in got.coeffs]
    assert len(got) == len(want), what
    for g, w in zip(got, want):
        assert torch.equal(torch.isinf(g), torch.isinf(w)), what
        assert torch.equal(torch.sign(g[torch.isinf(w)]), torch.sign(w[torch.isinf(w)])), what
    finite = [(g.nan_to_num(posinf=0.0, neginf=0.0), w.nan_to_num(posinf=0.0, neginf=0.0)) for g, w in zip(got, want)]
    errs = ref.plane_errors([f[0].double() for f in finite], [f[1].double() for f in finite])
    assert max(errs) <= tol, (what, errs)


def test_default_mode_range_matches_the_reference(golden):
    g = golden("default_mode_range_f32_n3")
    x, s, w, wt = (_cuda(g[k]) for k in ("X", "S", "W", "Wt"))
    y = x * x
    got = {
        "square_public": y, "square_back": y / x, "square_back_t": y.t() / x.t(), "tiny_back": (s * s) / s,
        "sub": (y - 0.5 * y) / x, "rsub_back": (1.0 - y) / x, "matmul_scaled": (x @ w) * 1e-35, "linear_scaled": F.linear(x, wt) * 1e-35,
        "sum_scaled": (x * x).sum(dim=1) * 1e-35, "mean_scaled": (x * x).mean() * 1e-35,
        "reciprocal_back": torch.reciprocal(y) * 1e30 * 1e30,
    }
    z = x * 1.0
    z.mul_(x)
    z.div_(x)
    got["inplace_back"] = z
    e = torch.exp(_cuda(g["E"]))
    got["exp_public"] = e
    got["exp_scaled"] = e * 1e-30
    for key, value in got.items():
        _same(value, g[key], 1e-5, key)


def test_plain_range_overflows_where_default_mode_does_not(golden):
    """The same chain inside plain_range() keeps no hidden copy: (x * x) / x overflows."""
    from polytensors_b200 import PolyTensor

    g = golden("default_mode_range_f32_n3")
    x = _cuda(g["X"])
    with PolyTensor.plain_range():
        back = (x * x) / x
    assert not torch.isfinite(back.coeffs[0]).all()
    assert torch.isfinite((x * x / x).coeffs[0]).all()


def test_hidden_copy_is_dropped_after_a_public_write(golden):
    """A direct write to a public coefficient invalidates the hidden copy (the reference's version
    snapshots, src/polytensors/_range.py:40-52): the next operation reads the public values."""
    g = golden("default_mode_range_f32_n3")
    x = _cuda(g["X"])
    y = x * x
    y.coeffs[0].fill_(2.0)
    back = y / x
    want = 2.0 / g["X"][0]
    assert torch.allclose(back.coeffs[0].cpu(), want, rtol=1e-5)


def test_backward_inside_plain_range_stays_plain():
    """CUDA backward runs on the autograd engine's threads; started inside plain_range() it keeps
    plain-range arithmetic (no extended-range kernel launches), as the forward did."""
    from polytensors_b200 import PolyTensor, _lib

    g = torch.Generator().manual_seed(5)
    planes = lambda *shape: tuple(torch.randn(*shape, generator=g).cuda() for _ in range(3))  # noqa: E731
    a = PolyTensor(planes(16, 8), requires_grad=True)
    b = PolyTensor(planes(8, 4), requires_grad=True)
    _lib.profile_query("scaled_map")
    _lib.profile_enable(True)
    try:
        with PolyTensor.plain_range(), PolyTensor.retain_wrappers():
            ((a @ b) * (a @ b)).sum().backward()
        torch.cuda.synchronize()
        assert _lib.profile_query("scaled_map")[1] == 0
        assert a.grad is not None and torch.isfinite(a.grad.coeffs[2]).all()
        with PolyTensor.retain_wrappers():
            (a.detach() * 2.0).sum()
        torch.cuda.synchronize()
        assert _lib.profile_query("scaled_map")[1] > 0
    finally:
        _lib.profile_enable(False)
