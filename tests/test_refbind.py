"""The reference binding (polytensors_b200.refbind) without a GPU: installing it replaces the
reference's gate functions and uninstalling puts them back; calls the kernels do not take (here:
CPU tensors) reach the reference's own code, so its results are unchanged."""

import pytest
import torch
import torch.nn.functional as F

from refpkg import reference_package


@pytest.fixture
def bound():
    ref = reference_package()
    from polytensors_b200 import refbind

    refbind.install(ref)
    try:
        yield ref
    finally:
        refbind.uninstall(ref)


def _sites(ref):
    import importlib

    name = ref.__name__
    return [(importlib.import_module(f"{name}.{m}"), a) for m, a in (
        ("_plain", "plain_polynomial_product"), ("_fused_activation", "maybe_activation"),
        ("_fused_norm", "eligible"), ("_fused_norm", "rms_norm"), ("_fused_cross_entropy", "eligible"),
        ("_fused_cross_entropy", "fused"), ("_fused_attention", "eligible"), ("_fused_attention", "attention"))]


def test_install_and_uninstall_swap_the_gate_functions():
    ref = reference_package()
    from polytensors_b200 import refbind

    before = [getattr(m, a) for m, a in _sites(ref)]
    refbind.install(ref)
    try:
        assert refbind.installed(ref)
        now = [getattr(m, a) for m, a in _sites(ref)]
        assert all(n is not b and n.__wrapped__ is b for n, b in zip(now, before))
        refbind.install(ref)   # idempotent
        assert [getattr(m, a) for m, a in _sites(ref)] == now
    finally:
        refbind.uninstall(ref)
    assert [getattr(m, a) for m, a in _sites(ref)] == before
    assert not refbind.installed(ref)


def _ops(P, seed):
    g = torch.Generator().manual_seed(seed)
    planes = lambda *s: tuple(torch.randn(*s, generator=g, dtype=torch.float64) for _ in range(4))   # noqa: E731
    a, b = P(planes(5, 6)), P(planes(6, 3))
    x = P(planes(4, 8))
    w = P(planes(8))
    q, k, v = (P(planes(1, 2, 7, 4)) for _ in range(3))
    target = torch.randint(0, 8, (4,), generator=g)
    with P.plain_range():
        return [a @ b, a * a, F.gelu(x), F.rms_norm(x, (8,), w), F.cross_entropy(x, target),
                F.scaled_dot_product_attention(q, k, v, is_causal=True)]


def test_cpu_results_unchanged_by_the_binding():
    ref = reference_package()
    from polytensors_b200 import refbind

    want = _ops(ref.PolyTensor, 3)
    refbind.install(ref)
    try:
        got = _ops(ref.PolyTensor, 3)
    finally:
        refbind.uninstall(ref)
    for g, w in zip(got, want):
        assert type(g) is ref.PolyTensor
        for cg, cw in zip(g.coeffs, w.coeffs):
            assert torch.equal(cg, cw)
