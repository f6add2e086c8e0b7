"""Host-side behaviour of the PolyTensor mirror that needs no GPU: construction rules,
context managers, retention scopes, error behaviour (mirrors the reference's
tests/test_tensor.py and tests/test_retention.py where they do not compute)."""

import pytest
import torch

import polytensors_b200
from polytensors_b200 import PolyTensor


def test_only_public_export():
    assert polytensors_b200.__all__ == ["PolyTensor"]


def test_validation():
    with pytest.raises(ValueError, match="at least one"):
        PolyTensor([])
    for degree in (-1, -3):
        with pytest.raises(ValueError):
            PolyTensor([1.0], degree=degree)
    for degree in (True, 1.2):
        with pytest.raises(TypeError):
            PolyTensor([1.0], degree=degree)
    with pytest.raises(ValueError, match="at least"):
        PolyTensor([1.0, 2.0], degree=0)
    with pytest.raises(TypeError, match="floating-point"):
        PolyTensor([torch.tensor(1)])
    with pytest.raises(ValueError, match="same device"):
        PolyTensor([torch.tensor(1.0), torch.empty((), device="meta")])
    with pytest.raises(TypeError, match="nested"):
        PolyTensor([PolyTensor([1.0])])


def test_integer_literals_and_constant_padding():
    x = PolyTensor([1, 2], degree=4)
    assert x.dtype == torch.get_default_dtype()
    assert [c.item() for c in x.coeffs] == [1, 2, 0, 0, 0]
    constant = PolyTensor.constant(2, degree=3)
    assert [c.item() for c in constant.coeffs] == [2, 0, 0, 0]
    with pytest.raises(ValueError, match="no tangent"):
        _ = PolyTensor([1.0]).tangent


def test_complex_direction_dtypes():
    x = PolyTensor([torch.tensor(1.0, dtype=torch.float64), 2 + 3j], degree=3)
    assert x.dtype == torch.float64
    assert all(c.dtype == torch.complex128 for c in x.coeffs[1:])
    assert x.tangent == 2 + 3j


def test_overlapping_orders_get_independent_storage():
    zero = torch.tensor(0.0)
    x = PolyTensor([torch.tensor(1.0), zero, zero], degree=2)
    assert not torch._C._overlaps(x.coeffs[1], x.coeffs[2])


def test_constructor_broadcasting_materialises_coefficients():
    x = PolyTensor((torch.tensor([1.0, 2.0]), torch.tensor(1.0)), degree=2)
    assert all(c.shape == (2,) for c in x.coeffs)
    assert x.coeffs[1].stride() == (1,)


def test_python_direction_does_not_round_through_float32():
    direction = 0.12345678912345678
    x = PolyTensor((torch.tensor(0.0, dtype=torch.float64), direction))
    assert x.tangent.item() == direction
    z = PolyTensor((torch.tensor(0.0, dtype=torch.float64), complex(direction, direction)))
    assert z.tangent.item() == complex(direction, direction)


def test_backward_requires_explicit_gradient_for_vector():
    x = PolyTensor([torch.tensor([1.0, 2.0])], degree=1, requires_grad=True)
    with pytest.raises(RuntimeError, match="scalar"):
        x.backward()


def test_unimplemented_operation_fails_explicitly():
    x = PolyTensor([torch.eye(2)], degree=1)
    with pytest.raises(NotImplementedError, match="PolyTensor"):
        torch.linalg.det(x)


def test_series_arithmetic_has_no_cpu_fallback():
    x = PolyTensor((torch.randn(3), torch.randn(3)), degree=2)
    for op in (lambda: x * x, lambda: torch.exp(x), lambda: x.sum(), lambda: x @ x):
        with pytest.raises(NotImplementedError, match="CUDA"):
            op()


def test_views_are_per_coefficient():
    x = PolyTensor((torch.arange(6.0).view(2, 3), torch.ones(2, 3)), degree=1)
    t = x.t()
    assert t.shape == (3, 2) and t.degree == 1
    assert torch.equal(t.coeffs[0], torch.arange(6.0).view(2, 3).t())
    v = x.view(6)
    assert v.shape == (6,) and torch.equal(v.coeffs[1], torch.ones(6))
    s = x[1]
    assert s.shape == (3,) and torch.equal(s.value, torch.tensor([3.0, 4.0, 5.0]))


def test_degree_mismatch_raises():
    a = PolyTensor((torch.ones(2),), degree=1)
    b = PolyTensor((torch.ones(2),), degree=2)
    with pytest.raises(ValueError, match="same degree"):
        torch.cat([a, b])


def test_inplace_update_of_ordinary_tensor_with_polytensor_raises():
    a = torch.zeros(2)
    b = PolyTensor((torch.ones(2),), degree=1)
    with pytest.raises(RuntimeError, match="regular Tensor in-place"):
        a.add_(b)


def test_retention_scopes_nest_and_isolate():
    x = PolyTensor((torch.randn(4, 3), torch.randn(4, 3)), degree=1)
    with PolyTensor.retain_wrappers() as outer:
        x.t()
        before = len(outer)
        assert before >= 1
        with PolyTensor.retain_wrappers(isolated=True) as inner:
            x.t()
            assert len(inner) >= 1
        assert len(inner) == 0 and len(outer) == before
        with PolyTensor.retain_wrappers() as nested:
            x.t()
            assert len(nested) >= 1
        assert len(outer) > before
    assert len(outer) == 0


def test_context_managers_are_context_local():
    from polytensors_b200 import _state

    assert not _state.plain_range.get()
    with PolyTensor.plain_range():
        assert _state.plain_range.get()
        with PolyTensor.fused_attention(False), PolyTensor.fused_cross_entropy(False):
            assert not _state.fused_attention.get() and not _state.fused_cross_entropy.get()
        assert _state.fused_attention.get() and _state.fused_cross_entropy.get()
    assert not _state.plain_range.get()


def test_coefficient_autograd_mode_on_shape_operations():
    """coefficient_autograd(): output coefficients are ordinary tensors with a graph back to the
    input coefficients (shape operations need no GPU); the coefficient map of a transpose is the
    per-plane transpose, so d sum(W * y_1) / d x_1 = W^T and d / d x_0 = 0."""
    c0, c1 = torch.randn(2, 3, requires_grad=True), torch.randn(2, 3, requires_grad=True)
    x = PolyTensor((c0, c1), requires_grad=False)
    W = torch.randn(3, 2)
    with PolyTensor.coefficient_autograd():
        y = x.t()
    assert y.coeffs[1].grad_fn is not None and not y.requires_grad
    g0, g1 = torch.autograd.grad((y.coeffs[1] * W).sum(), (c0, c1), allow_unused=True)
    assert torch.equal(g1, W.t())
    assert g0 is None or torch.equal(g0, torch.zeros_like(c0))
    other = torch.randn(3, 2, requires_grad=True)
    with PolyTensor.coefficient_autograd(), pytest.raises(NotImplementedError, match="coefficient_autograd"):
        torch.mm(x, other)


def test_checkpoint_round_trip_stacked_planes(tmp_path):
    """polytensors_b200.checkpoint: PolyTensors (one dtype, and a real base with complex directions),
    parameters, plain tensors and nested containers survive save/load bit for bit; the stored form
    of a PolyTensor is one (n+1, *shape) plane stack."""
    from polytensors_b200 import PolyTensor, checkpoint

    g = torch.Generator().manual_seed(5)
    a = PolyTensor(tuple(torch.randn(3, 4, generator=g) for _ in range(4)), requires_grad=True)
    base = torch.randn(2, 3, generator=g, dtype=torch.float64)
    dirs = tuple(torch.complex(torch.randn(2, 3, generator=g, dtype=torch.float64),
                               torch.randn(2, 3, generator=g, dtype=torch.float64)) for _ in range(2))
    b = PolyTensor((base,) + dirs)
    w = torch.nn.Parameter(PolyTensor((torch.ones(5), torch.zeros(5)), degree=3))
    state = {"a": a, "nested": [b, (torch.arange(3), "tag", 7)], "w": w}
    path = tmp_path / "ckpt.pt"
    checkpoint.save(state, path)
    raw = checkpoint.load(path, stacked=True)
    assert raw["a"]["planes"].shape == (4, 3, 4) and raw["a"]["degree"] == 3
    assert raw["nested"][0]["directions"].shape == (2, 2, 3) and raw["nested"][0]["base"].dtype == torch.float64
    got = checkpoint.load(path)
    assert isinstance(got["a"], PolyTensor) and got["a"].requires_grad
    for x, y in zip(got["a"].coeffs, a.coeffs):
        assert torch.equal(x, y.detach())
    for x, y in zip(got["nested"][0].coeffs, b.coeffs):
        assert x.dtype == y.dtype and torch.equal(x, y)
    assert got["nested"][1][1] == "tag" and got["nested"][1][2] == 7 and torch.equal(got["nested"][1][0], torch.arange(3))
    assert got["w"].degree == 3 and torch.equal(got["w"].coeffs[0], torch.ones(5))
    bad = tmp_path / "other.pt"
    torch.save({"x": 1}, bad)
    with pytest.raises(ValueError):
        checkpoint.load(bad)


def test_construction_matches_the_reference_rules():
    """Differential check of the constructor against the reference's own class (when the reference
    package is installed): dtypes, shapes, values and storage independence of the coefficients."""
    from refpkg import reference_package

    ref = reference_package()
    t = torch.tensor
    base = torch.arange(3.0)
    cases = [
        ([1, 2], 4), ([1.5], None), ([t(1.0, dtype=torch.float64), 2 + 3j], 3), ([base, 1.0, base[:1]], None),
        ([t([1.0, 2.0], dtype=torch.float16), t(3.0)], 2), ([t(1.0, dtype=torch.bfloat16), 0.5], None),
        ([t(1.0), t(2.0, dtype=torch.complex64)], 1), ([t(1.0, dtype=torch.complex128), t(1.0)], None),
        ([base, base, base], None), ([base.view(3, 1), t([1.0, 2.0])], 2), ([0.1234567891234], 1),
        ([t(2.0, dtype=torch.float64), 0.1234567891234], None), ([True], 1),
    ]
    for coeffs, degree in cases:
        got = PolyTensor(list(coeffs), degree=degree)
        want = ref.PolyTensor(list(coeffs), degree=degree)
        assert got.degree == want.degree, coeffs
        for a, b in zip(got.coeffs, want.coeffs):
            assert a.dtype == b.dtype and a.shape == b.shape and torch.equal(a, b), (coeffs, a, b)
        for i in range(len(got.coeffs)):
            for j in range(i):
                assert not torch._C._overlaps(got.coeffs[i], got.coeffs[j])
    for bad, degree, kind in (([], None, ValueError), ([1.0], -1, ValueError), ([1.0], True, TypeError),
                              ([1.0], 1.5, TypeError), ([1.0, 2.0], 0, ValueError),
                              ([t(1)], None, TypeError)):
        for cls in (PolyTensor, ref.PolyTensor):
            with pytest.raises(kind):
                cls(list(bad), degree=degree)


def test_default_mode_constants_round_like_the_reference():
    """A scalar operand of the extended-range rules is rounded to the operation's dtype first, as
    the reference lifts it (torch.full((), value, dtype=result_type(like, value)))."""
    from polytensors_b200 import _scaled

    for dtype in (torch.float32, torch.bfloat16, torch.float16, torch.float64):
        like = torch.zeros((), dtype=dtype)
        for value in (0.1, 1 / 3, 1e30, 7, -2.5):
            want = torch.full((), value, dtype=torch.result_type(like, value)).item()
            assert _scaled.constant(value, torch.result_type(like, value)) == want
    assert _scaled.constant(0.1, torch.bfloat16) != 0.1


def test_default_mode_hidden_copy_bookkeeping():
    """Default mode's hidden extended-range coefficients, host bookkeeping only (no kernel runs):
    views of a series carry the same view of the mantissas and exponents (the reference's
    map_tensor over its hidden copy), and an in-place write to a public coefficient drops the copy
    from the series and from its views (version snapshots, src/polytensors/_range.py:40-52)."""
    from polytensors_b200 import PolyTensor, _scaled

    g = torch.Generator().manual_seed(3)
    x = PolyTensor(tuple(torch.randn(3, 4, generator=g) for _ in range(3)))
    scs = [_scaled.SC(torch.randn(3, 4, generator=g), torch.randint(-9, 9, (3, 4), generator=g, dtype=torch.int32))
           for _ in range(3)]
    _scaled.attach(x, scs)
    assert _scaled.get(x) is not None
    views = {"t": (x.t(), lambda t: t.t()), "slice": (x[1:], lambda t: t[1:]),
             "detach": (x.detach(), lambda t: t)}
    for name, (v, fn) in views.items():
        got = _scaled.get(v)
        assert got is not None, name
        for a, s in zip(got, scs):
            assert torch.equal(a.m, fn(s.m)) and torch.equal(a.e, fn(s.e)), name
    with PolyTensor.plain_range():
        plain_view = x.t()
    assert _scaled.get(plain_view) is None
    x.coeffs[0].add_(1.0)
    assert _scaled.get(x) is None
    assert _scaled.get(views["t"][0]) is None


def test_plain_range_block_count_survives_exceptions():
    """The process-wide count of open plain_range() blocks (which decides plain-range arithmetic
    inside backward on the autograd engine's threads) is restored when a block exits by an
    exception, and nesting counts each block."""
    from polytensors_b200 import PolyTensor, _state

    before = _state._plain_open
    with pytest.raises(ValueError):
        with PolyTensor.plain_range():
            with PolyTensor.plain_range():
                assert _state._plain_open == before + 2
            raise ValueError
    assert _state._plain_open == before
    assert not _state.plain_mode()
