"""Helpers shared by the GPU parity tests."""

import math

import torch

from oracle import polyref as ref


def series(shape, n, seed, dtype=torch.float64, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(*shape, generator=g, dtype=torch.float64) / math.factorial(k)).to(dtype).to(device)
            for k in range(n + 1)]


def cuda(planes):
    return [p.cuda() for p in planes]


def poly(planes, requires_grad=False, device="cuda"):
    from polytensors_b200 import PolyTensor

    return PolyTensor(tuple(p.to(device) for p in planes), requires_grad=requires_grad)


def coeffs(p):
    return [c.detach().cpu() for c in p.coeffs]


def assert_close(got, want, tol, what=""):
    got = [g.detach().cpu() if isinstance(g, torch.Tensor) else g for g in got]
    errs = ref.plane_errors(got, want)
    assert len(got) == len(want), what
    for g, w in zip(got, want):
        assert tuple(g.shape) == tuple(w.shape), (what, g.shape, w.shape)
    assert max(errs) <= tol, (what, errs)
    return errs
