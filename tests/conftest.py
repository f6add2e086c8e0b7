"""pytest configuration: the ``gpu`` marker and import paths.

``python -m pytest tests -m "not gpu"`` runs on any machine (oracle vs golden vectors,
host logic, the C ABI's exported symbols); ``-m gpu`` runs the CUDA parity tests on a
B200.  The package lives in ``poly-tensors_b200/`` and the oracle in ``oracle/``.
"""

import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
for path in (ROOT / "poly-tensors_b200", ROOT):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    import torch

    cache = {}

    def load(name):
        if name not in cache:
            cache[name] = torch.load(ROOT / "tests" / "golden" / f"{name}.pt", weights_only=False)
        return cache[name]

    return load
