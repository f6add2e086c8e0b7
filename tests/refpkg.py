"""Import the reference package (samuel-gunn/poly-tensors) for the binding tests: from the
directory named by POLYTENSORS_REFERENCE, else from baseline/_ref (the reference pip-installed
into this repository, which travels with it).  Tests skip when neither holds it."""

import importlib
import os
import sys

import pytest

from conftest import ROOT


def reference_package():
    path = os.environ.get("POLYTENSORS_REFERENCE") or str(ROOT / "baseline" / "_ref")
    if not os.path.isdir(os.path.join(path, "polytensors")):
        pytest.skip("the reference package is not installed (baseline/_ref)")
    if path not in sys.path:
        sys.path.insert(0, path)
    return importlib.import_module("polytensors")
