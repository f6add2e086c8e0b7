"""B200-native PolyTensor: truncated Taylor-series tensors whose arithmetic runs in
hand-written sm_100a kernels (libpolykern.so).

    from polytensors_b200 import PolyTensor
"""

from ._tensor import PolyTensor

__all__ = ["PolyTensor"]
