"""Out-of-range embedding indices and cross-entropy targets raise IndexError before any
launch, as the reference's torch ops do (its embedding rule, src/polytensors/_dispatch.py:530-532,
and NLL rule, :537-543, hand the indices to torch.embedding / torch.nll_loss).  The check runs
on the host side of the wrappers, so these tests need no GPU: with CPU tensors a valid call gets
past the check and stops at the CUDA requirement instead."""

import pytest
import torch


def test_embedding_index_out_of_range_raises():
    from polytensors_b200 import _kernels as K

    W = [torch.zeros(10, 4) for _ in range(3)]
    for bad in ([3, 10], [-1, 2], [[0, 1], [11, 2]]):
        with pytest.raises(IndexError, match="embedding"):
            K.gather_rows(W, torch.tensor(bad))
    with pytest.raises(NotImplementedError, match="CUDA"):
        K.gather_rows(W, torch.tensor([0, 9, 3]))


def test_embedding_backward_index_out_of_range_raises():
    from polytensors_b200 import _kernels as K

    G = [torch.zeros(2, 4) for _ in range(3)]
    with pytest.raises(IndexError, match="embedding backward"):
        K.scatter_add_rows(G, torch.tensor([1, 10]), 10)
    with pytest.raises(NotImplementedError, match="CUDA"):
        K.scatter_add_rows(G, torch.tensor([1, 9]), 10)


def test_cross_entropy_target_out_of_range_raises():
    from polytensors_b200 import _kernels as K

    Z = [torch.zeros(4, 7) for _ in range(2)]
    for bad in ([0, 7, 1, 2], [0, -5, 1, 2]):
        with pytest.raises(IndexError, match="cross_entropy target"):
            K.cross_entropy_fwd(Z, torch.tensor(bad), -100, None)
    # ignore_index is allowed even though it lies outside [0, C)
    with pytest.raises(NotImplementedError, match="CUDA"):
        K.cross_entropy_fwd(Z, torch.tensor([0, -100, 6, 2]), -100, None)
    with pytest.raises(IndexError):
        K.cross_entropy_fwd(Z, torch.tensor([0, -100, 6, 2]), 3, None)
