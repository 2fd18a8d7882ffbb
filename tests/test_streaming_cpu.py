"""host_mm argument handling, checked before any device work (no GPU needed)."""

import pytest
import torch

import memfast_b200 as mf
from memfast_b200.streaming import _check_operands


class _FakeSimulator(mf.Simulator):
    """A Simulator shell for argument checks only (no device is touched)."""

    def __init__(self):
        pass


def test_host_operands_are_validated_like_mm():
    sim = _FakeSimulator()
    a, b = torch.randn(4, 8), torch.randn(8, 3)
    _check_operands(a, b, sim, None)
    with pytest.raises(TypeError):
        _check_operands(a, b, object(), None)
    with pytest.raises(ValueError, match="incompatible"):
        _check_operands(a, torch.randn(7, 3), sim, None)
    with pytest.raises(ValueError, match="same dtype"):
        _check_operands(a, b.double(), sim, None)
    with pytest.raises(ValueError, match="rank-two"):
        _check_operands(a[0], b, sim, None)
    with pytest.raises(TypeError):
        _check_operands(a.to(torch.int32), b, sim, None)
    with pytest.raises(ValueError, match="out"):
        _check_operands(a, b, sim, torch.empty(4, 4))
    with pytest.raises(NotImplementedError):
        _check_operands(a.requires_grad_(), b, sim, None)
