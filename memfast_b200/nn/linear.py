"""Linear inference on a programmed analog matrix (memfast/nn/linear.py:8-14)."""

from torch import nn

from ..simulator import AnalogMatrix


class AnalogLinear(AnalogMatrix):
    """An ``nn.Linear`` programmed once into analog arrays: its [out, in] weight becomes
    the matrix (same orientation) and its bias is added to every output."""

    def __init__(self, source, simulator, *, name="linear"):
        if not isinstance(source, nn.Linear):
            raise TypeError("source must be torch.nn.Linear")
        super().__init__(source.weight, simulator, bias=source.bias, name=name)
