"""memfast_b200: B200-native engine for MemFast's bit-sliced analog matrix product.

Drop-in for the reference ``memfast`` inference API on CUDA devices::

    import memfast_b200 as memfast
    sim = memfast.Simulator(memfast.Config(...))
    y = sim.mm(a, b)            # a, b: CUDA tensors
"""

from .config import Config, Nonidealities
from .functional import matmul, mm
from .nn import AnalogConv2d, AnalogLinear, convert_model, reset_read_events
from .simulator import AnalogMatrix, Simulator

__version__ = "0.1.0"
__all__ = [
    "Config", "Nonidealities", "Simulator", "mm", "matmul", "AnalogMatrix", "AnalogLinear",
    "AnalogConv2d", "convert_model", "reset_read_events",
]
