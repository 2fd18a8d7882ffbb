"""Analog inference layers on the B200 engine."""

from .conversion import convert_model, reset_read_events
from .convolution import AnalogConv2d
from .linear import AnalogLinear

__all__ = ["AnalogLinear", "AnalogConv2d", "convert_model", "reset_read_events"]
