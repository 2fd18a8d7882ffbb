"""Physical array geometry, number formats and device nonidealities.

Behavioural mirror of the reference ``memfast/config.py`` (v0.3.0):
``Nonidealities`` follows ``config.py:21-45`` and ``Config`` follows
``config.py:48-224`` -- the same fields, defaults, validation rules and error
messages, so that code written against the reference constructs and validates
configurations identically here.  The derived properties are the tables the
CUDA engine consumes:

* ``input_layout`` / ``weight_layout``: per physical slice, least significant
  first, ``(shift, mask, signed_factor)`` (``config.py:193-209``);
* ``adc_maxima``: ADC count limits per weight slice, least significant first
  (``config.py:175-183``);
* ``read_rows`` / ``reads_per_array``: rows converted per ADC read and reads
  per physical array (``config.py:185-191``);
* ``wide`` / ``precise_currents``: FP64 reconstruction and FP64 current
  triggers (``config.py:211-224``).
"""

import math
import operator
import struct
from dataclasses import dataclass, fields

_FLT_MAX = 3.4028234663852886e38
_FLT_TRUE_MIN = 1.401298464324817e-45


def _require_int(value, name, low, high):
    # bool is an int subclass; the reference rejects it by exact type check.
    if type(value) is not int or value < low or value > high:
        raise ValueError(f"{name} must be an integer in [{low}, {high}]")


def _require_nonnegative(value, name):
    ok = not isinstance(value, bool) and isinstance(value, (int, float))
    if not ok or not math.isfinite(value) or value < 0:
        raise ValueError(f"{name} must be a finite nonnegative number")


@dataclass(frozen=True)
class Nonidealities:
    """Dimensionless noise magnitudes; retention times are in seconds."""

    write_variation: float = 0.02
    read_variation: float = 0.0
    read_mode: str = "shared"
    voltage_variation: float = 0.0
    adc_nonlinearity: float = 0.0
    stuck_at_low: float = 0.0
    stuck_at_high: float = 0.0
    drift_coefficient: float = 0.0
    drift_time: float = 0.0
    drift_reference_time: float = 1.0

    def __post_init__(self):
        for item in fields(self):
            if item.name == "read_mode":
                continue
            _require_nonnegative(getattr(self, item.name), item.name)
        if self.read_mode not in ("shared", "slice_pair", "output"):
            raise ValueError("read_mode must be shared, slice_pair, or output")
        if self.stuck_at_low + self.stuck_at_high > 1:
            raise ValueError("stuck-at probabilities must sum to at most one")
        if self.drift_reference_time <= 0:
            raise ValueError("drift_reference_time must be positive")

    @property
    def drift_factor(self):
        """Multiplicative conductance retention factor ``(1+t/t0)^-c``."""
        return (1 + self.drift_time / self.drift_reference_time) ** (-self.drift_coefficient)

    @property
    def ideal(self):
        """True when no effect perturbs currents, so ADC counts are exact integers."""
        return (
            self.write_variation == 0
            and self.read_variation == 0
            and self.voltage_variation == 0
            and self.adc_nonlinearity == 0
            and self.stuck_at_low == 0
            and self.stuck_at_high == 0
            and self.drift_factor == 1
        )


def _slice_widths(value, name, bits, signed):
    try:
        raw = tuple(value)
        if any(isinstance(item, bool) for item in raw):
            raise ValueError
        widths = tuple(operator.index(item) for item in raw)
    except (TypeError, ValueError):
        raise ValueError(f"{name} must contain integer slice widths") from None
    if not widths or sum(widths) != bits:
        raise ValueError(f"{name} slice widths must sum to {bits}")
    if signed and widths[0] != 1:
        raise ValueError(f"{name} must start with a one-bit sign slice and sum to {bits}")
    if any(width < 1 or width > 16 for width in widths):
        raise ValueError(f"{name} slice widths must be in [1,16]")
    return widths


@dataclass(frozen=True)
class Config:
    """Matrices use [reduction rows, output columns] for geometry and scale groups.

    Activations use signed two's complement significance. ``weight_signed=False``
    uses unsigned INT weight codes and positive significance for every slice.
    """

    activation_bits: int = 8
    weight_bits: int = 8
    array_size: tuple = (64, 64)
    weight_quant_gran: tuple = (None, 1)
    input_quant_gran: tuple = (1, None)
    adc_bits: object = 6
    high_conductance: float = 1e-5
    low_conductance: float = 1e-7
    read_voltage: float = 0.2
    seed: int = 135
    nonidealities: Nonidealities = Nonidealities()
    rows_per_read: object = None
    input_slice: object = None
    weight_slice: object = None
    bw_e: object = None
    weight_signed: bool = True

    def __post_init__(self):
        _require_int(self.activation_bits, "activation_bits", 2, 32)
        _require_int(self.weight_bits, "weight_bits", 2, 32)
        if type(self.weight_signed) is not bool:
            raise ValueError("weight_signed must be a boolean")
        if self.bw_e is not None:
            _require_int(self.bw_e, "bw_e", 2, 11)
            if not self.weight_signed:
                raise ValueError("unsigned weights require INT quantization (bw_e=None)")
        if self.input_slice is not None:
            object.__setattr__(
                self,
                "input_slice",
                _slice_widths(self.input_slice, "input_slice", self.activation_bits, True),
            )
        if self.weight_slice is not None:
            object.__setattr__(
                self,
                "weight_slice",
                _slice_widths(
                    self.weight_slice, "weight_slice", self.weight_bits, self.weight_signed
                ),
            )
        if isinstance(self.adc_bits, (tuple, list)):
            resolutions = tuple(self.adc_bits)
            if len(resolutions) != len(self.weight_layout):
                raise ValueError("adc_bits must have one entry per weight slice, MSB first")
            for bits in resolutions:
                _require_int(bits, "adc_bits", 1, 16)
            object.__setattr__(self, "adc_bits", resolutions)
        else:
            _require_int(self.adc_bits, "adc_bits", 1, 16)
        # Worst-case |sum_a sum_w s_a s_w count| must fit the signed 64-bit totals.
        input_weight = sum(abs(factor) for _, _, factor in self.input_layout)
        weight_weight = sum(
            abs(factor) * maximum
            for (_, _, factor), maximum in zip(self.weight_layout, self.adc_maxima)
        )
        if input_weight * weight_weight > 2**63 - 1:
            raise ValueError(
                "slice reconstruction exceeds the signed 64-bit accumulator; "
                "reduce precision, ADC bits, or use wider multibit slices"
            )
        _require_int(self.seed, "seed", 0, 2**32 - 1)
        for name in ("array_size", "weight_quant_gran", "input_quant_gran"):
            pair = getattr(self, name)
            if not isinstance(pair, tuple) or len(pair) != 2:
                raise ValueError(f"{name} must be a pair")
            for value in pair:
                if value is None and name != "array_size":
                    continue
                _require_int(value, name, 1, 65536)
        rows, columns = self.array_size
        if self.rows_per_read is not None:
            _require_int(self.rows_per_read, "rows_per_read", 1, rows)
        if columns % 4:
            raise ValueError("array columns must be divisible by four")
        for group in (self.weight_quant_gran[0], self.input_quant_gran[1]):
            if group is None or group % rows == 0:
                continue
            if rows % self.read_rows != 0 or group % self.read_rows != 0:
                raise ValueError(
                    "reduction scale groups must align with every ADC read boundary; "
                    "use a multiple of array rows, or a multiple of rows_per_read "
                    "when it divides array rows"
                )
        for name in ("high_conductance", "low_conductance", "read_voltage"):
            value = getattr(self, name)
            _require_nonnegative(value, name)
            if value <= 0:
                raise ValueError(f"{name} must be positive")
        if self.high_conductance <= self.low_conductance:
            raise ValueError("high_conductance must exceed low_conductance")
        try:
            high32 = struct.unpack("f", struct.pack("f", self.high_conductance))[0]
            low32 = struct.unpack("f", struct.pack("f", self.low_conductance))[0]
        except OverflowError:
            raise ValueError("conductances must be representable in FP32") from None
        if not (0 < low32 < high32 <= _FLT_MAX):
            raise ValueError("conductances must remain distinct and positive in FP32")
        if not _FLT_TRUE_MIN <= self.read_voltage <= _FLT_MAX:
            raise ValueError("read_voltage must be representable in FP32")
        if not 1 / _FLT_MAX <= self.current_unit <= _FLT_MAX:
            raise ValueError("current unit and reciprocal must be representable in FP32")
        if not isinstance(self.nonidealities, Nonidealities):
            raise TypeError("nonidealities must be Nonidealities")

    # ----------------------------------------------------------- derived layout
    @property
    def current_unit(self):
        """Current of one ideal digit-product count: (G_high - G_low) * V_read."""
        return (self.high_conductance - self.low_conductance) * self.read_voltage

    @property
    def adc_maxima(self):
        """ADC count limits in least-significant-slice-first order."""
        if type(self.adc_bits) is int:
            per_slice = (self.adc_bits,) * len(self.weight_layout)
        else:
            per_slice = tuple(reversed(self.adc_bits))
        return tuple((1 << bits) - 1 for bits in per_slice)

    @property
    def adc_maximum(self):
        return max(self.adc_maxima)

    @property
    def read_rows(self):
        return self.array_size[0] if self.rows_per_read is None else self.rows_per_read

    @property
    def reads_per_array(self):
        return -(-self.array_size[0] // self.read_rows)

    @staticmethod
    def _layout(widths, bits, signed=True):
        """(shift, mask, signed factor) per slice, least significant slice first."""
        widths = (1,) * bits if widths is None else widths
        table, shift = [], 0
        order = tuple(reversed(widths))
        for index, width in enumerate(order):
            factor = 1 << shift
            if signed and index == len(order) - 1:
                factor = -factor
            table.append((shift, (1 << width) - 1, factor))
            shift += width
        return tuple(table)

    @property
    def input_layout(self):
        return self._layout(self.input_slice, self.activation_bits)

    @property
    def weight_layout(self):
        return self._layout(self.weight_slice, self.weight_bits, self.weight_signed)

    @property
    def wide(self):
        """FP64 scales and reconstruction (``config.py:211-213``)."""
        return max(self.activation_bits, self.weight_bits) > 8 or self.bw_e is not None

    @property
    def wide_codes(self):
        """Codes are stored as int64 instead of uint8 (``quantization.py:101,133``)."""
        return max(self.activation_bits, self.weight_bits) > 8

    @property
    def precise_currents(self):
        """Use FP64 where physical FP32 rounding can change ideal ADC counts."""
        masks = [mask for _, mask, _ in (*self.input_layout, *self.weight_layout)]
        return (
            max(masks) > 255
            or self.high_conductance - self.low_conductance < self.high_conductance * 1e-4
            or self.high_conductance * self.read_voltage * self.read_rows > 8e37
            or min(self.low_conductance, self.read_voltage) < 1e-18
            or max(self.high_conductance, self.read_voltage) > 1e18
        )
