"""Shared test helpers: golden-case loading and Config reconstruction."""

import hashlib
import json
from pathlib import Path

import numpy as np

from memfast_b200.config import Config, Nonidealities

GOLDEN = Path(__file__).resolve().parent / "golden"


def config_from_json(text):
    kwargs = json.loads(str(text))
    effects = kwargs.pop("nonidealities", {})
    for key in ("array_size", "weight_quant_gran", "input_quant_gran", "input_slice", "weight_slice"):
        if key in kwargs and kwargs[key] is not None:
            kwargs[key] = tuple(kwargs[key])
    if isinstance(kwargs.get("adc_bits"), list):
        kwargs["adc_bits"] = tuple(kwargs["adc_bits"])
    return Config(**kwargs, nonidealities=Nonidealities(**effects))


def seed_operands(n, k, o, seed):
    """A [n, k] and B [k, o], N(0,1) FP32 from numpy's PCG64 generator: scalar C code,
    so every host draws the same values (golden cases too large to store keep only
    the seed)."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal((n, k), dtype=np.float32), rng.standard_normal((k, o), dtype=np.float32)


def digest(*arrays):
    """Short SHA-256 of the arrays' bytes (C order)."""
    h = hashlib.sha256()
    for array in arrays:
        h.update(np.ascontiguousarray(array).tobytes())
    return h.hexdigest()[:24]


def load_case(name):
    """(config, arrays, meta) of a golden case; the operands of a seeded case are
    regenerated here, checked against the digest stored with the reference's output."""
    data = np.load(GOLDEN / f"{name}.npz")
    arrays = {key: data[key] for key in data.files if key not in ("config_json", "meta_json")}
    meta = json.loads(str(data["meta_json"]))
    if "seeded" in meta:
        a, b = seed_operands(*meta["shape"], meta["seeded"])
        assert digest(a, b) == meta["digest"], f"{name}: regenerated operands differ from the reference's"
        arrays.update(A=a, B=b)
    return config_from_json(data["config_json"]), arrays, meta


def mm_cases():
    names = []
    for path in sorted(GOLDEN.glob("*.npz")):
        meta = json.loads(str(np.load(path)["meta_json"]))
        if meta.get("kind") == "mm":
            names.append(path.stem)
    return names


def cases_of(kind):
    names = []
    for path in sorted(GOLDEN.glob("*.npz")):
        meta = json.loads(str(np.load(path)["meta_json"]))
        if meta.get("kind") == kind:
            names.append(path.stem)
    return names


def conv_arguments(conv):
    """Conv2d keyword arguments of a golden case as (kernel, stride, padding, dilation) pairs + the rest."""
    def pair(value):
        return tuple(value) if isinstance(value, (list, tuple)) else (value, value)

    return dict(kernel=pair(conv["kernel_size"]), stride=pair(conv.get("stride", 1)),
                padding=pair(conv.get("padding", 0)), dilation=pair(conv.get("dilation", 1)),
                groups=conv.get("groups", 1), padding_mode=conv.get("padding_mode", "zeros"))


# Nonideal currents are real-valued FP32 dot products.  Summing them in another
# order than the reference's CPU bmm flips an ADC rounding where a current sits
# within an ulp of a count boundary, and one flip of the most significant slice
# pair moves an output by |s_a s_w| * xs * ws (about 1% of the output range for
# INT8 (1,1,2,2,2) in small products; up to about 13% for the sign x sign pair of
# a 4096-deep product of N(0,1) operands, whose outputs are relatively smaller).
# Tolerance for such cases, stated once and used by every parity test:
#   - at most 0.5% of output elements differ, and at least two may (one or two
#     rounding flips in a product of a few hundred elements are the same event
#     at the same rate); when the caller states the ADC events behind each output
#     (reads x slice pairs), the bound is max(0.5%, 1e-5 per event): an output of
#     a 4096-deep INT8 product aggregates 3200 events, so flips at the same
#     per-event rate touch proportionally more outputs (the reference's own CPU
#     path and its restatement in the oracle differ on 0.23-0.29% of them there);
#   - no element differs by more than 5% of the output range (a few flips), or,
#     where the caller knows the operands' scales, by more than four flips of the
#     most significant slice pair (``flip`` = max |s_a s_w| * max xs * max ws);
#   - the RMS difference stays below 0.2% and the mean difference below 0.01%
#     of the range;
#   - the output distribution matches: mean within 0.1% of the std, std within 0.1%.
MISMATCH_FRACTION = 5e-3
FLIPS_PER_EVENT = 1e-5
MIN_MISMATCHES = 2


def adc_events(config, k):
    """ADC conversions behind one output of a k-deep product: reads x slice pairs."""
    arrays = -(-k // config.array_size[0])
    return arrays * config.reads_per_array * len(config.input_layout) * len(config.weight_layout)


def flip_size(config, a, b):
    """One ADC count of the most significant slice pair at the largest input and weight
    scales: the largest output change a single rounding flip can make."""
    from oracle import quantize as Q

    pair = max(abs(fa) for _, _, fa in config.input_layout) * max(abs(fw) for _, _, fw in config.weight_layout)
    return pair * float(Q.input_tiles(np.asarray(a), config)[1].max()) * \
        float(Q.weight_tiles(np.asarray(b).T, config)[1].max())
MAX_ERROR_OF_RANGE = 5e-2
RMS_ERROR_OF_RANGE = 2e-3
MEAN_ERROR_OF_RANGE = 1e-4
DISTRIBUTION_TOLERANCE = 1e-3


def assert_close_nonideal(got, want, label="", *, flip=None, events=None):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, label
    scale = max(np.abs(want).max(), 1e-30)
    diff = got - want
    fraction = MISMATCH_FRACTION if events is None else max(MISMATCH_FRACTION, FLIPS_PER_EVENT * events)
    assert np.sum(diff != 0) <= max(fraction * diff.size, MIN_MISMATCHES), (
        label, "mismatch fraction", np.mean(diff != 0), fraction)
    bound = MAX_ERROR_OF_RANGE * scale if flip is None else 4 * flip
    assert np.abs(diff).max() <= bound, (label, "max error", np.abs(diff).max() / scale, bound / scale)
    assert np.sqrt(np.mean(diff**2)) <= RMS_ERROR_OF_RANGE * scale, (label, "rms", np.sqrt(np.mean(diff**2)) / scale)
    assert abs(diff.mean()) <= MEAN_ERROR_OF_RANGE * scale, (label, "mean error", diff.mean() / scale)
    std = max(want.std(), 1e-30)
    assert abs(got.mean() - want.mean()) <= DISTRIBUTION_TOLERANCE * std, (label, "distribution mean")
    assert abs(got.std() / std - 1) <= DISTRIBUTION_TOLERANCE, (label, "distribution std")


def assert_parity(got, want, config, label="", *, flip=None, events=None):
    """Bit-exact for ideal devices; the nonideal tolerance above otherwise."""
    got = np.ascontiguousarray(got)
    want = np.ascontiguousarray(want)
    assert got.dtype == want.dtype and got.shape == want.shape, (label, got.dtype, want.dtype)
    if config.nonidealities.ideal:
        assert np.array_equal(got.view(np.uint8), want.view(np.uint8)), (
            label, np.mean(got != want), np.abs(got.astype(np.float64) - want).max())
    else:
        assert_close_nonideal(got, want, label, flip=flip, events=events)
