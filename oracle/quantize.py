"""TEST INFRASTRUCTURE ONLY -- numpy restatement of the reference quantisation.

Follows HUST-ISMD-Odyssey/MemFast v0.3.0 ``memfast/quantization.py``:

* ``grouped_quantize``  quantization.py:9-44   (INT and BFP group quantisation)
* ``read_starts``       quantization.py:76-79
* ``weight_tiles``      quantization.py:82-91
* ``pack_weight``       quantization.py:94-112
* ``input_tiles``       quantization.py:115-137

Every array operation uses the dtype the reference computes in (FP32 for
narrow INT, FP64 for wide/BFP), with round-half-to-even and the same clamps,
so codes and scales are bit-identical to the reference's.
"""

import math

import numpy as np


def _full(size, group):
    return size if group is None else group


def grouped_quantize(value, bits, granularity, bw_e=None, signed=True):
    dtype = np.float64 if bits > 8 or bw_e is not None else np.float32
    value = np.asarray(value).astype(dtype)
    if not np.isfinite(value).all():
        raise ValueError(f"quantized values must be finite in {np.dtype(dtype).name}")
    if not signed and ((value < 0).any() or bw_e is not None):
        raise ValueError("unsigned floating weights must be nonnegative INT values")
    rows, cols = value.shape
    gr = min(_full(rows, granularity[0]), rows)
    gc = min(_full(cols, granularity[1]), cols)
    nr, nc = math.ceil(rows / gr), math.ceil(cols / gc)
    padded = np.zeros((nr * gr, nc * gc), dtype)
    padded[:rows, :cols] = value
    grouped = padded.reshape(nr, gr, nc, gc)
    maximum = np.abs(grouped).max(axis=(1, 3), keepdims=True)
    upper = (1 << (bits - int(signed))) - 1
    if bw_e is None:
        scale = np.where(maximum > 0, maximum, dtype(1.0)).astype(dtype) / dtype(upper)
        scale = np.maximum(scale, np.nextafter(dtype(0), dtype(1))).astype(dtype)
        lower = -upper if signed else 0
    else:
        limit = (1 << (bw_e - 1)) - 1
        exponent = np.floor(np.log2(np.maximum(maximum, np.finfo(dtype).tiny)))
        exponent = np.clip(exponent, 1 - limit, limit)
        scale = np.power(2.0, exponent + 2 - bits).astype(dtype)
        lower = -(1 << (bits - 1))
    code = np.clip(np.rint(grouped / scale), lower, upper)
    code = code.reshape(nr * gr, nc * gc)[:rows, :cols].astype(np.int64)
    expanded = np.broadcast_to(scale, (nr, gr, nc, gc)).reshape(nr * gr, nc * gc)
    return code, np.ascontiguousarray(expanded[:rows, :cols])


def read_starts(partitions, config):
    physical = np.arange(partitions)[:, None] * config.array_size[0]
    reads = np.arange(config.reads_per_array)[None] * config.read_rows
    return (physical + reads).reshape(-1)


def _scale_dtype(config):
    return np.float64 if config.wide else np.float32


def pack_weight(code, scale, config):
    """Logical [K,O] codes -> packed [m,p,R,C] (int64 here) and [m*reads,p,C] scales."""
    k, o = code.shape
    r, c = config.array_size
    m, p = math.ceil(k / r), math.ceil(o / c)
    scale = np.asarray(scale).astype(_scale_dtype(config))
    padded = np.zeros((m * r, p * c), np.int64)
    padded[:k, :o] = code
    packed = padded & ((1 << config.weight_bits) - 1)
    packed = np.ascontiguousarray(packed.reshape(m, r, p, c).transpose(0, 2, 1, 3))
    scales = np.pad(scale, ((0, m * r - k), (0, p * c - o)), mode="edge")
    scales = scales[read_starts(m, config)].reshape(m * config.reads_per_array, p, c)
    return packed, np.ascontiguousarray(scales)


def weight_tiles(weight, config):
    """PyTorch-layout [O,K] floating weights -> (packed, weight_scale)."""
    code, scale = grouped_quantize(
        np.ascontiguousarray(np.asarray(weight).T),
        config.weight_bits,
        config.weight_quant_gran,
        config.bw_e,
        signed=config.weight_signed,
    )
    return pack_weight(code, scale, config)


def input_tiles(value, config, fixed_scale=None):
    """[n,K] activations -> codes [n,m,R] (int64 here) and per-read scales [n,m*reads]."""
    value = np.asarray(value)
    n, k = value.shape
    r = config.array_size[0]
    m = math.ceil(k / r)
    if fixed_scale is None:
        code, scale = grouped_quantize(
            value, config.activation_bits, config.input_quant_gran, config.bw_e
        )
    else:
        dtype = np.float64 if config.wide else np.float32
        scale = np.broadcast_to(np.asarray(fixed_scale).astype(dtype), value.shape)
        upper = (1 << (config.activation_bits - 1)) - 1
        lower = -(1 << (config.activation_bits - 1)) if config.bw_e is not None else -upper
        code = np.clip(np.rint(value.astype(dtype) / scale), lower, upper).astype(np.int64)
    scale = np.asarray(scale).astype(_scale_dtype(config))
    padded = np.zeros((n, m * r), np.int64)
    padded[:, :k] = code
    packed = padded & ((1 << config.activation_bits) - 1)
    scales = np.pad(scale, ((0, 0), (0, m * r - k)), mode="edge")
    scales = scales[:, read_starts(m, config)]
    return packed.reshape(n, m, r), np.ascontiguousarray(scales)
