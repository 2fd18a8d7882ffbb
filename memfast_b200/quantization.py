"""Device quantisation and packing (memfast/quantization.py behaviour, on CUDA).

* ``input_tiles``   -> ``mf_quantize_input``  (quantization.py:115-137 + :9-44)
* ``weight_tiles``  -> ``mf_program_weights`` (quantization.py:82-112 + :9-44)
* ``pack_weight``   packs already-integer codes for ``Simulator.map_quantized``
  (quantization.py:94-112) with device tensor ops; it runs once per programming.
* ``read_starts`` / ``check_read_scales`` / ``expanded_parameter`` keep the
  reference's semantics (quantization.py:47-79).

Every buffer keeps the reference layout: codes [n,m,R], per-read input scales
[n,m*reads], packed weights [m,p,R,C] and per-read weight scales [m*reads,p,C],
uint8 codes (int64 beyond 8 bits) and FP32 scales (FP64 when ``Config.wide``).
"""

import ctypes
import functools
import math

import torch
from torch.nn import functional as F

from . import _lib


def _code_dtype(config):
    return torch.int64 if config.wide_codes else torch.uint8


def _scale_dtype(config):
    return torch.float64 if config.wide else torch.float32


def _require_cuda(tensor, name):
    if not tensor.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (memfast_b200 runs on the GPU only)")


# Quantiser scratch, one growing buffer per (device, stream): calls on one stream
# run in order, so a buffer is reused only after the previous call's kernels.
_SCRATCH = {}


def _workspace(config, is_weight, rows, cols, device):
    need = ct_size(config, is_weight, rows, cols)
    return scratch(need, device), need


def scratch(need, device):
    """The current stream's quantiser scratch, at least ``need`` bytes."""
    key = (device.index, _lib.stream_of(device).value)
    buffer = _SCRATCH.get(key)
    if buffer is None or buffer.numel() < need:
        if len(_SCRATCH) >= 16:
            _SCRATCH.pop(next(iter(_SCRATCH)))
        buffer = _SCRATCH[key] = torch.empty(max(need, 1), dtype=torch.uint8, device=device)
    return buffer


@functools.lru_cache(maxsize=1024)
def ct_size(config, is_weight, rows, cols):
    import ctypes as ct

    size = ct.c_size_t()
    _lib.check(
        _lib.load().mf_quantize_workspace(
            ct.byref(_lib.native_config(config)), int(is_weight), rows, cols, ct.byref(size)
        ),
        "mf_quantize_workspace",
    )
    return size.value


def read_starts(partitions, config, device):
    physical = torch.arange(partitions, device=device)[:, None] * config.array_size[0]
    reads = torch.arange(config.reads_per_array, device=device)[None] * config.read_rows
    return (physical + reads).flatten()


def check_read_scales(value, config, name):
    """Each column has a single scale or zero point within one analog read."""
    indices = torch.arange(value.shape[0], device=value.device)
    physical_start = indices // config.array_size[0] * config.array_size[0]
    read_offset = (indices % config.array_size[0]) // config.read_rows * config.read_rows
    if not torch.equal(value, value[physical_start + read_offset]):
        raise ValueError(f"{name} changes inside an ADC read; reduce rows_per_read")


def expanded_parameter(value, shape, device, dtype, name, *, positive=False):
    original = (
        torch.as_tensor(value, device=device)
        if torch.is_tensor(value)
        else torch.as_tensor(value, device=device, dtype=torch.float64)
    )
    if original.is_complex() or not torch.isfinite(original).all():
        raise ValueError(f"{name} must be real and finite")
    if positive and (original < 0).any():
        raise ValueError(f"{name} must be finite and nonnegative")
    value = original.to(dtype)
    try:
        value = torch.broadcast_to(value, shape)
    except RuntimeError:
        raise ValueError(f"{name} must broadcast to {tuple(shape)}") from None
    if not torch.isfinite(value).all() or (positive and (value < 0).any()):
        raise ValueError(f"{name} must be finite" + (" and nonnegative" if positive else ""))
    return value


def finite_flags(*tensors, dtypes=None):
    """Whether each tensor holds only finite values (in ``dtypes[i]`` when given),
    with one device synchronisation: NaN propagates through aminmax and an
    infinity or an overflow on narrowing shows in the extremes."""
    extremes = []
    for index, tensor in enumerate(tensors):
        if tensor.numel() == 0:
            extremes.append(torch.zeros(2, device=tensor.device, dtype=torch.float64))
            continue
        low, high = torch.aminmax(tensor.detach())
        pair = torch.stack([low, high])
        if dtypes is not None and dtypes[index] is not None:
            pair = pair.to(dtypes[index])
        extremes.append(pair.to(torch.float64))
    return [bool(flag) for flag in torch.isfinite(torch.stack(extremes)).all(dim=1).tolist()]


def check_finite(tensor, flag, code, narrow_code=0):
    """Enqueue a finiteness check of ``tensor`` (no synchronisation): the device int32
    ``flag`` (a one-element view) becomes ``code`` if it is still 0 and a value is not
    finite, or ``narrow_code`` if an FP64 value overflows FP32 (``mf_check_finite``)."""
    if tensor.numel() == 0:
        return
    if tensor.dtype not in _lib.DTYPES:
        tensor = tensor.float()
    if not tensor.is_contiguous():
        tensor = tensor.contiguous()
    _lib.check(
        _lib.load().mf_check_finite(_lib.ptr(tensor), _lib.DTYPES[tensor.dtype], tensor.numel(), code, narrow_code,
                                    _lib.ptr(flag), _lib.stream_of(tensor.device)),
        "mf_check_finite",
    )


def compute_dtype(config, bits):
    """grouped_quantize computes in FP64 for wide codes or BFP, else FP32 (quantization.py:10-13)."""
    return torch.float64 if bits > 8 or config.bw_e is not None else torch.float32


def _as_native_float(value, config, bits, checked=False):
    """The float operand the kernels read (FP16/BF16/FP32/FP64), checked finite in the
    dtype grouped_quantize computes in (quantization.py:10-13).  ``checked`` marks an
    operand the caller already verified in that dtype."""
    if value.dtype not in _lib.DTYPES:
        value = value.float()
    if checked:
        return value
    compute = compute_dtype(config, bits)
    narrowed = value.dtype == torch.float64 and compute == torch.float32
    if not finite_flags(value, dtypes=[compute if narrowed else None])[0]:
        raise ValueError(f"quantized values must be finite in {compute}")
    return value


def input_tiles(value, config, fixed_scale=None, *, checked=False):
    """[n, K] activations -> (codes [n, m, R], per-read scales [n, m*reads]).

    ``checked``: the caller verified the activations finite in the quantiser's dtype."""
    _require_cuda(value, "input")
    n, k = value.shape
    r = config.array_size[0]
    m = math.ceil(k / r)
    codes = torch.empty((n, m, r), dtype=_code_dtype(config), device=value.device)
    xscale = torch.empty((n, m * config.reads_per_array), dtype=_scale_dtype(config), device=value.device)
    if n == 0:
        return codes, xscale
    if fixed_scale is None:
        value = _as_native_float(value, config, config.activation_bits, checked)
    else:
        if not checked and not finite_flags(value)[0]:
            raise ValueError("quantized values must be finite")
        if value.dtype not in _lib.DTYPES:
            value = value.float()
        fixed_scale = fixed_scale.to(_scale_dtype(config)).reshape(-1).contiguous()
        if fixed_scale.numel() != k:
            fixed_scale = fixed_scale.expand(k).contiguous()
    if value.stride(-1) != 1:
        value = value.contiguous()
    workspace, need = _workspace(config, False, n, k, value.device)
    _lib.check(
        _lib.load().mf_quantize_input(
            _lib.native_config(config), _lib.ptr(value), _lib.DTYPES[value.dtype], n, k, value.stride(0),
            _lib.ptr(fixed_scale), _lib.ptr(codes), _lib.ptr(xscale), _lib.ptr(workspace), need,
            _lib.stream_of(value.device),
        ),
        "mf_quantize_input",
    )
    return codes, xscale


def conv_input_tiles(x, config, geometry, fixed_scale=None):
    """One convolution group's patches -> (codes [n, m, R], per-read scales [n, m*reads], flag).

    The buffers ``input_tiles`` gives for the group's ``F.unfold`` patches laid
    out as [batch*OH*OW, Cg*kh*kw] (memfast/nn/convolution.py:49-55), quantised
    straight from the NCHW input ``x`` (any strides) without building them.
    ``geometry``: the group's ``_lib.MFConv2d`` (kernel, stride, padding, dilation,
    channels); ``x``'s shape and strides are filled in here.  ``flag`` is a device
    int32 pair whose first word the kernels set to 1 when a quantised value is not
    finite (the reference raises ValueError then); the second is for the output
    check."""
    _require_cuda(x, "input")
    if x.dtype not in _lib.DTYPES:
        x = x.float()
    geometry.batch, geometry.channels, geometry.height, geometry.width = x.shape
    geometry.stride_n, geometry.stride_c, geometry.stride_h, geometry.stride_w = x.stride()
    oh, ow = conv_output_size(geometry)
    n = x.shape[0] * oh * ow
    k = geometry.group_channels * geometry.kernel_h * geometry.kernel_w
    r = config.array_size[0]
    m = math.ceil(k / r)
    codes = torch.empty((n, m, r), dtype=_code_dtype(config), device=x.device)
    xscale = torch.empty((n, m * config.reads_per_array), dtype=_scale_dtype(config), device=x.device)
    flag = torch.zeros(2, dtype=torch.int32, device=x.device)   # [input error, output check]
    if n == 0:
        return codes, xscale, flag
    if fixed_scale is not None:
        fixed_scale = fixed_scale.to(_scale_dtype(config)).reshape(-1).contiguous()
        if fixed_scale.numel() != k:
            fixed_scale = fixed_scale.expand(k).contiguous()
        workspace, need = None, 0
    else:
        workspace, need = _workspace(config, False, n, k, x.device)
    _lib.check(
        _lib.load().mf_quantize_conv_input(
            _lib.native_config(config), ctypes.byref(geometry), _lib.ptr(x), _lib.DTYPES[x.dtype],
            _lib.ptr(fixed_scale), _lib.ptr(codes), _lib.ptr(xscale), _lib.ptr(flag), _lib.ptr(workspace), need,
            _lib.stream_of(x.device),
        ),
        "mf_quantize_conv_input",
    )
    return codes, xscale, flag


def conv_output_size(geometry):
    """(OH, OW) of a convolution group; ValueError when the window does not fit."""
    oh, ow = ctypes.c_int64(), ctypes.c_int64()
    _lib.check(_lib.load().mf_conv_output(ctypes.byref(geometry), ctypes.byref(oh), ctypes.byref(ow)),
               "mf_conv_output")
    return oh.value, ow.value


def weight_tiles(weight, config, *, checked=False, kmajor=None, out=None):
    """PyTorch-layout [O, K] floating weights -> (packed [m,p,R,C], weight_scale [m*reads,p,C], kmajor_written).

    ``checked``: the caller verified the weights finite in the quantiser's dtype.
    ``kmajor``: optional uint8 buffer for the K-major code copy of the tensor-core
    kernels; it is filled (and ``kmajor_written`` is True) when the weights are the
    transpose of a row-major [K, O] matrix, the right-hand operand of ``mm``, which
    is then programmed in place through ``mf_program_rhs``.  ``out``: (packed, weight_scale)
    buffers of the right shapes to program into instead of new ones."""
    _require_cuda(weight, "weight")
    o, k = weight.shape
    if not config.weight_signed and (weight < 0).any():
        raise ValueError(
            "unsigned floating weights must be nonnegative INT values; "
            "use map_quantized with zero_points for affine weights"
        )
    weight = _as_native_float(weight, config, config.weight_bits, checked)
    r, c = config.array_size
    m, p = math.ceil(k / r), math.ceil(o / c)
    if out is None:
        packed = torch.empty((m, p, r, c), dtype=_code_dtype(config), device=weight.device)
        wscale = torch.empty((m * config.reads_per_array, p, c), dtype=_scale_dtype(config), device=weight.device)
    else:
        packed, wscale = out
        if (packed.shape != (m, p, r, c) or packed.dtype != _code_dtype(config) or not packed.is_contiguous()
                or wscale.shape != (m * config.reads_per_array, p, c) or wscale.dtype != _scale_dtype(config)
                or not wscale.is_contiguous()):
            raise ValueError("programming buffers do not match the matrix")
    workspace, need = _workspace(config, True, o, k, weight.device)
    if weight.stride(0) == 1 and weight.stride(1) >= max(o, 1):
        # The transpose of a row-major [K, O] matrix: program it in place.
        rhs = weight.T
        _lib.check(
            _lib.load().mf_program_rhs(
                _lib.native_config(config), _lib.ptr(rhs), _lib.DTYPES[rhs.dtype], k, o, rhs.stride(0),
                _lib.ptr(packed), _lib.ptr(wscale), _lib.ptr(kmajor), _lib.ptr(workspace), need,
                _lib.stream_of(weight.device),
            ),
            "mf_program_rhs",
        )
        return packed, wscale, kmajor is not None
    if weight.stride(-1) != 1:
        weight = weight.contiguous()
    _lib.check(
        _lib.load().mf_program_weights(
            _lib.native_config(config), _lib.ptr(weight), _lib.DTYPES[weight.dtype], o, k, weight.stride(0),
            _lib.ptr(packed), _lib.ptr(wscale), _lib.ptr(workspace), need, _lib.stream_of(weight.device),
        ),
        "mf_program_weights",
    )
    return packed, wscale, False


def pack_weight(code, scale, config):
    """Pack logical [K,O] integer codes without estimating or changing their scales."""
    k, o = code.shape
    r, c = config.array_size
    m, p = math.ceil(k / r), math.ceil(o / c)
    scale = scale.to(_scale_dtype(config))
    padded = F.pad(code, (0, p * c - o, 0, m * r - k))
    packed = (padded & ((1 << config.weight_bits) - 1)).to(_code_dtype(config))
    packed = packed.reshape(m, r, p, c).permute(0, 2, 1, 3).contiguous()
    scales = F.pad(scale[None, None], (0, p * c - o, 0, m * r - k), mode="replicate")[0, 0]
    scales = scales[read_starts(m, config, code.device)].reshape(m * config.reads_per_array, p, c)
    return packed, scales.contiguous()
