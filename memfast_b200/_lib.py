"""ctypes binding of libmemfast_b200.so (C ABI in include/memfast_b200.h).

This module is the only place Python touches the native library.  It replaces
the reference's NVRTC loader (memfast/cuda.py:24-310): kernels are prebuilt for
sm_100a, so there is no runtime compilation and no PTX cache.  If the library is
missing the import fails loudly -- there is no CPU or PyTorch fallback.
"""

import ctypes as ct
import functools
import threading
from pathlib import Path

import torch

PACKAGE = Path(__file__).resolve().parent
LIBRARY = PACKAGE / "libmemfast_b200.so"
ABI_VERSION = 3
MAX_SLICES = 32
MAX_PEERS = 7

STATIC_QUANTIZE_SCRATCH_BYTES = 4 << 20
MF_OK, MF_ERR_INVALID, MF_ERR_RESOURCE, MF_ERR_CUDA, MF_ERR_UNSUPPORTED = range(5)
# mf_path: the kernel family of a thread's last mf_sliced_mm call (mf_last_path).
PATHS = {0: "none", 1: "generic_ideal", 2: "packed", 3: "fp8_planes", 4: "tc_currents", 5: "simt_currents"}
DTYPES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.float64: 3}


class ResourceError(RuntimeError):
    """A launch exceeds a kernel or device resource limit (memfast/cuda.py:15)."""


class MFConfig(ct.Structure):
    _fields_ = [
        ("abi_version", ct.c_int32),
        ("activation_bits", ct.c_int32), ("weight_bits", ct.c_int32),
        ("weight_signed", ct.c_int32), ("bw_e", ct.c_int32),
        ("n_in", ct.c_int32), ("n_w", ct.c_int32),
        ("in_shift", ct.c_int32 * MAX_SLICES), ("in_mask", ct.c_int32 * MAX_SLICES),
        ("in_factor", ct.c_int64 * MAX_SLICES),
        ("w_shift", ct.c_int32 * MAX_SLICES), ("w_mask", ct.c_int32 * MAX_SLICES),
        ("w_factor", ct.c_int64 * MAX_SLICES),
        ("adc_max", ct.c_int32 * MAX_SLICES),
        ("rows", ct.c_int32), ("cols", ct.c_int32),
        ("read_rows", ct.c_int32), ("reads", ct.c_int32),
        ("in_group_rows", ct.c_int32), ("in_group_cols", ct.c_int32),
        ("w_group_rows", ct.c_int32), ("w_group_cols", ct.c_int32),
        ("wide", ct.c_int32), ("wide_codes", ct.c_int32),
        ("precise_currents", ct.c_int32), ("read_mode", ct.c_int32), ("ideal", ct.c_int32),
        ("high", ct.c_double), ("low", ct.c_double), ("voltage", ct.c_double), ("unit", ct.c_double),
        ("write_var", ct.c_double), ("read_var", ct.c_double), ("volt_var", ct.c_double),
        ("nonlinear", ct.c_double), ("saf_low", ct.c_double), ("saf_high", ct.c_double),
        ("drift", ct.c_double),
    ]


class MFSchedule(ct.Structure):
    _fields_ = [("kernel", ct.c_int32), ("tile_n", ct.c_int32), ("tile_o", ct.c_int32),
                ("arrays", ct.c_int32), ("kmajor_ready", ct.c_int32), ("raster", ct.c_int32)]


class MFResources(ct.Structure):
    _fields_ = [("workspace_bytes", ct.c_size_t), ("threads", ct.c_int32),
                ("shared_bytes", ct.c_int32), ("registers", ct.c_int32),
                ("local_bytes", ct.c_int32), ("blocks_per_sm", ct.c_int32),
                ("kmajor_bytes", ct.c_size_t), ("path", ct.c_int32)]


class MFConv2d(ct.Structure):
    _fields_ = [(name, ct.c_int64) for name in ("batch", "channels", "height", "width",
                                                "stride_n", "stride_c", "stride_h", "stride_w")] + \
               [(name, ct.c_int32) for name in ("kernel_h", "kernel_w", "stride_y", "stride_x", "pad_h",
                                                "pad_w", "dilation_h", "dilation_w", "channel_begin",
                                                "group_channels")]


class MFMMBuffers(ct.Structure):
    _fields_ = [("codes", ct.c_void_p), ("xscale", ct.c_void_p), ("packed", ct.c_void_p), ("wscale", ct.c_void_p),
                ("out", ct.c_void_p), ("flags", ct.c_void_p),
                ("quantize_workspace", ct.c_void_p), ("quantize_workspace_bytes", ct.c_size_t),
                ("program_workspace", ct.c_void_p), ("program_workspace_bytes", ct.c_size_t),
                ("mm_workspace", ct.c_void_p), ("mm_workspace_bytes", ct.c_size_t),
                ("peer_out", ct.c_void_p * MAX_PEERS), ("n_peers", ct.c_int32)]


_VOID = ct.c_void_p
_SIGNATURES = {
    "mf_abi_version": (ct.c_int32, []),
    "mf_launch_count": (ct.c_uint64, []),
    "mf_last_path": (ct.c_int32, []),
    "mf_enable_peer_access": (ct.c_int, [ct.c_int32]),
    "mf_ipc_export": (ct.c_int, [ct.c_void_p, ct.c_void_p, ct.c_size_t, ct.POINTER(ct.c_size_t)]),
    "mf_ipc_open": (ct.c_int, [ct.c_void_p, ct.c_size_t, ct.POINTER(ct.c_void_p)]),
    "mf_ipc_close": (ct.c_int, [ct.c_void_p]),
    "mf_debug_stall_next_launch": (ct.c_int, [ct.c_int32, ct.c_int64]),
    "mf_last_error": (ct.c_int32, [ct.c_char_p, ct.c_size_t]),
    "mf_device_check": (ct.c_int, [ct.c_int32, ct.POINTER(ct.c_int32)]),
    "mf_quantize_workspace": (ct.c_int, [ct.POINTER(MFConfig), ct.c_int32, ct.c_int64, ct.c_int64,
                                         ct.POINTER(ct.c_size_t)]),
    "mf_quantize_input": (ct.c_int, [ct.POINTER(MFConfig), _VOID, ct.c_int32, ct.c_int64, ct.c_int64,
                                     ct.c_int64, _VOID, _VOID, _VOID, _VOID, ct.c_size_t, _VOID]),
    "mf_quantize_input_static": (ct.c_int, [ct.POINTER(MFConfig), _VOID, ct.c_int32, ct.c_int64, ct.c_int64,
                                            ct.c_int64, _VOID, _VOID, _VOID, _VOID]),
    "mf_program_rhs": (ct.c_int, [ct.POINTER(MFConfig), _VOID, ct.c_int32, ct.c_int64, ct.c_int64, ct.c_int64,
                                  _VOID, _VOID, _VOID, _VOID, ct.c_size_t, _VOID]),
    "mf_quantize_conv_input": (ct.c_int, [ct.POINTER(MFConfig), ct.POINTER(MFConv2d), _VOID, ct.c_int32,
                                          _VOID, _VOID, _VOID, _VOID, _VOID, ct.c_size_t, _VOID]),
    "mf_check_finite": (ct.c_int, [_VOID, ct.c_int32, ct.c_int64, ct.c_uint32, ct.c_uint32, _VOID, _VOID]),
    "mf_check_operands": (ct.c_int, [_VOID, ct.c_int32, ct.c_int64, ct.c_uint32, _VOID, ct.c_int32, ct.c_int64,
                                     ct.c_uint32, _VOID, ct.c_int32, _VOID]),
    "mf_conv_output": (ct.c_int, [ct.POINTER(MFConv2d), ct.POINTER(ct.c_int64), ct.POINTER(ct.c_int64)]),
    "mf_program_weights": (ct.c_int, [ct.POINTER(MFConfig), _VOID, ct.c_int32, ct.c_int64, ct.c_int64,
                                      ct.c_int64, _VOID, _VOID, _VOID, ct.c_size_t, _VOID]),
    "mf_sliced_mm": (ct.c_int, [ct.POINTER(MFConfig), ct.POINTER(MFSchedule), _VOID, _VOID, _VOID, _VOID,
                                _VOID, _VOID, ct.c_int64, ct.c_int32, ct.c_int32, ct.c_int32, ct.c_int64,
                                ct.c_int32, ct.c_int32, ct.c_uint32, ct.c_uint64, ct.c_int64, ct.c_int32,
                                _VOID, ct.c_size_t, _VOID]),
    "mf_mm": (ct.c_int, [ct.POINTER(MFConfig), ct.POINTER(MFSchedule), _VOID, _VOID, ct.c_int32, ct.c_int64,
                         ct.c_int64, ct.c_int64, ct.c_uint32, ct.c_uint32, ct.POINTER(MFMMBuffers), ct.c_uint32,
                         ct.c_uint64, ct.c_int64, _VOID, _VOID]),
    "mf_sliced_mm_workspace": (ct.c_int, [ct.POINTER(MFConfig), ct.POINTER(MFSchedule), ct.c_int64,
                                          ct.c_int32, ct.c_int32, ct.c_int32, ct.c_int32,
                                          ct.POINTER(ct.c_size_t)]),
    "mf_take_device_error": (ct.c_int, [ct.POINTER(ct.c_uint32)]),
    "mf_stage_device_error": (ct.c_int, [ct.c_void_p, ct.c_void_p]),
    "mf_query": (ct.c_int, [ct.POINTER(MFConfig), ct.POINTER(MFSchedule), ct.c_int64, ct.c_int32,
                            ct.c_int32, ct.POINTER(MFResources)]),
}

_lock = threading.Lock()
_handle = None


def load():
    """Load the library once; raise if it is absent or of another ABI."""
    global _handle
    if _handle is not None:
        return _handle
    with _lock:
        if _handle is None:
            if not LIBRARY.exists():
                raise ImportError(
                    f"{LIBRARY} is not built; run `python -m memfast_b200.build` "
                    "(memfast_b200 has no CPU fallback)"
                )
            handle = ct.CDLL(str(LIBRARY))
            for name, (restype, argtypes) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype, fn.argtypes = restype, argtypes
            version = handle.mf_abi_version()
            if version != ABI_VERSION:
                raise ImportError(f"libmemfast_b200 ABI {version}, expected {ABI_VERSION}")
            _handle = handle
    return _handle


def exported_symbols():
    return sorted(_SIGNATURES)


def last_error():
    buf = ct.create_string_buffer(1024)
    load().mf_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status, what):
    if status == MF_OK:
        return
    message = f"{what}: {last_error()}"
    if status == MF_ERR_INVALID:
        raise ValueError(message)
    if status == MF_ERR_RESOURCE:
        raise ResourceError(message)
    if status == MF_ERR_UNSUPPORTED:
        raise NotImplementedError(message)
    raise RuntimeError(message)


# native_config by object identity first: hashing a Config costs about a microsecond
# and the hot path asks several times per call.  Each entry keeps its Config alive,
# so an id cannot be reused while its entry exists.
_NATIVE_BY_ID = {}


def native_config(config):
    """mf_config for a (frozen, hashable) Config; derived values as the reference derives them."""
    entry = _NATIVE_BY_ID.get(id(config))
    if entry is not None and entry[0] is config:
        return entry[1]
    native = _native_config(config)
    if len(_NATIVE_BY_ID) >= 256:
        _NATIVE_BY_ID.pop(next(iter(_NATIVE_BY_ID)))
    _NATIVE_BY_ID[id(config)] = (config, native)
    return native


@functools.lru_cache(maxsize=256)
def _native_config(config):
    """Build the mf_config (equal Configs share one)."""
    ni = config.nonidealities
    c = MFConfig()
    c.abi_version = ABI_VERSION
    c.activation_bits, c.weight_bits = config.activation_bits, config.weight_bits
    c.weight_signed = int(config.weight_signed)
    c.bw_e = 0 if config.bw_e is None else config.bw_e
    c.n_in, c.n_w = len(config.input_layout), len(config.weight_layout)
    if max(c.n_in, c.n_w) > MAX_SLICES:
        raise ValueError(f"at most {MAX_SLICES} physical slices per operand are supported")
    for i, (shift, mask, factor) in enumerate(config.input_layout):
        c.in_shift[i], c.in_mask[i], c.in_factor[i] = shift, mask, factor
    for i, (shift, mask, factor) in enumerate(config.weight_layout):
        c.w_shift[i], c.w_mask[i], c.w_factor[i] = shift, mask, factor
    for i, maximum in enumerate(config.adc_maxima):
        c.adc_max[i] = maximum
    c.rows, c.cols = config.array_size
    c.read_rows, c.reads = config.read_rows, config.reads_per_array
    c.in_group_rows = config.input_quant_gran[0] or 0
    c.in_group_cols = config.input_quant_gran[1] or 0
    c.w_group_rows = config.weight_quant_gran[0] or 0
    c.w_group_cols = config.weight_quant_gran[1] or 0
    c.wide, c.wide_codes = int(config.wide), int(config.wide_codes)
    c.precise_currents = int(config.precise_currents)
    c.read_mode = ("shared", "slice_pair", "output").index(ni.read_mode)
    c.ideal = int(ni.ideal)
    c.high, c.low, c.voltage = config.high_conductance, config.low_conductance, config.read_voltage
    c.unit = config.current_unit
    c.write_var, c.read_var, c.volt_var = ni.write_variation, ni.read_variation, ni.voltage_variation
    c.nonlinear, c.saf_low, c.saf_high = ni.adc_nonlinearity, ni.stuck_at_low, ni.stuck_at_high
    c.drift = ni.drift_factor
    return c


def schedule(kernel=0, tile_n=32, tile_o=64, arrays=2, kmajor_ready=0, raster=0):
    return MFSchedule(kernel, tile_n, tile_o, arrays, kmajor_ready, raster)


def stream_of(device):
    """The device's current CUDA stream as a handle (without building a Stream object)."""
    index = device.index if isinstance(device, torch.device) else device
    if index is None:
        index = torch.cuda.current_device()
    return ct.c_void_p(torch._C._cuda_getCurrentRawStream(index))


def ptr(tensor):
    return None if tensor is None else ct.c_void_p(tensor.data_ptr())
