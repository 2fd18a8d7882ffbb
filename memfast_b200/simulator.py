"""Simulator and programmed analog matrices on the B200 engine.

Behavioural mirror of the reference ``memfast/simulator.py``:

* ``Simulator``      simulator.py:69-347  (device selection, programming of the
  right-hand matrix of ``mm`` with reuse of the previous program, tuned mode,
  ``report``);
* ``AnalogMatrix``   simulator.py:350-646 (buffers, name-derived sampling seed,
  read-event counter, zero-point correction, bias, non-finite FP64 rerun,
  checkpoint state).

What changes is the execution: ``AnalogMatrix._execute`` makes one
``mf_sliced_mm`` call for all output tiles (quantised codes in, finished
outputs out) instead of looping over tile groups and reducing partials in
PyTorch (simulator.py:561-586).  Tuned mode searches this engine's own grid
(``tuning.py``).  There is no CPU path: a Simulator lives on a CUDA device and
fails loudly otherwise.
"""

import ctypes as ct
import functools
import hashlib
import math
import types
import weakref
from dataclasses import asdict
from pathlib import Path

import torch
from torch import nn

from . import _lib, quantization, tuning
from .config import Config
from .quantization import (
    check_finite,
    check_read_scales,
    expanded_parameter,
    finite_flags,
    input_tiles,
    pack_weight,
    read_starts,
    weight_tiles,
)
from .tuning import atomic_write, cache_root, default_schedule, device_identity, schedule_grid, source_hash

ResourceError = _lib.ResourceError

_INTEGER_DTYPES = (torch.uint8, torch.int8, torch.int16, torch.int32, torch.int64)

# A matrix keeps its tensor-core workspace between calls only when the part rewritten
# by every call (the conductance operand of nonideal currents, beyond the K-major code
# copy) is at most this large; bigger ones come from the allocator per call, so that
# a model of many programmed layers holds one such buffer at a time, not one per layer.
_KEPT_SCRATCH_BYTES = 64 << 20


@functools.lru_cache(maxsize=4096)
def _workspace_bytes(config, n, m, p, schedule):
    """mf_sliced_mm_workspace for (config, n, m, p, schedule items), cached."""
    size = ct.c_size_t()
    native = _lib.schedule(**dict(schedule))
    _lib.check(
        _lib.load().mf_sliced_mm_workspace(_lib.native_config(config), ct.byref(native), n, m, p, 0, p,
                                           ct.byref(size)),
        "mf_sliced_mm_workspace",
    )
    return size.value


@functools.lru_cache(maxsize=1024)
def _kmajor_bytes(config, m, p, schedule):
    """K-major weight copy bytes of the schedule's kernel (mf_query), cached."""
    return tuning.resolve(config, dict(schedule), 1, m, p)[1].kmajor_bytes


def restore_scales(value, input_scale, weight_scale):
    """``value * input_scale * weight_scale`` in FP64 without overflow or underflow of
    the intermediate products (simulator.py:57-66): the three mantissas are multiplied
    (a product in [1/8, 1)) and the summed binary exponent is applied in two ldexp
    steps, each clamped to the normal range.  torch.ldexp scales by 2.0 ** e, so the
    steps match the reference's rounding."""
    parts = [torch.frexp(term.double()) for term in (value, input_scale, weight_scale)]
    mantissa = parts[0][0] * parts[1][0] * parts[2][0]
    exponent = parts[0][1] + parts[1][1] + parts[2][1]
    step = exponent.clamp(-1022, 1023)
    scaled = torch.ldexp(torch.ldexp(mantissa, step), exponent - step)
    return torch.where(mantissa == 0, 0.0, scaled)


def check_device_error():
    """Raise if a bounded device-side wait inside a kernel gave up (synchronises)."""
    code = ct.c_uint32()
    _lib.check(_lib.load().mf_take_device_error(ct.byref(code)), "device-side wait")


_STAGED_WORDS = {}


def _staged_word(device, stream):
    """The pinned host word receiving the device error word for (device, stream)."""
    key = (device.index, stream.value)
    word = _STAGED_WORDS.get(key)
    if word is None:
        if len(_STAGED_WORDS) >= 64:
            _STAGED_WORDS.pop(next(iter(_STAGED_WORDS)))
        word = _STAGED_WORDS[key] = torch.zeros(1, dtype=torch.int32, pin_memory=True)
    return word


def stage_device_error(device):
    """Enqueue a copy of the device error word into a pinned host word (per device and
    stream) and return that word: read it after the caller's next synchronisation of
    the current stream, and call check_device_error() when it is non-zero."""
    stream = _lib.stream_of(device)
    word = _staged_word(device, stream)
    _lib.check(_lib.load().mf_stage_device_error(word.data_ptr(), stream), "mf_stage_device_error")
    return word


def _tensor_layout(tensor):
    """What must be unchanged for a cached program of ``tensor`` to stay valid: its
    geometry, storage address, dtype and device (values are checked separately)."""
    return (tuple(tensor.shape), tuple(tensor.stride()), tensor.storage_offset(), tensor.data_ptr(), tensor.dtype,
            tensor.device)


class _ProgramCache:
    """Programs of right-hand operands, keyed by the operand tensor object.

    The reference reprograms ``B`` on every ``mm`` call and keeps the previous
    program when the new codes and scales are the same (simulator.py:133-171).
    An entry lives while its tensor does: a finalizer removes it, and a token
    makes sure a finalizer never removes a newer entry of a tensor that reuses
    the id.
    """

    def __init__(self):
        self._entries = {}

    def get(self, tensor):
        """(program, same_layout) of ``tensor``'s entry, or (None, False)."""
        entry = self._entries.get(id(tensor))
        if entry is None or entry["tensor"]() is not tensor:
            return None, False
        return entry["program"], entry["layout"] == _tensor_layout(tensor)

    def put(self, tensor, program):
        key, token = id(tensor), object()
        self._entries[key] = dict(tensor=weakref.ref(tensor), layout=_tensor_layout(tensor), program=program,
                                  token=token)
        weakref.finalize(tensor, _ProgramCache._drop, weakref.ref(self), key, token)

    @staticmethod
    def _drop(cache_ref, key, token):
        cache = cache_ref()
        if cache is not None and cache._entries.get(key, {}).get("token") is token:
            del cache._entries[key]

    def __len__(self):
        return len(self._entries)


def _budget_bytes(workspace_mb):
    if isinstance(workspace_mb, bool) or not isinstance(workspace_mb, (int, float)) or \
            not math.isfinite(workspace_mb) or workspace_mb <= 0:
        raise ValueError("workspace_mb must be positive and finite")
    return int(workspace_mb * 1024**2)


class Simulator:
    """Use fixed defaults or traverse the complete declared execution grid.

    ``tuned`` selects per input shape, saves the winner, and validates cached
    winners against default execution without timing candidates again.
    """

    def __init__(self, config=None, *, mode="default", device=None, cache_dir=None, workspace_mb=1024):
        config = Config() if config is None else config
        if not isinstance(config, Config):
            raise TypeError("config must be Config")
        if mode not in ("default", "tuned"):
            raise ValueError("mode must be default or tuned")
        budget = _budget_bytes(workspace_mb)
        device = torch.device(device or "cuda")
        if device.type != "cuda":
            raise ValueError("memfast_b200 runs on CUDA devices only; use the reference memfast package for CPU")
        if not torch.cuda.is_available():
            raise RuntimeError("CUDA is unavailable")
        _lib.load()
        self.config, self.mode, self.workspace_bytes = config, mode, budget
        self.device = torch.device("cuda", torch.cuda.current_device() if device.index is None else device.index)
        self.cache_dir = Path(cache_dir) if cache_dir is not None else cache_root() / "tuning"
        self.records = []
        self._selections = {}
        self._fingerprint = source_hash()
        self._programs = _ProgramCache()
        self._names = 0

    def _next_name(self):
        name = f"matrix.{self._names}"
        self._names += 1
        return name

    def map(self, weight, *, bias=None, name=None):
        """Low-level layer-weight adapter using PyTorch [O,K] weight layout."""
        return AnalogMatrix(weight, self, bias=bias, name=self._next_name() if name is None else name)

    def map_quantized(self, codes, scales, *, zero_points=None, bias=None, name=None):
        """Import integer [O,K] weights as ``scales * (codes - zero_points)``."""
        return AnalogMatrix(codes, self, bias=bias, name=self._next_name() if name is None else name, scales=scales,
                            zero_points=zero_points)

    def mm(self, input, mat2, *, out=None):
        """Simulate a two-dimensional matrix product, following torch.mm."""
        from .functional import mm

        return mm(input, mat2, simulator=self, out=out)

    def matmul(self, input, other, *, out=None):
        """Simulate a vector, matrix, or broadcast batch product like torch.matmul."""
        from .functional import matmul

        return matmul(input, other, simulator=self, out=out)

    def report(self):
        return dict(mode=self.mode, device=str(self.device), config=asdict(self.config), selections=self.records)

    def _matrix_for(self, matrix, checked=False, rows=1, program=None):
        """The programmed matrix for right-hand operand ``matrix`` [K, O] of a product.

        As in the reference, every call programs ``matrix``'s current values, and a
        program of the same tensor object keeps its name (sampling seed) and read
        event.  In default mode the cached module is reprogrammed in place (the
        result equals a new program with that name and event, so nothing is
        compared).  Tuned mode builds a new program and keeps the cached one when
        the codes and scales are unchanged, since the cached one also holds the
        schedules selected for it.  ``checked``: the caller verified the matrix
        finite in the quantiser's dtype; ``rows``: vectors of the coming product
        (sizes the tensor-core workspace); ``program``: a device copy of a host
        ``matrix`` to program from (the cache follows the caller's tensor).
        """
        cached, same_layout = self._programs.get(matrix)
        reusable = self._reusable(cached, same_layout)
        source = matrix if program is None else program
        if self.mode == "default" and reusable and cached.zero_correction is None and cached.input_scale is None:
            cached._reprogram(source.T, checked, rows)
            return cached
        name = self._next_name() if cached is None else cached.name
        fresh = AnalogMatrix(source.T, self, name=name, _checked=checked, _rows=rows)
        if self.mode == "tuned" and reusable and torch.equal(cached.packed, fresh.packed) and \
                torch.equal(cached.weight_scale, fresh.weight_scale):
            return cached
        if cached is not None:
            fresh._event = cached._event
        self._programs.put(matrix, fresh)
        return fresh

    def _reusable(self, cached, same_layout):
        return (cached is not None and same_layout and cached.packed.device == self.device
                and (cached.config is self.config or cached.config == self.config))

    def _in_place_program(self, matrix):
        """The cached program that ``_matrix_for(matrix)`` would reprogram in place
        (default mode, same layout, no imported zero points or fixed input scale), or
        None when that call would build a new program."""
        cached, same_layout = self._programs.get(matrix)
        if (self.mode == "default" and self._reusable(cached, same_layout) and cached.zero_correction is None
                and cached.input_scale is None):
            return cached
        return None

    def _select(self, matrix, x, q, xscale, event):
        """Tuned-mode schedule for ``matrix`` on inputs shaped like ``x`` (tuning.Search)."""
        return tuning.Search(self, matrix, x.shape, x.dtype, q, xscale, event).select(default_schedule(self.config))


# ----------------------------------------------------------- checkpoints --
def _check_checkpoint_codes(packed, config):
    if not torch.is_tensor(packed) or packed.dtype not in _INTEGER_DTYPES:
        raise ValueError("checkpoint packed weights must have an integer dtype")
    if packed.numel():
        low, high = torch.aminmax(packed.to(torch.int64))
        if low.item() < 0 or high.item() > (1 << config.weight_bits) - 1:
            raise ValueError("checkpoint packed weights exceed the configured bit width")


def _finite_nonnegative(tensor):
    return bool(torch.isfinite(tensor).all()) and not bool((tensor < 0).any())


def _check_checkpoint_scales(scales):
    if not torch.is_tensor(scales) or not scales.is_floating_point() or not _finite_nonnegative(scales):
        raise ValueError("checkpoint weight scales must be finite and nonnegative")


def _saved_configuration(saved):
    """A checkpoint's Config dictionary in today's form: the removed ``output_noise``
    effect must be zero and fields added since default (simulator.py:522-530)."""
    config = dict(saved)
    effects = dict(config["nonidealities"])
    if effects.pop("output_noise", 0) != 0:
        raise ValueError("checkpoint uses a removed noise model")
    config["nonidealities"] = effects
    for name in ("rows_per_read", "input_slice", "weight_slice", "bw_e"):
        config.setdefault(name, None)
    config.setdefault("weight_signed", True)
    return config


def _import_codes(codes, scales, zero_points, config, device):
    """Program integer [O, K] weight codes meaning ``scales * (codes - zero_points)``
    (simulator.py:173-185, 372-412): packed codes, per-read scales and, with zero
    points, the per-read correction ``-zero * scale`` applied digitally after the
    analog product."""
    if codes.dtype not in _INTEGER_DTYPES:
        raise ValueError("imported weight codes must have an integer dtype")
    if config.bw_e is not None:
        raise ValueError("native INT weight import requires bw_e=None")
    signed = config.weight_signed
    low = -(1 << (config.weight_bits - 1)) if signed else 0
    high = (1 << (config.weight_bits - int(signed))) - 1
    values = codes.detach().to(device=device, dtype=torch.int64)
    smallest, largest = torch.aminmax(values)
    if smallest.item() < low or largest.item() > high:
        raise ValueError("weight codes exceed configured signedness or bit width")
    dtype = torch.float64 if config.wide else torch.float32
    shape = codes.shape

    def per_element(value, name, **kwargs):
        # [K, O]: rows follow the reduction dimension, as the packed codes do.
        return expanded_parameter(value, shape, device, dtype, name, **kwargs).detach().T.contiguous()

    code_ko = values.T.contiguous()
    scale_ko = per_element(scales, "scales", positive=True)
    check_read_scales(scale_ko, config, "weight scale")
    packed, scale = pack_weight(code_ko, scale_ko, config)
    correction = None
    if zero_points is not None:
        zeros_ko = per_element(zero_points, "zero_points")
        check_read_scales(zeros_ko, config, "weight zero point")
        k = shape[1]
        first_rows = read_starts(math.ceil(k / config.array_size[0]), config, device).clamp_max(k - 1)
        correction = -(zeros_ko[first_rows] * scale_ko[first_rows])
        if not torch.isfinite(correction).all():
            raise ValueError("scaled zero points exceed the reconstruction dtype")
    return packed, scale, correction


class _NativePlan:
    """Buffers and ctypes arguments of ``AnalogMatrix._native_mm`` for one (vectors,
    stream) pair of one program: input codes and scales, check flags, quantiser
    scratch, the product workspace whose K-major prefix programming writes, and the
    mf_mm argument structures.  Valid while the program's buffers and this stream's
    workspace entry are the ones it was made for."""

    def __init__(self, matrix, a, b, stream):
        config, device = matrix.config, a.device
        n, k = a.shape
        o = b.shape[1]
        schedule = default_schedule(config)
        m = matrix.packed.shape[0]
        self.k, self.stream = k, stream.value
        self.workspace_bytes = matrix._workspace_size(n, schedule)
        kmajor_bytes = matrix._kmajor_size(m, schedule)
        entry = matrix._workspaces.get(stream.value)
        matrix._workspaces = {} if entry is None else {stream.value: entry}
        if kmajor_bytes and self.workspace_bytes - kmajor_bytes <= _KEPT_SCRATCH_BYTES:
            if entry is None or entry[0].numel() < self.workspace_bytes:
                entry = matrix._workspaces[stream.value] = [
                    torch.empty(self.workspace_bytes, dtype=torch.uint8, device=device), False]
            self.entry, self.workspace = entry, entry[0]
        else:
            self.entry = self.workspace = None
        matrix._kmajor_bytes = kmajor_bytes
        rows = config.array_size[0]
        self.out_dtype = torch.float64 if config.wide else torch.float32
        self.codes = torch.empty((n, m, rows), dtype=torch.int64 if config.wide_codes else torch.uint8,
                                 device=device)
        self.xscale = torch.empty((n, m * config.reads_per_array), dtype=self.out_dtype, device=device)
        self.flags = torch.empty(2, dtype=torch.int32, device=device)
        quantize_need = quantization.ct_size(config, False, n, k)
        program_need = quantization.ct_size(config, True, o, k)
        # One scratch serves both quantisers: the call runs them one after the other.
        self.scratch = quantization.scratch(max(quantize_need, program_need), device)
        self.packed_ptr, self.wscale_ptr = matrix.packed.data_ptr(), matrix.weight_scale.data_ptr()
        self.buffers = _lib.MFMMBuffers(
            self.codes.data_ptr(), self.xscale.data_ptr(), self.packed_ptr, self.wscale_ptr, None,
            self.flags.data_ptr(), self.scratch.data_ptr(), quantize_need, self.scratch.data_ptr(), program_need,
            None if self.workspace is None else self.workspace.data_ptr(), self.workspace_bytes)
        self.buffers_ref = ct.byref(self.buffers)
        self.config = _lib.native_config(config)
        self._schedule = _lib.schedule(**schedule)
        self.schedule = ct.byref(self._schedule)
        self.seed = matrix.seed & 0xFFFFFFFF
        self.word = _staged_word(device, stream)
        self.mm = _lib.load().mf_mm

    def valid(self, matrix, stream):
        return (matrix.packed.data_ptr() == self.packed_ptr and matrix.weight_scale.data_ptr() == self.wscale_ptr
                and (self.entry is None or (matrix._workspaces.get(stream) is self.entry
                                            and self.entry[0] is self.workspace)))


class AnalogMatrix(nn.Module):
    """Programmed matrix with optional digital zero-point compensation."""

    def __init__(self, weight, simulator, *, bias=None, name="matrix", scales=None, zero_points=None,
                 _checked=False, _rows=1):
        super().__init__()
        if weight.ndim != 2 or min(weight.shape) < 1:
            raise ValueError("weight must be a nonempty [O,K] matrix")
        if not _checked and not finite_flags(weight)[0]:
            raise ValueError("weights must be finite")
        config, device = simulator.config, simulator.device
        # Workspaces of the tensor-core kernels, one per stream, reused across calls:
        # each starts with the K-major copy of the packed codes (valid while flagged).
        self._workspaces, self._kmajor_bytes = {}, 0
        # One-call product plans (``_native_mm``), per (vectors, stream).
        self._native_plans = {}
        # Tensor-parallel column shard (sharding.shard_columns); None = all columns.
        self._column_shard = None
        self.simulator, self.config, self.name = simulator, config, name
        self.out_features, self.in_features = weight.shape
        self.p = math.ceil(self.out_features / config.array_size[1])
        reconstruction = torch.float64 if config.wide else torch.float32
        if scales is None:
            if not weight.is_floating_point():
                raise ValueError("unquantized weight must be floating")
            if zero_points is not None:
                raise ValueError("zero_points requires imported integer codes and scales")
            packed, scale = self._program_values(weight.detach().to(device), _checked, _rows)
            correction = None
        else:
            packed, scale, correction = _import_codes(weight, scales, zero_points, config, device)
        self.register_buffer("packed", packed)
        self.register_buffer("weight_scale", scale)
        self.register_buffer("zero_correction", correction)
        self.register_buffer("input_scale", None)
        if bias is not None and (not bias.is_floating_point() or bias.shape != (self.out_features,)
                                 or not torch.isfinite(bias).all()):
            raise ValueError("bias must be finite and match out_features")
        self.register_buffer("bias", None if bias is None else
                             bias.detach().to(device=device, dtype=reconstruction).clone())
        if self.bias is not None and not torch.isfinite(self.bias).all():
            raise ValueError("bias exceeds the reconstruction dtype")
        self._event = 0
        self.seed = config.seed ^ int.from_bytes(hashlib.sha256(name.encode()).digest()[:4], "little")
        self._prepared = {}

    def _program_values(self, weight, checked, rows):
        """Quantise and pack floating [O, K] weights, writing the tensor-core kernels'
        K-major copy into this stream's workspace in the same pass when they read one."""
        device = self.simulator.device
        self._prepare_workspace(math.ceil(self.in_features / self.config.array_size[0]), device, rows)
        entry = self._workspaces.get(_lib.stream_of(device).value)
        packed, scale, written = weight_tiles(weight, self.config, checked=checked,
                                              kmajor=None if entry is None else entry[0][: self._kmajor_bytes])
        if entry is not None:
            entry[1] = written
        return packed, scale

    def set_input_scale(self, scale):
        """Fix symmetric activation scales for subsequent calls; None restores dynamic scales."""
        if scale is None:
            self.input_scale = None
        else:
            dtype = torch.float64 if self.config.wide else torch.float32
            expanded = expanded_parameter(scale, (1, self.in_features), self.packed.device, dtype,
                                          "input scale").detach()
            if (expanded <= 0).any():
                raise ValueError("input scale must be strictly positive")
            check_read_scales(expanded.T, self.config, "input scale")
            self.input_scale = expanded.clone()
        self._prepared.clear()
        return self

    # ----------------------------------------------------------- checkpoints
    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        """Validate a checkpoint's buffers before loading them (simulator.py:452-493)."""
        if prefix + "packed" in state_dict:
            _check_checkpoint_codes(state_dict[prefix + "packed"], self.config)
        if prefix + "weight_scale" in state_dict:
            _check_checkpoint_scales(state_dict[prefix + "weight_scale"])
        # Optional buffers this module does not hold yet take the saved shape first.
        for optional in ("input_scale", "zero_correction"):
            saved = state_dict.get(prefix + optional)
            if saved is not None and self._buffers[optional] is None:
                self._buffers[optional] = torch.empty_like(saved, device=self.packed.device)
        super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)
        self._drop_workspace()
        if not _finite_nonnegative(self.weight_scale):
            raise ValueError("checkpoint weight scales exceed the reconstruction dtype")
        if self.bias is not None and not torch.isfinite(self.bias).all():
            raise ValueError("checkpoint bias exceeds the reconstruction dtype")
        if self.input_scale is not None:
            self.set_input_scale(self.input_scale)
        correction = self.zero_correction
        if correction is not None:
            if tuple(correction.shape) != (self.weight_scale.shape[0], self.out_features):
                raise ValueError("checkpoint zero-point correction has an invalid shape")
            if not torch.isfinite(correction).all():
                raise ValueError("checkpoint zero-point correction must be finite")

    def _apply(self, fn, recurse=True):
        """Device moves apply to the programmed buffers; dtype casts do not (the codes and
        scales are the device's programmed state).  A cast buffer is replaced by its
        original values on the new device, so no precision is lost."""
        originals = {name: tensor for name, tensor in self._buffers.items() if tensor is not None}
        super()._apply(fn, recurse=recurse)
        moved = False
        for name, original in originals.items():
            current = self._buffers[name]
            moved |= current.device != original.device
            if current.dtype != original.dtype:
                self._buffers[name] = original.to(device=current.device)
        if moved:
            self._prepared.clear()
            self._drop_workspace()
        return self

    def get_extra_state(self):
        return dict(config=asdict(self.config), in_features=self.in_features, out_features=self.out_features,
                    name=self.name, seed=self.seed, event=self._event)

    def set_extra_state(self, state):
        for dimension in ("in_features", "out_features"):
            saved = state.get(dimension, getattr(self, dimension))
            if type(saved) is not int or saved != getattr(self, dimension):
                raise ValueError("checkpoint logical matrix dimensions differ")
        if _saved_configuration(state["config"]) != asdict(self.config):
            raise ValueError("checkpoint physical configuration differs")
        seed = state["seed"]
        if type(seed) is not int or not 0 <= seed < 2**32:
            raise ValueError("invalid checkpoint sampling seed")
        self.reset_read(state["event"])
        self.name, self.seed = state["name"], seed
        self._prepared.clear()

    def reset_read(self, event=0):
        if type(event) is not int or not 0 <= event < 2**63:
            raise ValueError("event must be a nonnegative signed 64-bit integer")
        self._event = event

    @torch.no_grad()
    def update_weight(self, matrix):
        """Reprogram a right-hand [K,O] matrix without replacing this module."""
        if not isinstance(matrix, torch.Tensor) or tuple(matrix.shape) != (self.in_features, self.out_features):
            raise ValueError("replacement matrix must have the original [K,O] shape")
        replacement = AnalogMatrix(matrix.T, self.simulator, bias=self.bias, name=self.name)
        self.packed.copy_(replacement.packed)
        self.weight_scale.copy_(replacement.weight_scale)
        self._drop_workspace()
        self.zero_correction = None
        self._prepared.clear()
        self.reset_read()
        return self

    # --------------------------------------------------------------- engine
    def _kmajor_size(self, m, schedule):
        """Bytes of the K-major weight copy the schedule's kernel reads (0: none)."""
        return _kmajor_bytes(self.config, m, self.p, tuple(sorted(schedule.items())))

    def _prepare_workspace(self, m, device, rows=1):
        """Reserve the persistent workspace (sized for ``rows`` vectors) when the default
        schedule reads a K-major copy, so that programming can write that copy in place."""
        self._kmajor_bytes = self._kmajor_size(m, default_schedule(self.config))
        if self._kmajor_bytes:
            need = self._workspace_size(max(rows, 1), default_schedule(self.config), m)
            if need - self._kmajor_bytes > _KEPT_SCRATCH_BYTES:
                return   # a per-call workspace (see _launch): nothing to program in place
            self._workspaces[_lib.stream_of(device).value] = [torch.empty(need, dtype=torch.uint8, device=device),
                                                               False]

    def _reprogram(self, weight, checked, rows):
        """Program new [O, K] weights of this module's shape into its buffers, as the
        reference reprograms the right-hand matrix of every mm call (simulator.py:149)."""
        if not checked and not finite_flags(weight)[0]:
            raise ValueError("weights must be finite")
        device = self.packed.device
        stream = _lib.stream_of(device).value
        entry = self._workspaces.get(stream)
        self._workspaces = {} if entry is None else {stream: entry}
        if entry is None:
            self._prepare_workspace(self.packed.shape[0], device, rows)
            entry = self._workspaces.get(stream)
        _, _, written = weight_tiles(weight.detach(), self.config, checked=checked,
                                     kmajor=None if entry is None else entry[0][: self._kmajor_bytes],
                                     out=(self.packed, self.weight_scale))
        if entry is not None:
            entry[1] = written

    def _drop_workspace(self):
        self._workspaces.clear()

    @property
    def _ws(self):
        """The current stream's tensor-core workspace (None before the first call)."""
        entry = self._workspaces.get(_lib.stream_of(self.packed.device).value)
        return None if entry is None else entry[0]

    @property
    def _ws_ready(self):
        """Whether the current stream's workspace holds the K-major weight copy."""
        entry = self._workspaces.get(_lib.stream_of(self.packed.device).value)
        return entry is not None and entry[1]

    def _workspace_size(self, n, schedule, m=None):
        m = self.packed.shape[0] if m is None else m
        return _workspace_bytes(self.config, n, m, self.p, tuple(sorted(schedule.items())))

    def _execute(self, q, xscale, schedule, event, stable=False, *, vector_offset=0, input_flag=None,
                 input_errors=None, tiles=None, agree=None, output=None, before_sync=None, launched=None):
        """One fused device call: analog partials, scales, read sums and bias.

        ``input_flag``: device int32 set by a quantiser that checks finiteness on the
        device (or a deferred operand check); read in the same synchronisation as the
        output check, non-zero raising ``ValueError(input_errors[value])``.
        ``tiles``: output tiles [t0, t1) only (a column shard; noise addresses stay
        global), giving columns [t0*cols, min(t1*cols, out_features)).
        ``agree``: combines this shard's finiteness with the other shards' (the FP64
        rerun is decided for the whole product); ``output``: a buffer of the product's
        shape and dtype to write into (the FP64 rerun allocates its own);
        ``before_sync(output, flags)``: work to enqueue on the stream after the product
        and its checks but before the host reads the flags (collectives of a sharded
        product, which may also combine the flags of every rank); it runs again for
        the FP64 rerun.  ``launched``: (output, flags, staged error word) of a product
        already enqueued with its checks (``_native_mm``); only the synchronisation and
        what follows it remain."""
        if launched is None:
            output = self._launch(q, xscale, schedule, event, stable=stable, vector_offset=vector_offset,
                                  tiles=tiles, output=output)
            # One host synchronisation decides both the FP64 rerun of a narrow config
            # (simulator.py:614-615) and, in forward, the non-finite error.
            # flags: [input error code, output non-finite]; one device-to-host read.
            flags = input_flag if input_flag is not None else torch.zeros(2, dtype=torch.int32, device=q.device)
            check_finite(output, flags[1:2], 1)
            staged = stage_device_error(q.device)
        else:
            output, flags, staged = launched
        if before_sync is not None:
            before_sync(output, flags)
        bad, nonfinite = flags.tolist()
        if bad:
            raise ValueError((input_errors or {}).get(bad, "quantized values must be finite"))
        if staged[0]:
            check_device_error()
        self._finite = not nonfinite
        if agree is not None:
            self._finite = agree(self._finite)
        if not self.config.wide and not stable and not self._finite:
            return self._execute(q, xscale, schedule, event, stable=True, vector_offset=vector_offset, tiles=tiles,
                                 before_sync=before_sync)
        return output

    def _zero_point_correction(self, q, xscale, output, c0, c1, wide):
        """Add the digital zero-point correction of imported codes (simulator.py:587-611):
        per read, the sum of the signed input codes times the input scale times
        ``-zero * weight scale``, summed over reads."""
        n = q.shape[0]
        half = 1 << (self.config.activation_bits - 1)
        codes = (q.to(torch.int64).reshape(n, -1) ^ half) - half
        rows, read = self.config.array_size[0], self.config.read_rows
        spans = torch.nn.functional.pad(codes.reshape(n, -1, rows), (0, self.config.reads_per_array * read - rows))
        read_sums = spans.reshape(n, -1, read).sum(-1)
        if not wide:
            dtype = output.dtype
            output += (read_sums.to(dtype) * xscale.to(dtype)) @ self.zero_correction[:, c0:c1].to(dtype)
            return
        width = self.config.array_size[1]
        for begin in range(c0, c1, width):
            end = min(begin + width, c1)
            terms = restore_scales(read_sums[:, :, None], xscale[:, :, None],
                                   self.zero_correction[None, :, begin:end])
            output[:, begin - c0:end - c0] += terms.sum(1)

    def _launch(self, q, xscale, schedule, event, *, stable=False, vector_offset=0, tiles=None, output=None):
        """Enqueue the product on the current stream (no host synchronisation) into
        ``output`` ([n, shard width], allocated when None) and return it."""
        n = q.shape[0]
        wide = self.config.wide or stable
        dtype = torch.float64 if wide else torch.float32
        t0, t1 = (0, self.p) if tiles is None else tiles
        cols = self.config.array_size[1]
        c0, c1 = t0 * cols, min(t1 * cols, self.out_features)
        if output is None:
            output = torch.empty((n, c1 - c0), device=q.device, dtype=dtype)
        elif output.shape != (n, c1 - c0) or output.dtype != dtype or output.stride(-1) != 1:
            raise ValueError("output buffer does not match the product")
        # The kernels address output columns globally: hand them the buffer shifted
        # back by c0 columns (only columns >= c0 are written).
        base = ct.c_void_p(output.data_ptr() - c0 * output.element_size())
        fuse_bias = self.bias is not None and self.zero_correction is None
        workspace_bytes = self._workspace_size(n, schedule)
        packed = self.packed.contiguous()
        stream = _lib.stream_of(q.device)
        kmajor_ready = 0
        kmajor_bytes = 0 if stable else self._kmajor_size(packed.shape[0], schedule)
        if kmajor_bytes and workspace_bytes - kmajor_bytes > _KEPT_SCRATCH_BYTES:
            # Per-call workspace; its K-major copy is rebuilt by the call (a pass over the
            # packed codes, small next to the conductance operand the call writes).
            workspace = torch.empty(workspace_bytes, dtype=torch.uint8, device=q.device)
            kmajor_bytes = 0
        elif kmajor_bytes:
            # Tensor-core kernels: keep a workspace per stream (launches on different
            # streams may overlap), whose leading K-major weight copy stays valid
            # until the codes change; a larger one keeps the copy.
            entry = self._workspaces.get(stream.value)
            if entry is None:
                if len(self._workspaces) >= 4:
                    self._workspaces.pop(next(iter(self._workspaces)))
                entry = self._workspaces[stream.value] = [
                    torch.empty(workspace_bytes, dtype=torch.uint8, device=q.device), False]
            elif entry[0].numel() < workspace_bytes:
                grown = torch.empty(workspace_bytes, dtype=torch.uint8, device=q.device)
                if entry[1]:
                    grown[:kmajor_bytes].copy_(entry[0][:kmajor_bytes])
                entry[0] = grown
            self._kmajor_bytes = kmajor_bytes
            workspace, workspace_bytes, kmajor_ready = entry[0], entry[0].numel(), int(entry[1])
        else:
            workspace = torch.empty(max(workspace_bytes, 1), dtype=torch.uint8, device=q.device)
        native = _lib.schedule(**dict(schedule, kmajor_ready=kmajor_ready))
        _lib.check(
            _lib.load().mf_sliced_mm(
                _lib.native_config(self.config), ct.byref(native), _lib.ptr(q), _lib.ptr(xscale),
                _lib.ptr(packed), _lib.ptr(self.weight_scale.contiguous()),
                _lib.ptr(self.bias) if fuse_bias else None, base, n, packed.shape[0], self.p,
                self.out_features, output.stride(0), t0, t1, self.seed & 0xFFFFFFFF, event,
                vector_offset, int(stable), _lib.ptr(workspace), workspace_bytes, stream,
            ),
            "mf_sliced_mm",
        )
        if kmajor_bytes:
            entry[1] = True
        if self.zero_correction is not None:
            self._zero_point_correction(q, xscale, output, c0, c1, wide)
            if self.bias is not None:
                output += self.bias[c0:c1]
        return output

    def _native_mm(self, a, b, *, a_narrow=0, b_narrow=0, input_errors=None, vector_offset=0, out=None,
                   before_sync=None, peers=()):
        """``mm(a, b)`` on this default-mode program of ``b`` in one ``mf_mm`` call: the
        operand checks, ``b`` reprogrammed in place (with the K-major copy the kernel
        reads), ``a`` quantised, the fused product and the output check are enqueued
        together, as ``_matrix_for`` + ``_forward`` enqueue them one by one; the
        synchronisation, errors, FP64 rerun and read event follow as in ``_product``.
        ``a``/``b``: contiguous [n, K] / [K, O] of one dtype; ``a_narrow``/``b_narrow``:
        the narrowing-check codes of ``functional._operand_code``.  The buffers and
        argument structures of a (vectors, stream) pair are kept in a plan, so a
        repeated call only fills in the operand and output addresses.  ``peers``:
        addresses in other GPUs' output buffers (``sharding.PeerOutputs``) that the
        kernel also stores every output to."""
        n, o = a.shape[0], b.shape[1]
        stream = _lib.stream_of(a.device)
        plan = self._native_plans.get((n, stream.value))
        if plan is None or not plan.valid(self, stream.value):
            plan = _NativePlan(self, a, b, stream)
            if len(self._native_plans) >= 4:
                self._native_plans.pop(next(iter(self._native_plans)))
            self._native_plans[(n, stream.value)] = plan
        elif len(self._workspaces) > 1:
            # Programming rewrites the codes: K-major copies kept for other streams go stale.
            self._workspaces = {stream.value: plan.entry}
        if self._event >= 2**63:
            raise OverflowError("read-event counter exhausted")
        direct = out is not None and out.dtype == plan.out_dtype and out.shape == (n, o) and out.is_contiguous()
        output = out if direct else torch.empty((n, o), dtype=plan.out_dtype, device=a.device)
        workspace = plan.workspace
        if workspace is None:
            # Large per-call scratch (the conductance operand): from the allocator each call.
            workspace = torch.empty(max(plan.workspace_bytes, 1), dtype=torch.uint8, device=a.device)
            plan.buffers.mm_workspace = workspace.data_ptr()
        plan.buffers.out = output.data_ptr()
        plan.buffers.n_peers = len(peers)
        for index, address in enumerate(peers):
            plan.buffers.peer_out[index] = address
        _lib.check(plan.mm(plan.config, plan.schedule, a.data_ptr(), b.data_ptr(), _lib.DTYPES[a.dtype],
                           n, plan.k, o, a_narrow, b_narrow, plan.buffers_ref, plan.seed, self._event,
                           vector_offset, plan.word.data_ptr(), stream), "mf_mm")
        if plan.entry is not None:
            plan.entry[1] = True
        return self._product(plan.codes, plan.xscale, a.shape, a.dtype, vector_offset=vector_offset,
                             input_errors=input_errors, out=out, before_sync=before_sync,
                             launched=(output, plan.flags, plan.word))

    @torch.no_grad()
    def forward(self, x):
        shard = self._column_shard
        return self._forward(x) if shard is None else shard(self, x)

    def _forward(self, x, checked=False, vector_offset=0, tiles=None, agree=None, input_flag=None,
                 input_errors=None, out=None, before_sync=None):
        """forward(); ``checked``: the caller verified x finite in the quantiser's dtype;
        ``vector_offset``: global index of x's first vector (noise addresses of row shards);
        ``tiles``/``agree``: a column shard, as in ``_execute``; ``input_flag`` /
        ``input_errors``: a deferred operand check, as in ``_execute``; ``out``: a
        contiguous-rows [vectors, width] buffer of x's dtype receiving the result;
        ``before_sync``: as in ``_execute``."""
        if x.ndim < 1 or x.shape[-1] != self.in_features or not x.is_floating_point():
            raise ValueError("input must be floating with matching in_features")
        if x.device != self.packed.device or x.device != self.simulator.device:
            raise ValueError("input and simulator must use the same device")
        if self.weight_scale.dtype != (torch.float64 if self.config.wide else torch.float32):
            raise RuntimeError("keep simulator scale buffers at their mapped dtype")
        shape = x.shape
        cols = self.config.array_size[1]
        t0, t1 = (0, self.p) if tiles is None else tiles
        width = min(t1 * cols, self.out_features) - t0 * cols
        if x.numel() == 0:
            return x.new_empty((*shape[:-1], width))
        if self._event >= 2**63:
            raise OverflowError("read-event counter exhausted")
        q, xscale = input_tiles(x.reshape(-1, self.in_features), self.config, self.input_scale, checked=checked)
        output = self._product(q, xscale, shape, x.dtype, vector_offset=vector_offset, tiles=tiles, agree=agree,
                               input_flag=input_flag, input_errors=input_errors, out=out, before_sync=before_sync)
        return output.reshape(*shape[:-1], width)

    def _product(self, q, xscale, shape, dtype, *, vector_offset=0, input_flag=None, input_errors=None,
                 tiles=None, agree=None, out=None, before_sync=None, launched=None):
        """forward() from quantised codes on (simulator.py:631-646): schedule, product,
        non-finite checks, ``dtype`` result, read event.  ``shape``/``dtype`` describe
        the caller's input (tuned-mode key); ``input_flag`` as in ``_execute``."""
        event = self._event
        schedule = default_schedule(self.config)
        if self.simulator.mode == "tuned":
            key = tuple(shape), str(dtype)
            if key not in self._prepared:
                if input_flag is not None and input_flag[0].item():
                    raise ValueError((input_errors or {}).get(input_flag[0].item(), "quantized values must be finite"))
                with torch.cuda.device(q.device):
                    self._prepared[key] = self.simulator._select(
                        self, types.SimpleNamespace(shape=tuple(shape), dtype=dtype), q, xscale, event)
            schedule = self._prepared[key]
        direct = out if out is not None and out.dtype == (torch.float64 if self.config.wide else torch.float32) \
            else None
        output = self._execute(q, xscale, schedule, event, vector_offset=vector_offset, input_flag=input_flag,
                               input_errors=input_errors, tiles=tiles, agree=agree, output=direct,
                               before_sync=before_sync, launched=launched)
        finite = self._finite and (output.dtype == dtype or finite_flags(output, dtypes=[dtype])[0])
        if agree is not None:
            finite = agree(finite)
        output = output.to(dtype)
        if not finite:
            raise FloatingPointError("nonfinite analog output")
        if out is not None and output.data_ptr() != out.data_ptr():
            out.copy_(output)
            output = out
        self._event += 1
        return output


__all__ = ["Simulator", "AnalogMatrix", "default_schedule", "schedule_grid", "restore_scales", "atomic_write",
           "device_identity", "ResourceError"]
