"""Natural-order analog matrix products (memfast/functional.py behaviour).

``mm(A, B)`` and ``matmul(A, B)`` follow torch.mm / torch.matmul shapes,
batching and dtype rules (functional.py:32-220).  The right-hand matrix is
programmed through ``Simulator._matrix_for``; each independently indexed
batched right-hand matrix is its own program, and broadcast copies share one.
Autograd is outside this engine's scope: the analog forward is inference-only,
so inputs that require grad are rejected with a clear error instead of
silently dropping gradients.
"""

import math
import weakref
from pathlib import Path

import torch

from . import _lib
from .config import Config
from .quantization import check_finite, compute_dtype, finite_flags
from .simulator import Simulator

_FLOATING = (torch.float16, torch.bfloat16, torch.float32, torch.float64)


def _operand_types(a, b):
    """Types, layouts, ranks, dtypes and devices of an operand pair (no device work)."""
    for name, value in (("A", a), ("B", b)):
        if not isinstance(value, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if value.layout != torch.strided or value.dtype not in _FLOATING:
            raise TypeError(f"{name} must be a real floating dense tensor")
        if value.ndim == 0:
            raise ValueError(f"{name} must have at least one dimension")
    if a.dtype != b.dtype:
        raise ValueError("A and B must have the same dtype")
    if a.device != b.device:
        raise ValueError("A and B must use the same device")
    if a.device.type != "cuda":
        raise ValueError("memfast_b200 simulates on CUDA operands only")


def _operands(a, b):
    """The checks above plus finiteness of both operands (one synchronisation)."""
    _operand_types(a, b)
    for name, finite in zip("AB", finite_flags(a, b)):
        if not finite:
            raise ValueError(f"{name} must be finite")


# Errors of a deferred operand check, in the reference's order: _operands (A, then
# B, each in its own dtype), then the quantisers (B is programmed before A is
# quantised) in the dtype they compute in (quantization.py:14-15).
OPERAND_ERRORS = {1: "A must be finite", 2: "B must be finite",
                  3: f"quantized values must be finite in {torch.float32}"}


def _operand_code(a, b, config):
    """Device int32 flags [operand error, output]: the first holds 0 when A and B pass
    the checks above, else the OPERAND_ERRORS key of the first failure, checked in that
    order on the device (no synchronisation); the second is left for the output check."""
    a_narrows = a.dtype == torch.float64 and compute_dtype(config, config.activation_bits) == torch.float32
    b_narrows = b.dtype == torch.float64 and compute_dtype(config, config.weight_bits) == torch.float32
    if (a.dtype not in _lib.DTYPES or b.dtype not in _lib.DTYPES or not a.is_contiguous()
            or not b.is_contiguous()):
        flags = torch.zeros(2, dtype=torch.int32, device=a.device)
        check_finite(a, flags[:1], 1)
        check_finite(b, flags[:1], 2, 3 if b_narrows else 0)
        if a_narrows:
            check_finite(a, flags[:1], 1, 3)
        return flags
    # One native call clears the flags and runs the checks in the order above.
    flags = torch.empty(2, dtype=torch.int32, device=a.device)
    _lib.check(_lib.load().mf_check_operands(
        _lib.ptr(a), _lib.DTYPES[a.dtype], a.numel(), 3 if a_narrows else 0,
        _lib.ptr(b), _lib.DTYPES[b.dtype], b.numel(), 3 if b_narrows else 0,
        _lib.ptr(flags), 2, _lib.stream_of(a.device)), "mf_check_operands")
    return flags


def _native_product(a, b, simulator, *, vector_offset=0, out=None, before_sync=None, peers=()):
    """A rank-two product through the one-call native path (``AnalogMatrix._native_mm``)
    when ``b`` already has a program that this call would reprogram in place and the
    operands are contiguous kernel dtypes; None otherwise (the caller then takes the
    step-by-step path, which gives the same result)."""
    if torch.is_grad_enabled() and (a.requires_grad or b.requires_grad):
        raise NotImplementedError(
            "memfast_b200 simulates the analog forward only; detach operands or use torch.no_grad()"
        )
    config = simulator.config
    if (a.dtype not in _lib.DTYPES or b.dtype != a.dtype or not a.is_contiguous() or not b.is_contiguous()
            or not config.weight_signed):
        return None
    matrix = simulator._in_place_program(b)
    scale_dtype = torch.float64 if config.wide else torch.float32
    if (matrix is None or not matrix.packed.is_contiguous() or not matrix.weight_scale.is_contiguous()
            or matrix.weight_scale.dtype != scale_dtype):
        return None
    a_narrows = a.dtype == torch.float64 and compute_dtype(config, config.activation_bits) == torch.float32
    b_narrows = b.dtype == torch.float64 and compute_dtype(config, config.weight_bits) == torch.float32
    with torch.no_grad():
        return matrix._native_mm(a.detach(), b.detach(), a_narrow=3 if a_narrows else 0,
                                 b_narrow=3 if b_narrows else 0, input_errors=OPERAND_ERRORS,
                                 vector_offset=vector_offset, out=out, before_sync=before_sync, peers=peers)


def _resolve_simulator(a, simulator, config, mode, cache_dir):
    """The simulator a call runs on: the caller's (whose settings the explicit options
    must agree with) or, without one, a new simulator for this call."""
    if mode not in ("default", "tuned"):
        raise ValueError("mode must be default or tuned")
    if config is not None and not isinstance(config, Config):
        raise TypeError("config must be Config")
    if simulator is None:
        return Simulator(config, mode=mode, device=a.device, cache_dir=cache_dir)
    if not isinstance(simulator, Simulator):
        raise TypeError("simulator must be Simulator")
    disagreements = (
        (simulator.device != a.device, "operands and simulator must use the same device"),
        (config is not None and config != simulator.config, "config differs from the supplied simulator"),
        (mode != "default" and mode != simulator.mode, "mode differs from the supplied simulator"),
        (cache_dir is not None and Path(cache_dir) != simulator.cache_dir,
         "cache_dir differs from the supplied simulator"),
    )
    for disagrees, message in disagreements:
        if disagrees:
            raise ValueError(message)
    return simulator


def _check_out(a, b, out, shape):
    """``out=`` must be a dense tensor of the result's shape, dtype and device."""
    if out is None:
        return
    if not isinstance(out, torch.Tensor) or out.layout != torch.strided:
        raise TypeError("out must be a dense torch.Tensor")
    if out.shape != shape or out.dtype != a.dtype or out.device != a.device:
        raise ValueError("out must have the result shape, dtype, and device")
    if torch.is_grad_enabled() and (a.requires_grad or b.requires_grad or out.requires_grad):
        raise RuntimeError("out= does not support automatic differentiation")


class _RhsViews:
    """Detached views of a batched right-hand operand, one per batch index, stable
    across calls with the same operand (so each keeps its program and read events)
    without keeping the caller's tensor alive."""

    def __init__(self):
        self._owners = {}

    @staticmethod
    def of(simulator):
        views = getattr(simulator, "_rhs_views", None)
        if views is None:
            views = simulator._rhs_views = _RhsViews()
        return views

    def view(self, owner, rhs, index):
        geometry = (tuple(owner.shape), tuple(owner.stride()), owner.storage_offset(), owner.data_ptr(),
                    owner.dtype, owner.device, owner.is_neg())
        entry = self._owners.get(id(owner))
        if entry is None or entry["owner"]() is not owner or entry["geometry"] != geometry:
            token = object()
            entry = dict(owner=weakref.ref(owner), geometry=geometry, views={}, token=token)
            self._owners[id(owner)] = entry
            weakref.finalize(owner, _RhsViews._forget, weakref.ref(self), id(owner), token)
        # detach() shares storage and version with the caller's tensor, not its identity.
        return entry["views"].setdefault(index, rhs.detach())

    @staticmethod
    def _forget(views_ref, key, token):
        views = views_ref()
        if views is not None and views._owners.get(key, {}).get("token") is token:
            del views._owners[key]


def _checked(tensor, config, bits):
    """_operands verified finiteness in the tensor's own dtype; that covers the
    quantiser's dtype unless FP64 values are narrowed to FP32."""
    return not (tensor.dtype == torch.float64 and compute_dtype(config, bits) == torch.float32)


def _product(a, b, simulator, cached_rhs=None, operand_code=None):
    """One programmed product.  ``operand_code``: the deferred operand check
    (``_operand_code``), read with the output check in one synchronisation; None when
    the caller already checked the operands."""
    if torch.is_grad_enabled() and (a.requires_grad or b.requires_grad):
        raise NotImplementedError(
            "memfast_b200 simulates the analog forward only; detach operands or use torch.no_grad()"
        )
    config = simulator.config
    deferred = operand_code is not None
    matrix = simulator._matrix_for(b if cached_rhs is None else cached_rhs,
                                   checked=deferred or _checked(b, config, config.weight_bits),
                                   rows=math.prod(a.shape[:-1]))
    with torch.no_grad():
        return matrix._forward(a.detach(), checked=deferred or _checked(a, config, config.activation_bits),
                               input_flag=operand_code, input_errors=OPERAND_ERRORS if deferred else None)


def _batched_products(left, right, b, batch, rows, columns, engine):
    """Products of a batch whose right-hand matrices differ along some batch dimension.

    Every batch index maps to the right-hand matrix at its index with the broadcast
    dimensions set to 0.  Indices sharing one matrix form one product (their vectors
    stacked in batch order); the products run in the order of their matrices' flat
    index, which is also the order in which each first appears in the batch, so the
    programs take the same automatic names (and sampling seeds) as the reference's
    (functional.py:170-185)."""
    rhs_batch = right.shape[:-2]
    flat_left = left.reshape(-1, rows, left.shape[-1])
    rhs_of = torch.arange(math.prod(rhs_batch)).reshape((1,) * (len(batch) - len(rhs_batch)) + rhs_batch)
    rhs_of = rhs_of.expand(batch).reshape(-1)
    result = flat_left.new_empty((flat_left.shape[0], rows, columns))
    for flat in torch.unique(rhs_of).tolist():
        members = torch.nonzero(rhs_of == flat).flatten()
        index = tuple(int(i) for i in torch.unravel_index(torch.tensor(flat), rhs_batch))
        rhs = right[index]
        cached = _RhsViews.of(engine).view(b, rhs, index)
        result[members.to(flat_left.device)] = _product(flat_left[members.to(flat_left.device)], rhs, engine, cached)
    return result.reshape(batch + (rows, columns))


def _matmul(a, b, *, simulator, config, mode, cache_dir, out):
    _operand_types(a, b)
    left = a.unsqueeze(0) if a.ndim == 1 else a
    right = b.unsqueeze(-1) if b.ndim == 1 else b
    if left.shape[-1] != right.shape[-2]:
        raise ValueError("A and B have incompatible reduction dimensions")
    try:
        batch = torch.broadcast_shapes(left.shape[:-2], right.shape[:-2])
    except RuntimeError:
        raise ValueError("A and B batch dimensions cannot broadcast") from None
    rows, reduction, columns = left.shape[-2], left.shape[-1], right.shape[-1]
    shape = batch + (() if a.ndim == 1 else (rows,)) + (() if b.ndim == 1 else (columns,))
    _check_out(a, b, out, shape)
    engine = _resolve_simulator(a, simulator, config, mode, cache_dir)
    if (a.ndim == 2 and b.ndim == 2 and out is None and a.numel() and b.numel()
            and not torch.is_autocast_enabled(a.device.type)):
        # Plain rank-two product outside autocast: one programmed product, no batch
        # bookkeeping (the general path below gives the same result); a matrix
        # programmed before goes through the one-call native path.
        native = _native_product(a, b, engine)
        if native is not None:
            return native
        return _product(a, b, engine, None, operand_code=_operand_code(a, b, engine.config))
    with torch.autocast(device_type=a.device.type, enabled=False):
        if a.numel() == 0 or b.numel() == 0 or 0 in shape:
            _operands(a, b)
            result = a.new_zeros(shape)
        else:
            left = left.expand(batch + (rows, reduction))
            if all(size == 1 for size in right.shape[:-2]):
                # One right-hand matrix: the operand check is read with the output check.
                rhs = right if right.ndim == 2 else right.reshape(reduction, columns)
                cached = None if b.ndim == 2 else _RhsViews.of(engine).view(b, rhs, ())
                result = _product(left, rhs, engine, cached, operand_code=_operand_code(a, b, engine.config))
            else:
                _operands(a, b)
                result = _batched_products(left, right, b, batch, rows, columns, engine)
            result = result.reshape(shape)
    if out is not None:
        out.copy_(result)
        return out
    return result


def mm(input, mat2, *, simulator=None, config=None, mode="default", cache_dir=None, out=None):
    """Simulate a rank-two A @ B with automatic RHS programming."""
    if not isinstance(input, torch.Tensor) or not isinstance(mat2, torch.Tensor):
        raise TypeError("A and B must be torch.Tensor operands")
    if input.ndim != 2 or mat2.ndim != 2:
        raise ValueError("mm requires two rank-two tensors")
    return _matmul(input, mat2, simulator=simulator, config=config, mode=mode, cache_dir=cache_dir, out=out)


def matmul(input, other, *, simulator=None, config=None, mode="default", cache_dir=None, out=None):
    """Simulate torch.matmul vector promotion and broadcast batch semantics."""
    return _matmul(input, other, simulator=simulator, config=config, mode=mode, cache_dir=cache_dir, out=out)


__all__ = ["mm", "matmul"]
