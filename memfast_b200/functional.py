"""Natural-order analog matrix products (memfast/functional.py behaviour).

``mm(A, B)`` and ``matmul(A, B)`` follow torch.mm / torch.matmul shapes,
batching and dtype rules (functional.py:32-220).  The RHS is programmed through
``Simulator._matrix_for``; each independently indexed batched RHS is its own
program, broadcast copies share one.  Autograd is outside this engine's scope:
the analog forward is inference-only, so inputs that require grad are rejected
with a clear error instead of silently dropping gradients.
"""

import itertools
import math
import weakref
from pathlib import Path

import torch

from . import _lib
from .config import Config
from .quantization import check_finite, compute_dtype, finite_flags
from .simulator import Simulator


def _operand_types(a, b):
    for name, value in (("A", a), ("B", b)):
        if not isinstance(value, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if value.layout != torch.strided or value.dtype not in (
            torch.float16, torch.bfloat16, torch.float32, torch.float64
        ):
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
    """Type, device and finiteness checks of an operand pair (one synchronisation)."""
    _operand_types(a, b)
    finite_a, finite_b = finite_flags(a, b)
    if not finite_a:
        raise ValueError("A must be finite")
    if not finite_b:
        raise ValueError("B must be finite")


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


def _engine(a, simulator, config, mode, cache_dir):
    if mode not in ("default", "tuned"):
        raise ValueError("mode must be default or tuned")
    if config is not None and not isinstance(config, Config):
        raise TypeError("config must be Config")
    if simulator is None:
        return Simulator(config, mode=mode, device=a.device, cache_dir=cache_dir)
    if not isinstance(simulator, Simulator):
        raise TypeError("simulator must be Simulator")
    if simulator.device != a.device:
        raise ValueError("operands and simulator must use the same device")
    if config is not None and config != simulator.config:
        raise ValueError("config differs from the supplied simulator")
    if mode != "default" and mode != simulator.mode:
        raise ValueError("mode differs from the supplied simulator")
    if cache_dir is not None and Path(cache_dir) != simulator.cache_dir:
        raise ValueError("cache_dir differs from the supplied simulator")
    return simulator


def _out(a, b, out, shape):
    if out is None:
        return
    if not isinstance(out, torch.Tensor) or out.layout != torch.strided:
        raise TypeError("out must be a dense torch.Tensor")
    if out.shape != shape or out.dtype != a.dtype or out.device != a.device:
        raise ValueError("out must have the result shape, dtype, and device")
    if torch.is_grad_enabled() and (a.requires_grad or b.requires_grad or out.requires_grad):
        raise RuntimeError("out= does not support automatic differentiation")


def _rhs_view(simulator, owner, rhs, index):
    """Stable detached cache keys that do not keep the caller's tensor alive."""
    cache = getattr(simulator, "_functional_rhs_views", None)
    if cache is None:
        cache = simulator._functional_rhs_views = {}
    identity = id(owner)
    geometry = (tuple(owner.shape), tuple(owner.stride()), owner.storage_offset(), owner.data_ptr(),
                owner.dtype, owner.device, owner.is_neg())
    record = cache.get(identity)
    if record is None or record[0]() is not owner or record[1] != geometry:
        engine = weakref.ref(simulator)

        def release(reference):
            instance = engine()
            if instance is not None:
                entries = instance._functional_rhs_views
                previous = entries.get(identity)
                if previous is not None and previous[0] is reference:
                    entries.pop(identity, None)

        record = (weakref.ref(owner, release), geometry, {})
        cache[identity] = record
    if index not in record[2]:
        record[2][index] = rhs.detach()
    return record[2][index]


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


def _matmul(a, b, *, simulator, config, mode, cache_dir, out):
    _operand_types(a, b)
    left_vector, right_vector = a.ndim == 1, b.ndim == 1
    left = a.unsqueeze(0) if left_vector else a
    right = b.unsqueeze(-1) if right_vector else b
    if left.shape[-1] != right.shape[-2]:
        raise ValueError("A and B have incompatible reduction dimensions")
    try:
        batch = torch.broadcast_shapes(left.shape[:-2], right.shape[:-2])
    except RuntimeError:
        raise ValueError("A and B batch dimensions cannot broadcast") from None
    rows, reduction, columns = left.shape[-2], left.shape[-1], right.shape[-1]
    shape = batch + (() if left_vector else (rows,)) + (() if right_vector else (columns,))
    _out(a, b, out, shape)
    engine = _engine(a, simulator, config, mode, cache_dir)
    if (a.ndim == 2 and b.ndim == 2 and out is None and a.numel() and b.numel()
            and not torch.is_autocast_enabled(a.device.type)):
        # Plain rank-two product outside autocast: one programmed product, no batch
        # bookkeeping (the general path below gives the same result).
        return _product(a, b, engine, None, operand_code=_operand_code(a, b, engine.config))
    with torch.autocast(device_type=a.device.type, enabled=False):
        if a.numel() == 0 or b.numel() == 0 or 0 in shape:
            _operands(a, b)
            result = a.new_zeros(shape)
        else:
            left = left.expand(batch + (rows, reduction))
            rhs_batch = right.shape[:-2]
            if all(size == 1 for size in rhs_batch):
                # One product: the operand check is read with the output check.
                rhs = right if right.ndim == 2 else right.reshape(reduction, columns)
                cached = None if b.ndim == 2 else _rhs_view(engine, b, rhs, ())
                result = _product(left, rhs, engine, cached, operand_code=_operand_code(a, b, engine.config))
            else:
                _operands(a, b)
                groups = {}
                padding = len(batch) - len(rhs_batch)
                for index in itertools.product(*(range(size) for size in batch)):
                    key = tuple(0 if size == 1 else index[padding + axis] for axis, size in enumerate(rhs_batch))
                    groups.setdefault(key, []).append(index)
                outputs = {}
                for key, indices in groups.items():
                    inputs = torch.stack([left[index] for index in indices])
                    rhs = right[key]
                    values = _product(inputs, rhs, engine, _rhs_view(engine, b, rhs, key))
                    outputs.update((index, values[row]) for row, index in enumerate(indices))
                result = torch.stack(
                    [outputs[index] for index in itertools.product(*(range(size) for size in batch))]
                ).reshape(batch + (rows, columns))
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
