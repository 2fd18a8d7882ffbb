"""``Simulator.mm`` on host operands with the PCIe copies overlapped.

A caller whose operands live in host memory (the reference's CPU users:
``memfast.mm(A, B)`` with CPU tensors, memfast/functional.py:130-208) gets the
same result as copying both operands to the GPU, calling ``Simulator.mm`` and
copying the product back, but the three phases run as a pipeline:

* copy stream: B, then A in row chunks (pinned host memory → HBM);
* compute streams (the caller's current stream and one more): program B in
  place once it has arrived (``mf_program_rhs``, with the tensor-core K-major
  copy), then per chunk, alternating between the two streams so that one
  launch's last wave overlaps the next launch, the input quantiser and one
  ``mf_sliced_mm`` launch into the chunk's rows of the device output, with
  ``vector_offset`` = the chunk's first row;
* copy-back stream: each finished chunk of rows → host.

Every row of A is independent when input groups span one row
(``input_quant_gran[0] == 1``): its scales come from its own values and its
noise draws are addressed by its global vector index
(memfast/reference.py:81-115), so the chunked product equals the one-call
product bit for bit.  Other input groupings, tuned mode, and a product that
needs the FP64 rerun (non-finite outputs, simulator.py:614-615) take the plain
path: one copy in, the device ``mm``, one copy out; so do nonideal devices, whose
per-launch conductance restore would be repeated for every chunk while their
product outlasts the copies many times over.  Finiteness of A and B is
checked on the device and read with the output check in one synchronisation
at the end; errors are the reference's (``ValueError`` for non-finite operands,
``FloatingPointError`` for a non-finite result), raised before the read event
advances.
"""

import math
import threading

import torch

from .functional import _checked
from .quantization import check_finite, input_tiles
from .simulator import Simulator, check_device_error, default_schedule, stage_device_error


_STREAMS = {}
_STREAMS_LOCK = threading.Lock()


def _helper_streams(device):
    """The pipeline's second compute stream and its copy streams, created once per
    device: the caching allocator keeps freed blocks per stream, so fresh streams on
    every call would strand memory in pools that later calls cannot reuse."""
    key = torch.device(device).index
    with _STREAMS_LOCK:
        if key not in _STREAMS:
            _STREAMS[key] = tuple(torch.cuda.Stream(device) for _ in range(3))
        return _STREAMS[key]


def _flag_nonfinite(tensor, flag, narrowed):
    """Enqueue the finiteness check of ``tensor`` into the device word ``flag`` (set to 1
    if a value is not finite, or, when ``narrowed``, not finite once narrowed to FP32)."""
    check_finite(tensor, flag, 1, 1 if narrowed else 0)


def _check_operands(a, b, simulator, out):
    if not isinstance(simulator, Simulator):
        raise TypeError("simulator must be Simulator")
    for name, value in (("A", a), ("B", b)):
        if not isinstance(value, torch.Tensor) or value.layout != torch.strided:
            raise TypeError(f"{name} must be a dense torch.Tensor")
        if not value.is_floating_point() or value.is_complex():
            raise TypeError(f"{name} must be a real floating dense tensor")
        if value.device.type != "cpu":
            raise ValueError(f"{name} must be a host (CPU) tensor")
    if a.ndim != 2 or b.ndim != 2:
        raise ValueError("mm requires two rank-two tensors")
    if a.shape[1] != b.shape[0]:
        raise ValueError("A and B have incompatible reduction dimensions")
    if a.dtype != b.dtype:
        raise ValueError("A and B must have the same dtype")
    if out is not None and (not isinstance(out, torch.Tensor) or out.device.type != "cpu"
                            or out.shape != (a.shape[0], b.shape[1]) or out.dtype != a.dtype
                            or not out.is_contiguous()):
        raise ValueError("out must be a contiguous host tensor with the result shape and dtype")
    if torch.is_grad_enabled() and (a.requires_grad or b.requires_grad):
        raise NotImplementedError(
            "memfast_b200 simulates the analog forward only; detach operands or use torch.no_grad()")


@torch.no_grad()
def host_mm(a, b, *, simulator, out=None, row_offset=0, chunk_rows=None):
    """``simulator.mm(A, B)`` for host tensors A [n, k] and B [k, o]; returns the host
    result (``out`` when given).  Pinned host memory lets the copies overlap the
    product.  ``row_offset``: global vector index of A's first row (a row shard of
    a larger batch).  ``chunk_rows``: rows per pipeline stage (default: n/8,
    at least 256, a multiple of 128)."""
    _check_operands(a, b, simulator, out)
    if type(row_offset) is not int or row_offset < 0:
        raise ValueError("row_offset must be a non-negative int")
    n, k = a.shape
    o = b.shape[1]
    device = simulator.device
    config = simulator.config
    if out is None:
        out = torch.empty((n, o), dtype=a.dtype, pin_memory=a.is_pinned())
    if n == 0 or o == 0 or k == 0:
        return _plain(a, b, simulator, out, row_offset)
    # Nonideal products restore every conductance once per launch (noise of the
    # read event), a cost that does not shrink with the rows of a chunk, and their
    # compute dwarfs the PCIe copies: they take the plain path.
    chunkable = (config.input_quant_gran[0] == 1 and simulator.mode == "default"
                 and config.nonidealities.ideal)
    if not chunkable:
        return _plain(a, b, simulator, out, row_offset)
    if chunk_rows is None:
        chunk_rows = max(256, 128 * math.ceil(n / 8 / 128))
    if type(chunk_rows) is not int or chunk_rows < 1:
        raise ValueError("chunk_rows must be a positive int")

    compute = torch.cuda.current_stream(device)
    second, copy_in, copy_out = _helper_streams(device)
    a_dev = torch.empty(a.shape, dtype=a.dtype, device=device)
    b_dev = torch.empty(b.shape, dtype=b.dtype, device=device)
    out_dev = torch.empty((n, o), dtype=a.dtype, device=device)
    ready = torch.cuda.Event()
    ready.record(compute)           # the buffers above may reuse memory freed on `compute`
    copy_in.wait_event(ready)
    copy_out.wait_event(ready)
    second.wait_event(ready)
    b_arrived = torch.cuda.Event()
    spans = [(r0, min(r0 + chunk_rows, n)) for r0 in range(0, n, chunk_rows)]
    arrived = []
    with torch.cuda.stream(copy_in):
        b_dev.copy_(b, non_blocking=True)
        b_arrived.record(copy_in)
        for r0, r1 in spans:
            a_dev[r0:r1].copy_(a[r0:r1], non_blocking=True)
            event = torch.cuda.Event()
            event.record(copy_in)
            arrived.append(event)

    compute.wait_event(b_arrived)
    # Device words: [operand not finite, product not finite, output not finite].
    flags = torch.zeros(3, dtype=torch.int32, device=device)
    _flag_nonfinite(b_dev, flags[0:1], not _checked(b, config, config.weight_bits))
    matrix = simulator._matrix_for(b, checked=True, rows=min(chunk_rows, n), program=b_dev)
    schedule = default_schedule(config)
    event_index = matrix._event
    if event_index >= 2**63:
        raise OverflowError("read-event counter exhausted")
    narrowed_a = not _checked(a, config, config.activation_bits)
    wide = torch.float64 if config.wide else torch.float32
    product = out_dev if out_dev.dtype == wide else torch.empty((n, o), dtype=wide, device=device)
    programmed = torch.cuda.Event()
    programmed.record(compute)
    second.wait_event(programmed)
    finished = []
    for index, ((r0, r1), event) in enumerate(zip(spans, arrived)):
        stream = compute if index % 2 == 0 else second
        with torch.cuda.stream(stream):
            stream.wait_event(event)
            rows = a_dev[r0:r1]
            _flag_nonfinite(rows, flags[0:1], narrowed_a)
            q, xscale = input_tiles(rows, config, matrix.input_scale, checked=True)
            matrix._launch(q, xscale, schedule, event_index, vector_offset=row_offset + r0, output=product[r0:r1])
            if product is not out_dev:
                out_dev[r0:r1].copy_(product[r0:r1])
            done = torch.cuda.Event()
            done.record(stream)
            finished.append(done)
    compute.wait_stream(second)
    with torch.cuda.stream(copy_out):
        for (r0, r1), done in zip(spans, finished):
            copy_out.wait_event(done)
            out[r0:r1].copy_(out_dev[r0:r1], non_blocking=True)
    # One synchronisation: operands finite, product finite (and finite in A's dtype).
    staged = stage_device_error(device)
    _flag_nonfinite(product, flags[1:2], False)
    if product is not out_dev:
        _flag_nonfinite(out_dev, flags[2:3], False)
    flags = flags.tolist()
    copy_out.synchronize()
    compute.wait_stream(copy_out)
    if staged[0]:
        check_device_error()
    if flags[0]:
        raise ValueError("A and B must be finite")
    if flags[1] and not config.wide:
        # The FP64 rerun of a narrow configuration: redo the whole product the plain way.
        q, xscale = input_tiles(a_dev, config, matrix.input_scale, checked=True)
        matrix._event = event_index
        result = matrix._product(q, xscale, a.shape, a.dtype, vector_offset=row_offset)
        out.copy_(result.cpu())
        return out
    if flags[1] or flags[2]:
        raise FloatingPointError("nonfinite analog output")
    matrix._event = event_index + 1
    return out


def _plain(a, b, simulator, out, row_offset):
    """Copy in, the device product (Simulator.mm semantics), copy out."""
    device = simulator.device
    a_dev = a.to(device, non_blocking=True)
    b_dev = b.to(device, non_blocking=True)
    from .functional import _operands

    _operands(a_dev, b_dev)
    config = simulator.config
    matrix = simulator._matrix_for(b, checked=_checked(b_dev, config, config.weight_bits), rows=a.shape[0],
                                   program=b_dev)
    result = matrix._forward(a_dev, checked=_checked(a_dev, config, config.activation_bits),
                             vector_offset=row_offset)
    out.copy_(result)
    return out


__all__ = ["host_mm"]
