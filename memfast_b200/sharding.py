"""Batch (row) sharding of the sliced product across ranks.

Every vector of A is independent: its quantisation groups span one row
(input_quant_gran (1, n)) and its noise draws are addressed by the global
vector index (memfast/random.py:8-33, reference.py:81-115).  A rank that owns
rows [r0, r1) therefore computes exactly those rows of the single-device
result when it passes r0 as the vector offset, and the only exchange is the
final all-gather of output rows.  Column (tile) sharding is the C ABI's
``tile_begin``/``tile_end``.

Input groups that span several vectors (input_quant_gran[0] != 1) would need a
collective max over ranks; ``sharded_mm`` rejects them.

Tensor parallelism (``shard_columns`` / ``tensor_parallel``) splits a programmed
layer's output tiles over the ranks instead: every rank holds the same
programmed matrix and computes tiles ``tile_range(p, world, rank)``; cell and
noise addresses use the global tile index and the total tile count
(memfast/kernels.cu:53,118, reference.py:20-31), so each rank's columns equal
those of the single-device layer.  The column slabs are all-gathered over NCCL,
or kept sharded for a consumer that takes them.  Whether a non-finite output
triggers the FP64 rerun (simulator.py:614-615) is agreed over the group, so the
ranks rerun together exactly when the single-device layer would.
"""

import torch
import torch.distributed as dist

from . import _lib
from .functional import OPERAND_ERRORS, _native_product, _operand_code, _operand_types
from .simulator import AnalogMatrix, Simulator


def row_range(n, world, rank):
    """Rows [r0, r1) of rank ``rank``: balanced, the first n % world ranks get one more."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must lie in [0, world)")
    base, extra = divmod(n, world)
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


def sharded_mm(a_local, b, *, simulator, row_offset, out=None):
    """Rows [row_offset, row_offset + len(a_local)) of ``simulator.mm(A, B)``.

    Bit-identical to the same rows of the unsharded product (same simulator
    state): noise addresses use the global vector index.  ``out``: a [rows, O]
    buffer of A's dtype with unit column stride (for example this rank's rows of
    the full output, which ``gather_rows`` then fills in place) receiving the
    result.
    """
    _check_row_shard(a_local, b, simulator, row_offset)
    if out is not None and (out.shape != (a_local.shape[0], b.shape[1]) or out.dtype != a_local.dtype
                            or out.device != a_local.device or out.stride(-1) != 1):
        raise ValueError("out must be a [rows, O] buffer of A's dtype and device with unit column stride")
    return _row_product(a_local, b, simulator, row_offset, out)


class _NoPeerStores(Exception):
    """The product cannot store into peer buffers (it did not take the one-call path)."""


def _check_row_shard(a_local, b, simulator, row_offset):
    if not isinstance(simulator, Simulator):
        raise TypeError("simulator must be Simulator")
    _operand_types(a_local, b)
    if a_local.ndim != 2 or b.ndim != 2 or a_local.shape[1] != b.shape[0]:
        raise ValueError("sharded_mm needs [rows, K] and [K, O] operands")
    if type(row_offset) is not int or row_offset < 0:
        raise ValueError("row_offset must be a non-negative int")
    if simulator.config.input_quant_gran[0] not in (1,):
        raise ValueError("row sharding needs per-vector input groups (input_quant_gran[0] == 1)")
    if a_local.device != simulator.device:
        raise ValueError("operands and simulator must use the same device")


def _row_product(a_local, b, simulator, row_offset, out, before_sync=None, peers=()):
    """The rows' product with the operand checks read in the call's one synchronisation
    (functional.mm's deferred check: same errors, same order); after the first call
    on ``b``, one native call enqueues the whole product (``_native_product``), which
    also stores the rows into ``peers`` (other ranks' output buffers) when given."""
    native = _native_product(a_local, b, simulator, vector_offset=row_offset, out=out, before_sync=before_sync,
                             peers=peers)
    if native is not None:
        return native
    if peers:
        # The step-by-step path stores no rows into peers: its caller must gather them.
        raise _NoPeerStores
    code = _operand_code(a_local, b, simulator.config)
    matrix = simulator._matrix_for(b, checked=True, rows=a_local.shape[0])
    with torch.no_grad():
        return matrix._forward(a_local.detach(), checked=True, vector_offset=row_offset, input_flag=code,
                               input_errors=OPERAND_ERRORS, out=out, before_sync=before_sync)


class PeerOutputs:
    """Every rank's copy of one output buffer, mapped into every other rank's process
    over CUDA IPC (``mf_ipc_export`` there, ``mf_ipc_open`` on this rank's device),
    so that a row-sharded product can store its rows straight into all copies from
    the kernel's epilogue over NVLink instead of all-gathering them after it
    (``row_parallel_mm(..., peers=...)``).

    Collective: every rank of ``group`` constructs it with its own ``out`` (same
    shape and dtype, contiguous, on this node's GPUs).  ``enabled`` is False, on
    every rank alike, when the ranks are not on one node or a GPU cannot reach
    another's memory; the product then all-gathers as usual.  The buffers stay
    mapped while this object lives; every rank must keep its ``out`` alive as long."""

    def __init__(self, out, group=None):
        import ctypes as ct
        import socket

        self.out, self.group = out, group
        self._bases = []
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        usable = (out.is_cuda and out.is_contiguous() and out.numel() > 0 and 1 < world <= _lib.MAX_PEERS + 1
                  and dist.get_backend(group) == "nccl")
        shared = None
        lib = _lib.load()
        if usable:
            # The IPC handle of the allocation holding out, and out's byte offset in it.
            handle, offset = (ct.c_char * 64)(), ct.c_size_t()
            with torch.cuda.device(out.device):
                if lib.mf_ipc_export(ct.c_void_p(out.data_ptr()), handle, 64, ct.byref(offset)) == _lib.MF_OK:
                    shared = (bytes(handle), offset.value)
        infos = [None] * world
        dist.all_gather_object(infos, (socket.gethostname(), out.device.index if out.is_cuda else -1,
                                       str(out.dtype), tuple(out.shape), shared), group=group)
        addresses = []
        mine = all(info[4] is not None and info[0] == infos[0][0] and info[2:4] == infos[0][2:4] for info in infos)
        if mine:
            # Each peer's allocation is mapped into this device's address space, where
            # this device's kernels can store to it (lazy peer access).
            with torch.cuda.device(out.device):
                for q in range(world):
                    if q == rank:
                        continue
                    handle, offset = infos[q][4]
                    if lib.mf_enable_peer_access(infos[q][1]) != _lib.MF_OK:
                        mine = False
                        break
                    base = ct.c_void_p()
                    raw = (ct.c_char * len(handle)).from_buffer_copy(handle)
                    if lib.mf_ipc_open(raw, len(handle), ct.byref(base)) != _lib.MF_OK or not base.value:
                        mine = False
                        break
                    self._bases.append(base.value)
                    addresses.append(base.value + offset)
        votes = [None] * world
        dist.all_gather_object(votes, bool(mine), group=group)
        self.enabled = all(votes)
        # Other ranks' copies in rank order, as addresses in this process.
        self.buffers = tuple(addresses) if self.enabled else ()
        if self.enabled:
            self._start = torch.zeros(1, dtype=torch.int32, device=out.device)

    def __del__(self):
        lib = _lib.load()
        for base in getattr(self, "_bases", ()):
            lib.mf_ipc_close(base)

    def addresses(self, first_row):
        """Addresses of row ``first_row`` in every other rank's buffer."""
        row_bytes = self.out.stride(0) * self.out.element_size()
        return tuple(address + first_row * row_bytes for address in self.buffers)

    def enter(self):
        """Enqueue an all-reduce that completes only once every rank has entered the
        call: no rank's kernel writes into a buffer whose owner may still be using
        its previous contents."""
        dist.all_reduce(self._start, group=self.group)


def peer_outputs(out, group=None):
    """``PeerOutputs`` of ``out`` over ``group`` (collective)."""
    return PeerOutputs(out, group)


def _packed_path(simulator, n, m, p):
    """Whether products of this simulator run the packed tcgen05 kernel (the one that
    stores to peers)."""
    from . import tuning
    from .simulator import default_schedule

    return tuning.resolve(simulator.config, default_schedule(simulator.config), n, m, p)[0] == "packed"


def row_parallel_mm(a_local, b, *, simulator, row_offset, rows, out=None, group=None, peers=None):
    """The whole [rows, O] product ``A @ B`` on every rank of ``group``, each rank
    holding A's row block [row_offset, row_offset + rows / world) (equal blocks in
    rank order, as ``row_range`` gives when world divides rows).

    Each rank's rows are written straight into its rows of ``out`` (allocated when
    None).  The in-place NCCL all-gather of every rank's rows and an all-reduce of
    the ranks' check flags are enqueued on the stream right after the product,
    before the call's one host synchronisation, so the transfer follows the product
    on the device with no host round trip in between.  With ``peers`` (a
    ``PeerOutputs`` of ``out`` on this node) the packed kernel stores the rows into
    every rank's buffer itself and no all-gather runs; an all-reduce at the start of
    the call keeps any rank from writing into a buffer its owner is still using.
    Because the flags are combined, the FP64 rerun of a product with non-finite
    outputs (simulator.py:614-615) is decided for the whole product, as on one
    device: every rank reruns its rows and gathers them; operand errors are raised
    on every rank.  Bit-identical to ``simulator.mm(A, B)`` on one device.
    """
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    _check_row_shard(a_local, b, simulator, row_offset)
    share = rows // world if type(rows) is int and rows >= 0 else -1
    if share < 0 or rows % world or a_local.shape[0] != share or row_offset != rank * share:
        raise ValueError("row_parallel_mm needs equal row blocks in rank order: rows divisible by the world size")
    width = b.shape[1]
    if out is None:
        out = torch.empty((rows, width), dtype=a_local.dtype, device=a_local.device)
    elif out.shape != (rows, width) or out.dtype != a_local.dtype or out.device != a_local.device \
            or not out.is_contiguous():
        raise ValueError("out must be a contiguous [rows, O] buffer of A's dtype and device")
    own = out[row_offset: row_offset + share]
    gathered = []
    addresses = ()
    if peers is not None and peers.enabled and peers.out is out and simulator._in_place_program(b) is not None:
        m = -(-a_local.shape[1] // simulator.config.array_size[0])
        p = -(-b.shape[1] // simulator.config.array_size[1])
        if _packed_path(simulator, share, m, p):
            addresses = peers.addresses(row_offset)
            peers.enter()
    # Rows stored into the peers by this call's first product (not by an FP64 rerun).
    stored = [bool(addresses)]

    def before_sync(output, flags):
        dist.all_reduce(flags, op=dist.ReduceOp.MAX, group=group)
        direct = output.data_ptr() == own.data_ptr()
        if stored[0]:
            stored[0] = False
        elif direct:
            dist.all_gather_into_tensor(out, own, group=group)
        gathered.append(direct)

    try:
        _row_product(a_local, b, simulator, row_offset, own, before_sync, peers=addresses)
    except _NoPeerStores:
        # Nothing was enqueued: the product runs step by step and its rows are gathered.
        stored[0] = False
        _row_product(a_local, b, simulator, row_offset, own, before_sync)
    if not gathered[-1]:
        # The rows reached `out` after the synchronisation (an FP64 rerun, or a result
        # cast to A's dtype): gather them now; every rank takes this branch together.
        dist.all_gather_into_tensor(out, own, group=group)
    return out


def gather_rows(local, n, group=None, out=None):
    """All-gather row shards (``row_range`` partition of n rows) into one [n, ...] tensor.

    Shards may differ by one row; they are padded to the largest shard for the
    collective and trimmed afterwards.  ``out``: a contiguous [n, ...] result
    buffer; when the shards are equal this rank's rows may already sit in it
    (``local`` is ``out[r0:r1]``), and the collective then runs in place.
    """
    world = dist.get_world_size(group)
    largest = row_range(n, world, 0)[1]
    if out is not None and n % world == 0 and out.is_contiguous() and local.is_contiguous():
        if (out.shape != (n,) + tuple(local.shape[1:]) or out.dtype != local.dtype
                or local.shape[0] != n // world):
            raise ValueError("out must be the [n, ...] gather of the shards")
        dist.all_gather_into_tensor(out, local, group=group)
        return out
    padded = local.new_zeros((largest,) + tuple(local.shape[1:]))
    padded[: local.shape[0]] = local
    stacked = local.new_empty((world * largest,) + tuple(local.shape[1:]))
    dist.all_gather_into_tensor(stacked, padded, group=group)
    parts = []
    for rank in range(world):
        r0, r1 = row_range(n, world, rank)
        parts.append(stacked[rank * largest: rank * largest + (r1 - r0)])
    if out is not None:
        return torch.cat(parts, out=out)
    return torch.cat(parts)


def tile_range(p, world, rank):
    """Output tiles [t0, t1) of rank ``rank`` when p tiles are split over ``world`` ranks."""
    return row_range(p, world, rank)


def gather_columns(local, out_features, cols, group=None):
    """All-gather column slabs (``tile_range`` partition of the output tiles) into
    [..., out_features].  Slabs are padded to the widest for the collective."""
    world = dist.get_world_size(group)
    p = -(-out_features // cols)
    widths = []
    for rank in range(world):
        t0, t1 = tile_range(p, world, rank)
        widths.append(max(0, min(t1 * cols, out_features) - t0 * cols))
    lead = local.shape[:-1]
    flat = local.reshape(-1, local.shape[-1])
    padded = flat.new_zeros((max(widths), flat.shape[0]))
    padded[: flat.shape[1]] = flat.T
    stacked = flat.new_empty((world * max(widths), flat.shape[0]))
    dist.all_gather_into_tensor(stacked, padded, group=group)
    parts = [stacked[r * max(widths): r * max(widths) + widths[r]] for r in range(world)]
    return torch.cat(parts).T.reshape(*lead, out_features)


class ColumnShard:
    """The tensor-parallel forward of one programmed layer (see module docstring)."""

    def __init__(self, group=None, *, gather=True):
        self.group, self.gather = group, gather
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def tiles(self, layer):
        return tile_range(layer.p, self.world, self.rank)

    def agree(self, flag):
        state = torch.tensor([1 if flag else 0], dtype=torch.int32, device=self.device)
        dist.all_reduce(state, op=dist.ReduceOp.MIN, group=self.group)
        return bool(state.item())

    def __call__(self, layer, x):
        self.device = x.device if dist.get_backend(self.group) == "nccl" else torch.device("cpu")
        tiles = self.tiles(layer)
        if tiles[0] >= tiles[1]:
            raise ValueError("more ranks than output tiles")
        local = layer._forward(x, tiles=tiles, agree=self.agree)
        if not self.gather:
            return local
        return gather_columns(local, layer.out_features, layer.config.array_size[1], self.group)


def shard_columns(layer, group=None, *, gather=True):
    """Make ``layer`` (an AnalogMatrix / AnalogLinear) compute only this rank's output
    tiles, all-gathering the full output unless ``gather`` is False.  Every rank of
    ``group`` must hold the same programmed layer and call it with the same input."""
    if not isinstance(layer, AnalogMatrix):
        raise TypeError("shard_columns needs a programmed AnalogMatrix")
    layer._column_shard = ColumnShard(group, gather=gather)
    return layer


def tensor_parallel(model, group=None, *, gather=True):
    """Column-shard every AnalogLinear of a converted model over ``group`` (in place)."""
    from .nn.linear import AnalogLinear

    for module in model.modules():
        if isinstance(module, AnalogLinear):
            shard_columns(module, group, gather=gather)
    return model


__all__ = ["row_range", "sharded_mm", "row_parallel_mm", "PeerOutputs", "peer_outputs", "gather_rows", "tile_range", "gather_columns",
           "shard_columns", "tensor_parallel", "ColumnShard"]
