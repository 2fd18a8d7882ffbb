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
"""

import torch
import torch.distributed as dist

from .functional import _checked, _operands
from .simulator import Simulator


def row_range(n, world, rank):
    """Rows [r0, r1) of rank ``rank``: balanced, the first n % world ranks get one more."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must lie in [0, world)")
    base, extra = divmod(n, world)
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


def sharded_mm(a_local, b, *, simulator, row_offset):
    """Rows [row_offset, row_offset + len(a_local)) of ``simulator.mm(A, B)``.

    Bit-identical to the same rows of the unsharded product (same simulator
    state): noise addresses use the global vector index.
    """
    if not isinstance(simulator, Simulator):
        raise TypeError("simulator must be Simulator")
    if a_local.ndim != 2 or b.ndim != 2 or a_local.shape[1] != b.shape[0]:
        raise ValueError("sharded_mm needs [rows, K] and [K, O] operands")
    if type(row_offset) is not int or row_offset < 0:
        raise ValueError("row_offset must be a non-negative int")
    config = simulator.config
    if config.input_quant_gran[0] not in (1,):
        raise ValueError("row sharding needs per-vector input groups (input_quant_gran[0] == 1)")
    _operands(a_local, b)
    if a_local.device != simulator.device:
        raise ValueError("operands and simulator must use the same device")
    matrix = simulator._matrix_for(b, checked=_checked(b, config, config.weight_bits), rows=a_local.shape[0])
    with torch.no_grad():
        return matrix._forward(a_local.detach(), checked=_checked(a_local, config, config.activation_bits),
                               vector_offset=row_offset)


def gather_rows(local, n, group=None):
    """All-gather row shards (``row_range`` partition of n rows) into one [n, ...] tensor.

    Shards may differ by one row; they are padded to the largest shard for the
    collective and trimmed afterwards.
    """
    world = dist.get_world_size(group)
    largest = row_range(n, world, 0)[1]
    padded = local.new_zeros((largest,) + tuple(local.shape[1:]))
    padded[: local.shape[0]] = local
    stacked = local.new_empty((world * largest,) + tuple(local.shape[1:]))
    dist.all_gather_into_tensor(stacked, padded, group=group)
    parts = []
    for rank in range(world):
        r0, r1 = row_range(n, world, rank)
        parts.append(stacked[rank * largest: rank * largest + (r1 - r0)])
    return torch.cat(parts)


__all__ = ["row_range", "sharded_mm", "gather_rows"]
