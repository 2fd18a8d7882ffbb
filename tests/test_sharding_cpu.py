"""Host-side logic of the multi-GPU path on CPU: row partition and the gather over gloo."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from memfast_b200.sharding import gather_rows, row_range


@pytest.mark.parametrize("n,world", [(0, 2), (1, 2), (5, 2), (4096, 8), (4097, 8), (7, 3), (3, 8)])
def test_row_range_partitions_every_row_once(n, world):
    spans = [row_range(n, world, rank) for rank in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0 and a0 <= a1
    sizes = [r1 - r0 for r0, r1 in spans]
    assert max(sizes) - min(sizes) <= 1


def test_row_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        row_range(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, n, mode, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        r0, r1 = row_range(n, world, rank)
        want = torch.arange(n * 3, dtype=torch.float32).reshape(n, 3)
        if mode == "in_place":
            # The strong-scaling bench: this rank's rows already sit in the full buffer.
            full = torch.full((n, 3), -1.0)
            full[r0:r1] = want[r0:r1]
            out = gather_rows(full[r0:r1], n, out=full)
            ok = out is full
        elif mode == "out":
            full = torch.full((n, 3), -1.0)
            out = gather_rows(want[r0:r1].clone(), n, out=full)
            ok = out is full
        else:
            out = gather_rows(want[r0:r1].clone(), n)
            ok = True
        result[rank] = ok and bool(torch.equal(out, want))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n,mode", [(5, "new"), (8, "new"), (1, "new"), (8, "in_place"), (4096, "in_place"),
                                    (5, "out"), (8, "out")])
def test_gather_rows_two_ranks_gloo(n, mode):
    """Uneven shards are padded for the collective and trimmed back in rank order; equal
    shards gather straight into the caller's buffer, also from rows already in it."""
    manager = mp.get_context("spawn").Manager()
    result = manager.dict()
    mp.spawn(_gather_worker, args=(2, _free_port(), n, mode, result), nprocs=2, join=True)
    assert result[0] and result[1]


@pytest.mark.parametrize("p,world", [(32, 8), (86, 8), (3, 2), (5, 5)])
def test_tile_range_partitions_every_tile_once(p, world):
    from memfast_b200.sharding import tile_range

    spans = [tile_range(p, world, rank) for rank in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == p
    assert all(a1 == b0 for (_, a1), (b0, _) in zip(spans, spans[1:]))
    assert all(t1 > t0 for t0, t1 in spans)


def _column_worker(rank, world, port, out_features, cols, result):
    from memfast_b200.sharding import ColumnShard, gather_columns, tile_range

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = torch.arange(2 * 3 * out_features, dtype=torch.float32).reshape(2, 3, out_features)
        t0, t1 = tile_range(-(-out_features // cols), world, rank)
        local = full[..., t0 * cols:min(t1 * cols, out_features)]
        gathered = gather_columns(local, out_features, cols)
        shard = ColumnShard()
        shard.device = torch.device("cpu")
        # Finiteness is agreed over the group: one rank's False makes everyone rerun.
        agreed = shard.agree(rank != 1)
        result[rank] = (bool(torch.equal(gathered, full)), agreed)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("out_features,cols", [(256, 64), (130, 64), (11008, 128)])
def test_gather_columns_and_agreement_two_ranks_gloo(out_features, cols):
    """Column slabs of a tensor-parallel layer are gathered in tile order; the FP64-rerun
    decision is the AND over ranks."""
    manager = mp.get_context("spawn").Manager()
    result = manager.dict()
    mp.spawn(_column_worker, args=(2, _free_port(), out_features, cols, result), nprocs=2, join=True)
    assert result[0] == (True, False) and result[1] == (True, False)


def _peer_worker(rank, world, port, result):
    from memfast_b200.sharding import peer_outputs

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # Host buffers over gloo cannot take peer stores: every rank must agree on that,
        # so that all of them keep the all-gather (the same collectives in the same order).
        peers = peer_outputs(torch.zeros(8, 4), None)
        result[rank] = (peers.enabled, peers.buffers)
    finally:
        dist.destroy_process_group()


def test_peer_outputs_agree_when_unavailable():
    manager = mp.Manager()
    result = manager.dict()
    mp.spawn(_peer_worker, args=(2, _free_port(), result), nprocs=2, join=True)
    assert dict(result) == {0: (False, ()), 1: (False, ())}
