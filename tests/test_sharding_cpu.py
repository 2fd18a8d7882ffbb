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


def _gather_worker(rank, world, port, n, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        r0, r1 = row_range(n, world, rank)
        local = torch.arange(r0 * 3, r1 * 3, dtype=torch.float32).reshape(-1, 3)
        out = gather_rows(local, n)
        result[rank] = bool(torch.equal(out, torch.arange(n * 3, dtype=torch.float32).reshape(n, 3)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [5, 8, 1])
def test_gather_rows_two_ranks_gloo(n):
    """Uneven shards are padded for the collective and trimmed back in rank order."""
    manager = mp.get_context("spawn").Manager()
    result = manager.dict()
    mp.spawn(_gather_worker, args=(2, _free_port(), n, result), nprocs=2, join=True)
    assert result[0] and result[1]
