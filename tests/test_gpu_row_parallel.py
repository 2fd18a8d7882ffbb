"""Row-parallel product over NCCL (``sharding.row_parallel_mm``; needs two B200s).

Every rank holds one block of A's rows and the whole B; the product's rows go
straight into the full output and are all-gathered in place before the host
synchronises.  The result on every rank must equal the one-device
``Simulator.mm`` bit for bit, including the case where only one rank's rows
overflow FP32 in the scale epilogue: the one-device product then reruns every
row with the FP64 epilogue (memfast/simulator.py:614-615), so every rank must.
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def operands(case):
    rng = np.random.default_rng(23)
    a = rng.standard_normal((256, 512), dtype=np.float32)
    b = rng.standard_normal((512, 384), dtype=np.float32)
    if case == "overflow":
        # Rows of rank 1 only: T * xs overflows FP32 (xs ~ 2e36), the final value does not.
        a[200] *= np.float32(3e37)
        b *= np.float32(1e-30)
    return a, b


def _worker(rank, world, port, case, path):
    import memfast_b200 as mf
    from memfast_b200.sharding import row_parallel_mm

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        config = bench.bench_config(mf, "noisy" if case == "noisy" else "ideal")
        a, b = operands(case)
        a_dev, b_dev = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        whole = mf.Simulator(config).mm(a_dev, b_dev)
        rows = a.shape[0] // world
        sim = mf.Simulator(config)
        first = row_parallel_mm(a_dev[rank * rows:(rank + 1) * rows], b_dev, simulator=sim, row_offset=rank * rows,
                                rows=a.shape[0])
        # A second call: the cached program's next read event, on both sides.
        whole2 = None
        if case == "noisy":
            single = mf.Simulator(config)
            single.mm(a_dev, b_dev)
            whole2 = single.mm(a_dev, b_dev).cpu()
        second = row_parallel_mm(a_dev[rank * rows:(rank + 1) * rows], b_dev, simulator=sim,
                                 row_offset=rank * rows, rows=a.shape[0])
        torch.save(dict(whole=whole.cpu(), first=first.cpu(), second=second.cpu(), whole2=whole2),
                   f"{path}.{rank}")
    finally:
        dist.destroy_process_group()


def _peer_worker(rank, world, port, case, path):
    """Three calls into one output buffer registered with ``peer_outputs``: the first
    programs B (all-gather), the next ones store the rows into the other rank's
    buffer from the kernel (no all-gather unless the FP64 rerun runs).  Each call
    starts on buffers filled with NaN on both ranks."""
    import memfast_b200 as mf
    from memfast_b200.sharding import peer_outputs, row_parallel_mm

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    gathers = []
    original = dist.all_gather_into_tensor

    def counting(*args, **kwargs):
        gathers.append(1)
        return original(*args, **kwargs)

    try:
        config = bench.bench_config(mf, "noisy" if case == "noisy" else "ideal")
        a, b = operands(case)
        a_dev, b_dev = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        single = mf.Simulator(config)
        wholes = [single.mm(a_dev, b_dev).cpu() for _ in range(3)]
        rows = a.shape[0] // world
        full = torch.empty((a.shape[0], b.shape[1]), device="cuda")
        peers = peer_outputs(full)
        sim = mf.Simulator(config)
        results, counts = [], []
        dist.all_gather_into_tensor = counting
        for _ in range(3):
            full.fill_(float("nan"))
            dist.barrier()
            gathers.clear()
            row_parallel_mm(a_dev[rank * rows:(rank + 1) * rows], b_dev, simulator=sim, row_offset=rank * rows,
                            rows=a.shape[0], out=full, peers=peers)
            results.append(full.cpu())
            counts.append(len(gathers))
        dist.all_gather_into_tensor = original
        torch.save(dict(wholes=wholes, results=results, counts=counts, enabled=peers.enabled), f"{path}.{rank}")
    finally:
        dist.all_gather_into_tensor = original
        dist.destroy_process_group()


@pytest.mark.parametrize("case", ["ideal", "noisy", "overflow"])
def test_peer_stores_replace_the_gather(case, tmp_path):
    """The packed kernel's stores into the other rank's buffer give the one-device
    product bit for bit; only the first call (programming B) and the FP64 rerun of
    the overflow case gather.  The noisy configuration does not run the packed
    kernel, so it keeps the gather throughout."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    path = str(tmp_path / "peers")
    mp.spawn(_peer_worker, args=(2, _free_port(), case, path), nprocs=2, join=True)
    for rank in range(2):
        got = torch.load(f"{path}.{rank}")
        assert got["enabled"], "peer access between the two GPUs"
        for result, whole in zip(got["results"], got["wholes"]):
            assert torch.equal(result.view(torch.int32), whole.view(torch.int32)), (case, rank)
        expected = {"ideal": [1, 0, 0], "noisy": [1, 1, 1], "overflow": [2, 1, 1]}[case]
        assert got["counts"] == expected, (case, got["counts"])


@pytest.mark.parametrize("case", ["ideal", "noisy", "overflow"])
def test_row_parallel_equals_one_device_product(case, tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    path = str(tmp_path / "rp")
    mp.spawn(_worker, args=(2, _free_port(), case, path), nprocs=2, join=True)
    for rank in range(2):
        got = torch.load(f"{path}.{rank}")
        assert torch.isfinite(got["whole"]).all()
        assert torch.equal(got["first"].view(torch.int32), got["whole"].view(torch.int32)), (case, rank)
        if case == "noisy":
            assert torch.equal(got["second"].view(torch.int32), got["whole2"].view(torch.int32))
            assert not torch.equal(got["second"], got["first"])
        else:
            assert torch.equal(got["second"].view(torch.int32), got["whole"].view(torch.int32))
