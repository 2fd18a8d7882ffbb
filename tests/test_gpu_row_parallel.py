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
