"""Tensor-parallel (column-sharded) AnalogLinear (needs a B200; the NCCL case needs two).

Every rank holds the same programmed layer and computes output tiles
``tile_range(p, world, rank)``; cell and noise addresses use the global tile
index (memfast/kernels.cu:53,118), so the shards put together equal the
single-device layer bit for bit, noisy configurations included.
"""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import memfast_b200

    return memfast_b200


INT8 = dict(array_size=(128, 128), rows_per_read=32, weight_quant_gran=(32, 1), input_quant_gran=(1, 32),
            input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=(6, 7, 7, 8, 8))
EFFECTS = {
    "ideal": dict(write_variation=0.0),
    "write": dict(write_variation=0.02),
    "read_shared": dict(write_variation=0.02, read_variation=0.02, voltage_variation=0.02),
    "output_mode": dict(write_variation=0.02, read_variation=0.05, read_mode="output"),
}


def make_layer(mf, effects, out_features=700, in_features=384, seed=3, bias=True):
    torch.manual_seed(seed)
    source = torch.nn.Linear(in_features, out_features, bias=bias)
    config = mf.Config(**INT8, nonidealities=mf.Nonidealities(**EFFECTS[effects]))
    return mf.nn.AnalogLinear(source, mf.Simulator(config, device="cuda"), name="proj")


@pytest.mark.parametrize("effects", list(EFFECTS))
@pytest.mark.parametrize("world", [2, 3, 6])
def test_column_shards_reassemble_the_layer(mf, effects, world):
    from memfast_b200.sharding import tile_range

    layer = make_layer(mf, effects)
    x = torch.randn(5, 7, 384, device="cuda")
    want = [layer(x), layer(x)]           # two read events
    for event in range(2):
        parts = []
        for rank in range(world):
            layer.reset_read(event)
            parts.append(layer._forward(x, tiles=tile_range(layer.p, world, rank)))
        assert torch.equal(torch.cat(parts, dim=-1), want[event])


def test_shard_of_an_imported_layer_with_zero_points(mf):
    from memfast_b200.sharding import tile_range

    config = mf.Config(**INT8, weight_signed=False, nonidealities=mf.Nonidealities(write_variation=0.0))
    sim = mf.Simulator(config, device="cuda")
    g = torch.Generator().manual_seed(5)
    codes = torch.randint(0, 256, (300, 256), generator=g)
    scales = torch.rand(300, 1, generator=g) * 0.01 + 0.001
    zeros = torch.randint(100, 156, (300, 1), generator=g).float()
    layer = sim.map_quantized(codes, scales, zero_points=zeros, bias=torch.randn(300), name="imported")
    x = torch.randn(9, 256, device="cuda")
    want = layer(x)
    parts = [layer._forward(x, tiles=tile_range(layer.p, 2, r)) for r in range(2)]
    assert torch.equal(torch.cat(parts, dim=-1), want)


def test_agreed_rerun_matches_the_fp64_path(mf):
    """A shard told that another shard was non-finite reruns with the FP64 epilogue,
    exactly as the whole layer would."""
    from memfast_b200.quantization import input_tiles
    from memfast_b200.simulator import default_schedule

    layer = make_layer(mf, "ideal")
    x = torch.randn(4, 384, device="cuda")
    q, xscale = input_tiles(x, layer.config)
    tiles = (1, 4)
    forced = layer._execute(q, xscale, default_schedule(layer.config), 0, tiles=tiles, agree=lambda ok: False)
    stable = layer._execute(q, xscale, default_schedule(layer.config), 0, stable=True)
    assert forced.dtype == torch.float64
    assert torch.equal(forced, stable[:, 128:512])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, effects, path):
    import memfast_b200 as mf
    from memfast_b200.sharding import tensor_parallel

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        model = torch.nn.Sequential(make_layer(mf, effects, seed=11), torch.nn.ReLU(),
                                    make_layer(mf, effects, out_features=260, in_features=700, seed=12))
        torch.manual_seed(0)
        x = torch.randn(6, 384).cuda()
        full = model(x)
        for layer in (model[0], model[2]):
            layer.reset_read()
        tensor_parallel(model)
        sharded = model(x)
        torch.save(dict(full=full.cpu(), sharded=sharded.cpu()), f"{path}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("effects", ["ideal", "read_shared"])
def test_tensor_parallel_two_gpus_nccl(mf, tmp_path, effects):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    path = str(tmp_path / "tp")
    mp.spawn(_nccl_worker, args=(2, _free_port(), effects, path), nprocs=2, join=True)
    for rank in range(2):
        got = torch.load(f"{path}.{rank}")
        assert torch.equal(got["sharded"], got["full"])
