"""Tuned mode over the engine's sm_100a grid (memfast/simulator.py:27-45, 195-347):
search, persisted winners re-checked bit for bit, damaged cache files, and
nonideal devices, where only schedules of the default's kernel family can
reproduce the default's output."""

import json

import pytest
import torch

import bench

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import memfast_b200

    return memfast_b200


def operands(seed=41):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(256, 512, generator=g).cuda(), torch.randn(512, 256, generator=g).cuda()


def tuned_layer(mf, config, b, cache_dir):
    sim = mf.Simulator(config, mode="tuned", cache_dir=cache_dir)
    return sim, sim.map(b.T, name="layer")


def bits(t):
    return t.view(torch.int32)


def test_search_then_cache_hit_rechecked_without_timing(mf, tmp_path):
    from memfast_b200.tuning import resolve

    config = bench.bench_config(mf, "ideal")
    a, b = operands()
    sim, layer = tuned_layer(mf, config, b, tmp_path)
    tuned = layer(a)
    record = sim.records[-1]
    assert record["complete"] and not record["cache_hit"]
    assert len(record["candidates"]) == record["domain_count"] == 5
    accepted = [c for c in record["candidates"] if c["status"] == "accepted"]
    assert {resolve(config, c["schedule"], 256, 4, 2)[0] for c in accepted} == {"packed", "fp8_planes",
                                                                                 "generic_ideal"}
    default = mf.Simulator(config).map(b.T, name="layer")(a)
    assert torch.equal(bits(tuned), bits(default))
    files = list(tmp_path.glob("*.json"))
    assert len(files) == 1 and json.loads(files[0].read_text())["selected"] == record["selected"]
    # Another simulator (another process's view): the saved winner, re-checked, no timing.
    sim2, layer2 = tuned_layer(mf, config, b, tmp_path)
    again = layer2(a)
    hit = sim2.records[-1]
    assert hit["cache_hit"] and hit["candidates"] == [] and hit["selected"] == record["selected"]
    assert torch.equal(bits(again), bits(tuned))
    assert sim2.report()["selections"][-1] is hit


@pytest.mark.parametrize("damage", ["not json", "truncated", "other fingerprint", "schedule outside grid"])
def test_damaged_cache_file_falls_back_to_a_search(mf, tmp_path, damage):
    config = bench.bench_config(mf, "ideal")
    a, b = operands(42)
    sim, layer = tuned_layer(mf, config, b, tmp_path)
    first = layer(a)
    path = next(tmp_path.glob("*.json"))
    content = json.loads(path.read_text())
    if damage == "not json":
        path.write_text("{not json")
    elif damage == "truncated":
        path.write_text(path.read_text()[: len(path.read_text()) // 2])
    elif damage == "other fingerprint":
        content["fingerprint"]["shape"] = [1, 1]
        path.write_text(json.dumps(content))
    else:
        content["selected"] = dict(kernel=7, tile_n=32, tile_o=64, arrays=2, raster=0)
        path.write_text(json.dumps(content))
    sim2, layer2 = tuned_layer(mf, config, b, tmp_path)
    again = layer2(a)
    record = sim2.records[-1]
    assert not record["cache_hit"] and record["candidates"]
    assert torch.equal(bits(again), bits(first))
    assert json.loads(path.read_text())["complete"] is True   # rewritten


def test_nonideal_search_keeps_the_default_kernel_family(mf, tmp_path):
    """With write variation the SIMT and tensor-core currents sum in different orders:
    SIMT candidates are rejected for differing, the winner reproduces default mode."""
    from memfast_b200.tuning import resolve

    config = bench.bench_config(mf, "write")
    a, b = operands(43)
    sim, layer = tuned_layer(mf, config, b, tmp_path)
    tuned = layer(a)
    record = sim.records[-1]
    default = mf.Simulator(config).map(b.T, name="layer")(a)
    assert torch.equal(bits(tuned), bits(default))
    paths = {}
    for candidate in record["candidates"]:
        paths.setdefault(resolve(config, candidate["schedule"], 256, 4, 2)[0], []).append(candidate)
    assert all(c["status"] == "accepted" for c in paths["tc_currents"])
    assert paths["simt_currents"] and all(c["status"] == "rejected" and "differs" in c["reason"]
                                          for c in paths["simt_currents"])
    assert resolve(config, record["selected"], 256, 4, 2)[0] == "tc_currents"


def test_saved_schedule_that_changes_output_raises(mf, tmp_path):
    """A saved winner is trusted only after the bitwise re-check (the reference raises
    when it fails): a SIMT schedule planted for a nonideal layer whose default runs
    on the tensor cores."""
    config = bench.bench_config(mf, "write")
    a, b = operands(44)
    sim, layer = tuned_layer(mf, config, b, tmp_path)
    layer(a)
    simt = next(c["schedule"] for c in sim.records[-1]["candidates"] if c["schedule"]["kernel"] == 1)
    path = next(tmp_path.glob("*.json"))
    content = json.loads(path.read_text())
    content["selected"] = simt
    path.write_text(json.dumps(content))
    sim2, layer2 = tuned_layer(mf, config, b, tmp_path)
    with pytest.raises(RuntimeError, match="cached schedule changes output"):
        layer2(a)


def test_raster_orders_agree_at_scale(mf):
    """Both CTA launch orders of each tensor-core kernel give the same bits on a
    multi-wave product (1024 CTAs over 148 SMs)."""
    from memfast_b200.quantization import input_tiles
    from memfast_b200.simulator import default_schedule

    config = bench.bench_config(mf, "ideal")
    g = torch.Generator().manual_seed(45)
    a, b = torch.randn(2048, 2048, generator=g).cuda(), torch.randn(2048, 4096, generator=g).cuda()
    sim = mf.Simulator(config)
    matrix = sim._matrix_for(b)
    q, xscale = input_tiles(a, config)
    outs = [matrix._execute(q, xscale, dict(default_schedule(config), kernel=k, raster=r), 0)
            for k in (2, 3) for r in (0, 1)]
    for other in outs[1:]:
        assert torch.equal(bits(outs[0]), bits(other))
