"""Failure detection without a GPU fault: a bounded device-side wait that runs out.

``mf_debug_stall_next_launch`` arms a one-shot stall: the next packed tcgen05
launch stops issuing loads at a pipeline stage, so each CTA's waits on that
stage give up after a short budget (a barrier that nothing completes).  The CTA
records the wait's code in the device error word, drains its own loads and
MMAs, frees its TMEM and exits.  The host sees the code on its next
synchronisation and raises RuntimeError; the context stays usable and the next
product is bit-exact.
"""

import numpy as np
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


@pytest.mark.parametrize("stop_stage", [0, 5])
def test_expired_wait_raises_and_the_next_call_is_exact(mf, stop_stage):
    from memfast_b200 import _lib
    from memfast_b200.simulator import check_device_error
    from oracle import oracle as O

    config = bench.bench_config(mf, "ideal")
    g = torch.Generator().manual_seed(77)
    a, b = torch.randn(256, 1024, generator=g), torch.randn(1024, 256, generator=g)
    want = O.mm(a.numpy(), b.numpy(), config)
    lib = _lib.load()
    sim = mf.Simulator(config)
    a_dev, b_dev = a.cuda(), b.cuda()
    first = sim.mm(a_dev, b_dev).cpu().numpy()
    assert _lib.PATHS[lib.mf_last_path()] == "packed"
    # About 1 ms per wait at 1.9 GHz: each of the 4 CTAs gives up well within a second.
    _lib.check(lib.mf_debug_stall_next_launch(stop_stage, 2_000_000), "arm stall")
    with pytest.raises(RuntimeError, match="device-side wait"):
        sim.mm(a_dev, b_dev)
    check_device_error()   # the raise read and cleared the word
    again = sim.mm(a_dev, b_dev).cpu().numpy()
    assert _lib.PATHS[lib.mf_last_path()] == "packed"
    assert np.array_equal(first.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(again.view(np.uint32), want.view(np.uint32))


def test_stall_is_consumed_by_the_next_call_whatever_its_path(mf):
    """An armed stall never outlives the next product, even one on another kernel."""
    from memfast_b200 import _lib

    config = bench.bench_config(mf, "ideal")
    g = torch.Generator().manual_seed(78)
    a, b = torch.randn(64, 512, generator=g).cuda(), torch.randn(512, 128, generator=g).cuda()
    sim = mf.Simulator(config)
    from memfast_b200.quantization import input_tiles
    from memfast_b200.simulator import default_schedule

    matrix = sim._matrix_for(b)
    q, xscale = input_tiles(a, config)
    lib = _lib.load()
    _lib.check(lib.mf_debug_stall_next_launch(0, 2_000_000), "arm stall")
    generic = matrix._execute(q, xscale, dict(default_schedule(config), kernel=1), 0)
    assert _lib.PATHS[lib.mf_last_path()] == "generic_ideal"
    packed = matrix._execute(q, xscale, default_schedule(config), 0)
    assert _lib.PATHS[lib.mf_last_path()] == "packed"
    assert torch.equal(generic.view(torch.int32), packed.view(torch.int32))
