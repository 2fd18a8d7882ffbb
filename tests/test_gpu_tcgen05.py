"""The tcgen05/TMEM kernels against the generic engine and the oracle (needs a B200).

Schedule kernel 2 runs the packed-count kernel when the configuration fits its
plan (the benchmark configuration does) and the FP8 digit-plane kernel
otherwise; kernel 3 always runs the FP8 digit-plane kernel.
"""

import numpy as np
import pytest
import torch

from helpers import assert_parity

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import memfast_b200

    return memfast_b200


def int8_config(mf, adc=(6, 7, 7, 8, 8), **kw):
    base = dict(array_size=(128, 128), rows_per_read=32, weight_quant_gran=(32, 1), input_quant_gran=(1, 32),
                input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=adc,
                nonidealities=mf.Nonidealities(write_variation=0.0))
    base.update(kw)
    return mf.Config(**base)


def run(mf, config, a, b, kernel):
    """One sliced product through the engine with an explicit kernel choice."""
    from memfast_b200.quantization import input_tiles
    from memfast_b200.simulator import check_device_error

    sim = mf.Simulator(config)
    matrix = sim.map(b.T.contiguous(), name="matrix.0")
    q, xscale = input_tiles(a, config)
    out = matrix._execute(q, xscale, dict(kernel=kernel, tile_n=32, tile_o=64, arrays=2), 0)
    torch.cuda.synchronize()
    check_device_error()
    return out.cpu().numpy()


def test_fast_path_is_selected_for_the_benchmark_config(mf):
    import ctypes as ct

    from memfast_b200 import _lib

    config = int8_config(mf)
    res = _lib.MFResources()
    sched = _lib.schedule(kernel=0)
    _lib.check(_lib.load().mf_query(_lib.native_config(config), ct.byref(sched), 4096, 32, 32, ct.byref(res)), "q")
    assert res.threads > 256   # the tcgen05 kernel (the SIMT kernels run 256 threads)


@pytest.mark.parametrize("kernel", [2, 3])
@pytest.mark.parametrize("shape", [(128, 128, 128), (1, 256, 128), (200, 384, 300), (333, 1024, 520),
                                   (1024, 2048, 1024), (64, 8192, 256)])
def test_tcgen05_bit_exact_vs_generic_random(mf, shape, kernel):
    n, k, o = shape
    g = torch.Generator().manual_seed(n * 7 + k + o)
    a = torch.randn(n, k, generator=g).cuda()
    b = torch.randn(k, o, generator=g).cuda()
    config = int8_config(mf)
    fast, slow = run(mf, config, a, b, kernel), run(mf, config, a, b, 1)
    assert np.array_equal(fast.view(np.uint32), slow.view(np.uint32)), np.mean(fast != slow)


@pytest.mark.parametrize("kernel", [2, 3])
@pytest.mark.parametrize("adc", [(6, 7, 7, 8, 8), 7, (4, 5, 6, 7, 8), 8])
def test_tcgen05_bit_exact_when_adcs_clip(mf, adc, kernel):
    """Saturated inputs drive every digit to 3: every clip-capable pair clips, rare pairs included.

    Columns 0-99 are saturated and 100-255 random, so with the packed kernel the
    first 128-column tile takes the exact rerun and the second does not.
    """
    g = torch.Generator().manual_seed(11)
    a = (1.0 + 0.02 * torch.rand(256, 512, generator=g)).cuda()
    a[:, ::3] *= -1
    b = (1.0 + 0.02 * torch.rand(512, 256, generator=g)).cuda()
    b[::5] *= -1
    b[:, 100:] = torch.randn(512, 156, generator=g).cuda()
    config = int8_config(mf, adc=adc)
    fast, slow = run(mf, config, a, b, kernel), run(mf, config, a, b, 1)
    assert np.array_equal(fast.view(np.uint32), slow.view(np.uint32)), np.mean(fast != slow)


def test_tcgen05_vs_oracle_with_bias_and_unsigned_weights(mf):
    from oracle import oracle as O

    config = int8_config(mf, weight_signed=False, weight_slice=(2, 2, 2, 2), adc=(6, 7, 7, 8))
    g = torch.Generator().manual_seed(3)
    a = torch.randn(96, 384, generator=g)
    w = torch.rand(160, 384, generator=g) * 3
    bias = torch.randn(160, generator=g)
    lin = torch.nn.Linear(384, 160)
    with torch.no_grad():
        lin.weight.copy_(w)
        lin.bias.copy_(bias)
    layer = mf.AnalogLinear(lin.cuda(), mf.Simulator(config), name="unsigned")
    got = layer(a.cuda()).cpu().numpy()
    want = O.linear(a.numpy(), w.numpy(), bias.numpy(), config, name="unsigned")
    assert_parity(got, want, config, "unsigned linear")


def test_tcgen05_column_shards_match_full_output(mf):
    """Tiles [begin, end) of a sharded call equal the same columns of the full product."""
    import ctypes as ct

    from memfast_b200 import _lib
    from memfast_b200.quantization import input_tiles

    config = int8_config(mf)
    g = torch.Generator().manual_seed(5)
    a = torch.randn(256, 512, generator=g).cuda()
    b = torch.randn(512, 640, generator=g).cuda()
    sim = mf.Simulator(config)
    matrix = sim.map(b.T.contiguous(), name="matrix.0")
    q, xs = input_tiles(a, config)
    full = matrix._execute(q, xs, dict(kernel=2, tile_n=32, tile_o=64, arrays=2), 0)
    part = torch.zeros_like(full)
    ws_bytes = matrix._workspace_size(256, dict(kernel=2, tile_n=32, tile_o=64, arrays=2))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    sched = _lib.schedule(kernel=2)
    for begin, end in ((0, 2), (2, 5)):
        _lib.check(_lib.load().mf_sliced_mm(
            _lib.native_config(config), ct.byref(sched), _lib.ptr(q), _lib.ptr(xs), _lib.ptr(matrix.packed),
            _lib.ptr(matrix.weight_scale), None, _lib.ptr(part), 256, matrix.packed.shape[0], matrix.p, 640, 640,
            begin, end, matrix.seed, 0, 0, 0, _lib.ptr(ws), ws_bytes, _lib.stream_of(a.device)), "shard")
    torch.cuda.synchronize()
    assert torch.equal(full, part)


def _default_ideal(mf):
    """Config's defaults (64x64 arrays, 1-bit slices, 6-bit ADCs, whole-array
    64-row reads), ideal devices: the packed kernel with two 32-row stages per read."""
    return mf.Config(nonidealities=mf.Nonidealities(write_variation=0.0))


def test_64_row_reads_take_the_packed_kernel(mf):
    import ctypes as ct

    from memfast_b200 import _lib

    config = _default_ideal(mf)
    assert config.read_rows == 64
    res = _lib.MFResources()
    sched = _lib.schedule(kernel=0)
    _lib.check(_lib.load().mf_query(_lib.native_config(config), ct.byref(sched), 4096, 64, 64, ct.byref(res)), "q")
    assert res.threads == 768
    # And a 64-row forward really launches it: the packed kernel, its K-major weight copy
    # (first call) and the rare-tile rerun filter, which finds no flagged tile here.
    g = torch.Generator().manual_seed(64)
    a, b = torch.randn(256, 512, generator=g).cuda(), torch.randn(512, 192, generator=g).cuda()
    lib = _lib.load()
    sim = mf.Simulator(config)
    sim.mm(a, b)
    assert _lib.PATHS[lib.mf_last_path()] == "packed"
    before = lib.mf_launch_count()
    sim.mm(a, b)
    assert _lib.PATHS[lib.mf_last_path()] == "packed"
    # Second call: operand checks, programming B (with its K-major copy), quantising A,
    # the packed kernel, the rerun filter, the output check: 12 launches; a fallback of
    # the product to the generic kernel shows in mf_last_path above.
    launches = lib.mf_launch_count() - before
    assert launches <= 12, launches


@pytest.mark.parametrize("shape", [(128, 128, 128), (200, 384, 300), (333, 1000, 520)])
def test_64_row_reads_bit_exact_vs_generic_and_oracle(mf, shape):
    from oracle import oracle as O

    config = _default_ideal(mf)
    n, k, o = shape
    g = torch.Generator().manual_seed(n + k + o)
    a = torch.randn(n, k, generator=g).cuda()
    b = torch.randn(k, o, generator=g).cuda()
    fast = run(mf, config, a, b, 2)
    slow = run(mf, config, a, b, 1)
    assert np.array_equal(fast.view(np.uint32), slow.view(np.uint32))
    want = O.mm(a[:16].cpu().numpy(), b.cpu().numpy(), config)
    assert np.array_equal(fast[:16].view(np.uint32), want.view(np.uint32))


def test_64_row_reads_all_ones_reads_clip_exactly(mf):
    """Codes of -1 (all bits set) over a whole 64-row read make a 1-bit digit dot
    reach 64, one past the 6-bit ADC: the packed kernel flags those columns and the
    exact rerun gives the reference's clipped counts."""
    from oracle import oracle as O

    config = _default_ideal(mf)
    n, k, o = 96, 256, 192
    g = torch.Generator().manual_seed(5)
    a = torch.randn(n, k, generator=g)
    b = torch.randn(k, o, generator=g)
    # Column 7 of B and rows 3 and 40 of A: one value 127 times the rest, which then
    # quantise to -1 (0xFF); the whole column / row is one quantisation group.
    b[:, 7] = -1.0
    b[10, 7] = 127.0
    a[3, :] = -1.0
    a[3, 70] = 127.0
    a[40, :] = -1.0
    a[40, 5] = 127.0
    a, b = a.cuda(), b.cuda()
    fast = run(mf, config, a, b, 2)
    slow = run(mf, config, a, b, 1)
    assert np.array_equal(fast.view(np.uint32), slow.view(np.uint32))
    want = O.mm(a.cpu().numpy(), b.cpu().numpy(), config)
    assert np.array_equal(fast.view(np.uint32), want.view(np.uint32))
    # The clipped pairs change the product: a 64-row dot without the clip differs.
    unclipped = mf.Config(adc_bits=7, nonidealities=mf.Nonidealities(write_variation=0.0))
    assert not np.array_equal(run(mf, unclipped, a, b, 1)[3], fast[3])
