"""``host_mm``: host operands in, host result out, copies overlapped (needs a B200).

The chunked pipeline must equal copying both operands in, ``Simulator.mm`` on
the device and copying the product out, bit for bit, read events included.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import memfast_b200

    return memfast_b200


INT8 = dict(array_size=(128, 128), rows_per_read=32, weight_quant_gran=(32, 1), input_quant_gran=(1, 32),
            input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=(6, 7, 7, 8, 8))
CONFIGS = {
    "ideal": dict(INT8, nonidealities=dict(write_variation=0.0)),
    "noisy": dict(INT8, nonidealities=dict(write_variation=0.02, read_variation=0.02, voltage_variation=0.02)),
    "vector_groups": dict(INT8, input_quant_gran=(None, 32), nonidealities=dict(write_variation=0.0)),
    "bfp16": dict(array_size=(256, 256), rows_per_read=64, input_quant_gran=(1, 64), weight_quant_gran=(64, 1),
                  activation_bits=16, weight_bits=16, input_slice=(1, 3, 4, 4, 4), weight_slice=(1, 3, 4, 4, 4),
                  bw_e=8, adc_bits=8, nonidealities=dict(write_variation=0.0)),
    "default": dict(),
}


def config_of(mf, name):
    kwargs = dict(CONFIGS[name])
    effects = kwargs.pop("nonidealities", {})
    return mf.Config(**kwargs, nonidealities=mf.Nonidealities(**effects))


def operands(n, k, o, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, k, generator=g).to(dtype).pin_memory(),
            torch.randn(k, o, generator=g).to(dtype).pin_memory())


@pytest.mark.parametrize("name", list(CONFIGS))
@pytest.mark.parametrize("shape", [(1000, 512, 300), (5, 200, 130), (2048, 256, 256)])
def test_host_mm_equals_device_mm(mf, name, shape):
    from memfast_b200.streaming import host_mm

    config = config_of(mf, name)
    a, b = operands(*shape, seed=sum(shape))
    device_sim, host_sim = mf.Simulator(config, device="cuda"), mf.Simulator(config, device="cuda")
    a_dev, b_dev = a.cuda(), b.cuda()
    for _ in range(2):                       # two read events of the same B
        want = device_sim.mm(a_dev, b_dev).cpu()
        got = host_mm(a, b, simulator=host_sim, chunk_rows=256)
        assert torch.equal(got, want)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float64])
def test_host_mm_dtypes(mf, dtype):
    from memfast_b200.streaming import host_mm

    config = config_of(mf, "ideal")
    a, b = operands(700, 384, 200, 7, dtype)
    want = mf.Simulator(config, device="cuda").mm(a.cuda(), b.cuda()).cpu()
    out = torch.empty(700, 200, dtype=dtype).pin_memory()
    got = host_mm(a, b, simulator=mf.Simulator(config, device="cuda"), out=out, chunk_rows=128)
    assert got is out and torch.equal(got, want)


def test_row_offset_matches_the_rows_of_a_larger_batch(mf):
    from memfast_b200.streaming import host_mm

    config = config_of(mf, "noisy")
    a, b = operands(1024, 256, 256, 8)
    full = mf.Simulator(config, device="cuda").mm(a.cuda(), b.cuda()).cpu()
    part = host_mm(a[512:].clone().pin_memory(), b, simulator=mf.Simulator(config, device="cuda"), row_offset=512)
    assert torch.equal(part, full[512:])


def test_tuned_mode_takes_the_plain_path(mf, tmp_path):
    from memfast_b200.streaming import host_mm

    config = config_of(mf, "ideal")
    a, b = operands(300, 256, 128, 9)
    want = mf.Simulator(config, device="cuda").mm(a.cuda(), b.cuda()).cpu()
    sim = mf.Simulator(config, device="cuda", mode="tuned", cache_dir=tmp_path)
    assert torch.equal(host_mm(a, b, simulator=sim), want)


def test_errors_leave_the_read_event(mf):
    from memfast_b200.streaming import host_mm

    config = config_of(mf, "noisy")
    a, b = operands(600, 256, 128, 10)
    sim = mf.Simulator(config, device="cuda")
    first = host_mm(a, b, simulator=sim)
    bad = a.clone()
    bad[550, 3] = float("nan")
    with pytest.raises(ValueError, match="finite"):
        host_mm(bad, b, simulator=sim)
    # The failed call did not consume a read event: the next call is the second read.
    reference = mf.Simulator(config, device="cuda")
    a_dev, b_dev = a.cuda(), b.cuda()
    reference.mm(a_dev, b_dev)
    second = reference.mm(a_dev, b_dev).cpu()
    assert torch.equal(host_mm(a, b, simulator=sim), second)
    assert not torch.equal(first, second)
    with pytest.raises(ValueError):
        host_mm(a.cuda(), b, simulator=sim)
    with pytest.raises(ValueError):
        host_mm(a, b[:100], simulator=sim)


def test_nonfinite_product_reruns_in_fp64(mf):
    """Huge operands overflow the FP32 epilogue; the plain path's FP64 rerun decides."""
    from memfast_b200.streaming import host_mm

    config = config_of(mf, "ideal")
    a, b = operands(300, 256, 128, 11)
    a = (a * 1e30).pin_memory()
    b = (b * 1e30).pin_memory()
    sim = mf.Simulator(config, device="cuda")
    try:
        want = mf.Simulator(config, device="cuda").mm(a.cuda(), b.cuda()).cpu()
    except FloatingPointError:
        with pytest.raises(FloatingPointError):
            host_mm(a, b, simulator=sim)
        return
    assert torch.equal(host_mm(a, b, simulator=sim), want)
