"""CUDA engine vs the reference's golden vectors and the CPU oracle (needs a B200)."""

import numpy as np
import pytest
import torch

from helpers import adc_events, assert_parity, flip_size, load_case, mm_cases

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import memfast_b200

    return memfast_b200


def cuda(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.mark.parametrize("case", mm_cases())
def test_mm_matches_reference_golden(mf, case):
    config, arrays, meta = load_case(case)
    sim = mf.Simulator(config, device="cuda")
    a, b = cuda(arrays["A"]), cuda(arrays["B"])
    for call in range(meta["calls"]):
        got = sim.mm(a, b).cpu().numpy()
        assert_parity(got, arrays[f"out{call}"], config, f"{case} call {call}")


@pytest.mark.parametrize("case", ["config1", "int8_ideal", "int8_ideal_ragged", "int8_ideal_clip", "bfp16_matrix"])
def test_quantisation_buffers_bit_exact(mf, case):
    from memfast_b200.quantization import input_tiles, weight_tiles

    config, arrays, _ = load_case(case)
    packed, wscale, _ = weight_tiles(cuda(arrays["B"]).T, config)
    q, xscale = input_tiles(cuda(arrays["A"]), config)
    torch.cuda.synchronize()
    assert np.array_equal(packed.cpu().numpy(), arrays["packed"])
    assert np.array_equal(wscale.cpu().numpy().view(np.uint8), arrays["weight_scale"].view(np.uint8))
    assert np.array_equal(q.cpu().numpy(), arrays["q"])
    assert np.array_equal(xscale.cpu().numpy().view(np.uint8), arrays["xscale"].view(np.uint8))


def test_map_quantized_zero_points(mf):
    config, arrays, meta = load_case("map_quantized")
    sim = mf.Simulator(config, device="cuda")
    layer = sim.map_quantized(cuda(arrays["codes"]), cuda(arrays["scales"]), zero_points=cuda(arrays["zeros"]),
                              name=meta["name"])
    got = layer(cuda(arrays["x"])).cpu().numpy()
    assert_parity(got, arrays["out0"], config, "map_quantized")


def test_fixed_input_scale(mf):
    config, arrays, meta = load_case("fixed_input_scale")
    sim = mf.Simulator(config, device="cuda")
    layer = sim.map(cuda(arrays["W"]), name=meta["name"])
    layer.set_input_scale(torch.full((1, arrays["W"].shape[1]), float(arrays["scale"]), device="cuda"))
    got = layer(cuda(arrays["x"])).cpu().numpy()
    assert_parity(got, arrays["out0"], config, "fixed_input_scale")


def test_convert_model_conv_and_linear(mf):
    config, arrays, _ = load_case("convert_model")
    net = torch.nn.Sequential(
        torch.nn.Conv2d(4, 6, 3, padding=1, stride=1, groups=2), torch.nn.ReLU(),
        torch.nn.Conv2d(6, 8, 3, padding=0, stride=2), torch.nn.Flatten(), torch.nn.Linear(8 * 3 * 3, 10),
    )
    net.load_state_dict({k[len("param::"):]: torch.from_numpy(v) for k, v in arrays.items() if k.startswith("param::")})
    analog = mf.convert_model(net, mf.Simulator(config, device="cuda"))
    x = cuda(arrays["x"])
    for call in range(2):
        got = analog(x).cpu().numpy()
        assert_parity(got, arrays[f"out{call}"], config, f"convert_model call {call}")


def _int8(mf, **effects):
    return mf.Config(array_size=(128, 128), rows_per_read=32, weight_quant_gran=(32, 1),
                     input_quant_gran=(1, 32), input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2),
                     adc_bits=(6, 7, 7, 8, 8), nonidealities=mf.Nonidealities(**effects))


@pytest.mark.parametrize("shape", [(1, 128, 128), (33, 257, 300), (256, 1024, 512), (7, 2048, 128),
                                   (8, 16384, 128), (3, 12320, 200)])
def test_ideal_int8_vs_oracle(mf, shape):
    """K = 16384 is 512 reads of 32 rows per output: PyTorch's CPU sum over reads
    (``value.sum(1)``, memfast/simulator.py:585) then cascades over more than 256
    elements, which the packed kernel declines (it keeps two 16-read levels), and
    12320 leaves a ragged last array and a ragged last cascade block."""
    from oracle import oracle as O

    n, k, o = shape
    config = _int8(mf, write_variation=0.0)
    g = torch.Generator().manual_seed(sum(shape))
    a, b = torch.randn(n, k, generator=g), torch.randn(k, o, generator=g)
    got = mf.Simulator(config).mm(a.cuda(), b.cuda()).cpu().numpy()
    assert_parity(got, O.mm(a.numpy(), b.numpy(), config), config, str(shape))


def test_nonideal_deep_cascade_vs_oracle(mf):
    """512 reads per output with write variation: the tensor-core current kernel's
    cascade above 256 reads, against the oracle within the nonideal tolerance."""
    from oracle import oracle as O

    config = _int8(mf, write_variation=0.02)
    g = torch.Generator().manual_seed(9)
    a, b = torch.randn(8, 16384, generator=g), torch.randn(16384, 128, generator=g)
    got = mf.Simulator(config).mm(a.cuda(), b.cuda()).cpu().numpy()
    tolerance = dict(flip=flip_size(config, a.numpy(), b.numpy()), events=adc_events(config, 16384))
    assert_parity(got, O.mm(a.numpy(), b.numpy(), config), config, "deep cascade", **tolerance)


def test_nonideal_all_effects_vs_oracle(mf):
    from oracle import oracle as O

    config = _int8(mf, write_variation=0.02, read_variation=0.02, voltage_variation=0.02,
                   adc_nonlinearity=0.05, stuck_at_low=1e-3, stuck_at_high=1e-3,
                   drift_coefficient=0.05, drift_time=100.0)
    g = torch.Generator().manual_seed(5)
    a, b = torch.randn(64, 512, generator=g), torch.randn(512, 384, generator=g)
    sim = mf.Simulator(config)
    a_dev, b_dev = a.cuda(), b.cuda()
    # The same RHS tensor keeps its program (name matrix.0) and advances its read event.
    # One flip of the sign x sign pair moves an output by far more than 5% of the range
    # here; the bound is four such flips (helpers.py).
    tolerance = dict(flip=flip_size(config, a.numpy(), b.numpy()), events=adc_events(config, 512))
    for event in range(2):
        got = sim.mm(a_dev, b_dev).cpu().numpy()
        assert_parity(got, O.mm(a.numpy(), b.numpy(), config, event=event), config, f"event {event}", **tolerance)
    # A new RHS tensor is a new program: next automatic name, read event 0 (simulator.py:111-171).
    got = sim.mm(a_dev, b.cuda()).cpu().numpy()
    assert_parity(got, O.mm(a.numpy(), b.numpy(), config, name="matrix.1"), config, "new rhs", **tolerance)


def test_prefix_rows_are_exact_subsets(mf):
    """Every vector is independent: a row prefix of the batch reproduces the same rows."""
    config = _int8(mf, write_variation=0.02, read_variation=0.02, voltage_variation=0.02)
    g = torch.Generator().manual_seed(9)
    a, b = torch.randn(300, 512, generator=g).cuda(), torch.randn(512, 256, generator=g).cuda()
    full = mf.Simulator(config).mm(a, b)
    prefix = mf.Simulator(config).mm(a[:37], b)
    assert torch.equal(full[:37], prefix)


def test_empty_and_vector_shapes(mf):
    config = _int8(mf, write_variation=0.0)
    sim = mf.Simulator(config)
    b = torch.randn(128, 64, device="cuda")
    assert sim.mm(torch.empty(0, 128, device="cuda"), b).shape == (0, 64)
    v = sim.matmul(torch.randn(128, device="cuda"), b)
    assert v.shape == (64,)


def test_nonfinite_inputs_rejected(mf):
    sim = mf.Simulator(_int8(mf, write_variation=0.0))
    a = torch.randn(4, 128, device="cuda")
    a[0, 0] = float("nan")
    with pytest.raises(ValueError):
        sim.mm(a, torch.randn(128, 32, device="cuda"))


@pytest.mark.parametrize("where", ["A", "B"])
def test_nonfinite_operands_raise_without_consuming_a_read_event(mf, where):
    """mm checks its operands after enqueueing the product (one synchronisation);
    the reference's errors and read-event behaviour are unchanged."""
    config, arrays, _ = load_case("shared_read_events")
    sim = mf.Simulator(config, device="cuda")
    a, b = cuda(arrays["A"]), cuda(arrays["B"])
    first = sim.mm(a, b)
    bad_a, bad_b = a.clone(), b.clone()
    (bad_a if where == "A" else bad_b)[1, 2] = float("inf")
    with pytest.raises(ValueError, match=f"{where} must be finite"):
        sim.mm(bad_a, bad_b)
    second = sim.mm(a, b).cpu().numpy()
    assert_parity(second, arrays["out1"], config, "second read after the error")
    assert not np.array_equal(first.cpu().numpy(), second)
    huge = b.double() * 1e300
    with pytest.raises(ValueError, match="finite in torch.float32"):
        sim.mm(a.double(), huge)
    # Both operands bad: A's error, as the reference checks A first.
    bad_a, bad_b = a.clone(), b.clone()
    bad_a[0, 0] = float("nan")
    bad_b[0, 0] = float("-inf")
    with pytest.raises(ValueError, match="A must be finite"):
        sim.mm(bad_a, bad_b)
