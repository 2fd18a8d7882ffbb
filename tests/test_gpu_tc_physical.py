"""Nonideal currents on the tensor cores (``csrc/tc_physical.cu``; needs a B200).

The tcgen05 path sums every slice pair's current as exact digit x FP16-part
products in FP32 (memfast/reference.py:63-117 computes them with an FP32 bmm).
It must agree with the SIMT kernel (schedule kernel 1) and the CPU oracle within
the nonideal tolerance of ``helpers.py``, and keep the exact structural
properties: column shards and row prefixes give the same values as the whole
product, bit for bit.
"""

import ctypes as ct

import numpy as np
import pytest
import torch

from helpers import MISMATCH_FRACTION, assert_close_nonideal

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import memfast_b200

    return memfast_b200


INT8 = dict(array_size=(128, 128), rows_per_read=32, weight_quant_gran=(32, 1), input_quant_gran=(1, 32),
            input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=(6, 7, 7, 8, 8))
MATRIX = dict(array_size=(256, 256), rows_per_read=64, input_quant_gran=(1, 64), weight_quant_gran=(64, 1))
ALL = dict(write_variation=0.05, adc_nonlinearity=0.02, stuck_at_low=1e-3, stuck_at_high=1e-3,
           drift_coefficient=0.05, drift_time=100.0)
CONFIGS = {
    "int8_write": dict(INT8, nonidealities=dict(write_variation=0.02)),
    "int8_read_shared": dict(INT8, nonidealities=dict(write_variation=0.02, read_variation=0.03)),
    "int8_rpr64_all": dict(MATRIX, input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=7,
                           nonidealities=ALL),
    "int4_rpr64_all": dict(MATRIX, activation_bits=4, weight_bits=4, input_slice=(1, 1, 2), weight_slice=(1, 1, 2),
                           adc_bits=6, nonidealities=ALL),
    "default_1bit": dict(nonidealities=dict(write_variation=0.02)),
    "int7_4slices": dict(INT8, activation_bits=7, weight_bits=7, input_slice=(1, 2, 2, 2), weight_slice=(1, 2, 2, 2),
                         adc_bits=8, nonidealities=dict(write_variation=0.02, drift_coefficient=0.1, drift_time=10.0)),
    "unsigned_weights": dict(INT8, weight_signed=False, nonidealities=dict(write_variation=0.02)),
    # Voltage noise: the noisy input voltages as two FP16 parts (a_operand_kernel).
    "int8_noisy": dict(INT8, nonidealities=dict(write_variation=0.02, read_variation=0.02, voltage_variation=0.02)),
    "int8_voltage_all": dict(INT8, nonidealities=dict(ALL, voltage_variation=0.05)),
    "int4_voltage": dict(INT8, activation_bits=4, weight_bits=4, input_slice=(1, 1, 2), weight_slice=(1, 1, 2),
                         adc_bits=6, nonidealities=dict(write_variation=0.02, voltage_variation=0.03)),
    # Wide configurations (16-bit BFP, BASELINE configs[2]'s third format): int64 codes,
    # 4-bit digits as FP16 tiles, int64 totals and the FP64 restore_scales epilogue.
    "bfp16_rpr64_all": dict(MATRIX, activation_bits=16, weight_bits=16, bw_e=8, input_slice=(1, 3, 4, 4, 4),
                            weight_slice=(1, 3, 4, 4, 4), adc_bits=8, nonidealities=ALL),
    "bfp16_write": dict(INT8, activation_bits=16, weight_bits=16, bw_e=8, input_slice=(1, 3, 4, 4, 4),
                        weight_slice=(1, 3, 4, 4, 4), adc_bits=8,
                        nonidealities=dict(write_variation=0.02, read_variation=0.02)),
    # Output-mode read noise: digit sums and second moments per job, a normal draw per
    # ADC event (OUTM kernels).
    "int8_read_output": dict(INT8, nonidealities=dict(write_variation=0.02, read_variation=0.05,
                                                      read_mode="output")),
    "int4_read_output_all": dict(INT8, activation_bits=4, weight_bits=4, input_slice=(1, 1, 2),
                                 weight_slice=(1, 1, 2), adc_bits=6,
                                 nonidealities=dict(ALL, read_variation=0.03, read_mode="output")),
    # Slice-pair read noise: one conductance operand per input slice (PAIRB kernels).
    "int8_read_pair": dict(INT8, nonidealities=dict(write_variation=0.02, read_variation=0.05,
                                                    read_mode="slice_pair")),
    "int4_read_pair_all": dict(INT8, activation_bits=4, weight_bits=4, input_slice=(1, 1, 2), weight_slice=(1, 1, 2),
                               adc_bits=6, nonidealities=dict(ALL, read_variation=0.03, read_mode="slice_pair")),
    "int7_read_pair": dict(INT8, activation_bits=7, weight_bits=7, input_slice=(1, 2, 2, 2), weight_slice=(1, 2, 2, 2),
                           adc_bits=8, nonidealities=dict(write_variation=0.02, read_variation=0.04,
                                                          read_mode="slice_pair")),
    "int7_read_output": dict(INT8, activation_bits=7, weight_bits=7, input_slice=(1, 2, 2, 2),
                             weight_slice=(1, 2, 2, 2), adc_bits=8,
                             nonidealities=dict(write_variation=0.02, read_variation=0.04, read_mode="output")),
}


# Ideal devices the packed and FP8 kernels do not take: the same kernel with the
# weight digits as the B operand, bit-exact.  ``saturating_adc`` (4-bit ADC, count
# limit 15 against digit dots up to 32 x 9) clamps most counts of the upper slices.
IDEAL = {
    # 1-bit slices with 7-bit ADCs: the packed kernel's 2^22 reconstruction bound
    # is exceeded, so the digit mode runs it (Config's 6-bit defaults go packed).
    "onebit_adc7": dict(adc_bits=7, nonidealities=dict(write_variation=0.0)),
    "int8_rpr64_ideal": dict(MATRIX, input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=7,
                             nonidealities=dict(write_variation=0.0)),
    "int4_rpr64_ideal": dict(MATRIX, activation_bits=4, weight_bits=4, input_slice=(1, 1, 2), weight_slice=(1, 1, 2),
                             adc_bits=6, nonidealities=dict(write_variation=0.0)),
    "int7_ideal": dict(INT8, activation_bits=7, weight_bits=7, input_slice=(1, 2, 2, 2), weight_slice=(1, 2, 2, 2),
                       adc_bits=8, nonidealities=dict(write_variation=0.0)),
    "wide_weight_digits": dict(INT8, input_slice=(1, 2, 2, 3), weight_slice=(1, 1, 2, 4), adc_bits=10,
                               nonidealities=dict(write_variation=0.0)),
    "saturating_adc": dict(INT8, adc_bits=4, nonidealities=dict(write_variation=0.0)),
    "rpr64_unsigned": dict(MATRIX, weight_signed=False, input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2),
                           adc_bits=6, nonidealities=dict(write_variation=0.0)),
}


def config_of(mf, name):
    kwargs = dict(CONFIGS[name] if name in CONFIGS else IDEAL[name])
    effects = kwargs.pop("nonidealities")
    return mf.Config(**kwargs, nonidealities=mf.Nonidealities(**effects))


def product(mf, config, a, b, kernel, *, tiles=None, offset=0, name="matrix.0"):
    from memfast_b200.quantization import input_tiles
    from memfast_b200.simulator import check_device_error

    sim = mf.Simulator(config)
    matrix = sim.map(b.T.contiguous(), name=name)
    q, xscale = input_tiles(a, config)
    out = matrix._execute(q, xscale, dict(kernel=kernel, tile_n=32, tile_o=64, arrays=2), 0,
                          vector_offset=offset, tiles=tiles)
    torch.cuda.synchronize()
    check_device_error()
    return out


def threads_of(mf, config, m, p):
    from memfast_b200 import _lib

    res = _lib.MFResources()
    sched = _lib.schedule(kernel=0)
    _lib.check(_lib.load().mf_query(_lib.native_config(config), ct.byref(sched), 256, m, p, ct.byref(res)), "q")
    return res.threads


def largest_flip(mf, config, a, b):
    """Output change of one ADC count of the most significant slice pair at the largest scales."""
    from memfast_b200.quantization import input_tiles, weight_tiles

    pair = max(abs(fa) for _, _, fa in config.input_layout) * max(abs(fw) for _, _, fw in config.weight_layout)
    xs = input_tiles(a, config)[1].max().item()
    ws = weight_tiles(b.T, config)[1].max().item()
    return pair * xs * ws


def operands(n, k, o, seed, *, nonnegative_b=False):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(n, k, generator=g)
    b = torch.randn(k, o, generator=g)
    if nonnegative_b:
        b = b.abs().round()
    return a.cuda(), b.cuda()


@pytest.mark.parametrize("name", list(CONFIGS))
def test_tensor_core_currents_match_the_oracle(mf, name):
    """Both current paths against the CPU restatement of the reference, each within the
    nonideal tolerance; against each other (two sets of ADC flips) within twice it."""
    from oracle import oracle as O

    config = config_of(mf, name)
    k = 1024 if config.array_size[0] == 256 else 768
    a, b = operands(160, k, 256, 3, nonnegative_b=not config.weight_signed)
    m = -(-k // config.array_size[0])
    p = -(-256 // config.array_size[1])
    assert threads_of(mf, config, m, p) == 640, "the tensor-core physical kernel is not selected"
    # Wide configurations reconstruct in FP64; the product is returned in the
    # operands' dtype, as Simulator.mm returns it (simulator.py:616).
    fast = product(mf, config, a, b, 0).float().cpu().numpy()
    simt = product(mf, config, a, b, 1).float().cpu().numpy()
    want = O.mm(a.cpu().numpy(), b.cpu().numpy(), config)
    assert np.isfinite(fast).all()
    flip = largest_flip(mf, config, a, b)
    assert_close_nonideal(fast, want, f"{name} tensor cores", flip=flip)
    assert_close_nonideal(simt, want, f"{name} SIMT", flip=flip)
    assert np.mean(fast != simt) <= 2 * MISMATCH_FRACTION


@pytest.mark.parametrize("name", list(IDEAL))
def test_ideal_digit_dots_are_bit_exact(mf, name):
    """Against the SIMT integer kernel (schedule kernel 1) and the CPU oracle, bit for bit."""
    from oracle import oracle as O

    config = config_of(mf, name)
    assert config.nonidealities.ideal
    k = 1024 if config.array_size[0] == 256 else 768
    a, b = operands(200, k, 384, 7, nonnegative_b=not config.weight_signed)
    m = -(-k // config.array_size[0])
    p = -(-384 // config.array_size[1])
    assert threads_of(mf, config, m, p) == 640, "the tensor-core digit kernel is not selected"
    fast = product(mf, config, a, b, 0)
    simt = product(mf, config, a, b, 1)
    assert torch.equal(fast, simt), (name, (fast != simt).float().mean().item())
    small = slice(0, 24)
    want = O.mm(a[small].cpu().numpy(), b.cpu().numpy(), config)
    got = fast[small].cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (name, np.mean(got != want))


@pytest.mark.parametrize("name", ["int8_write", "int8_rpr64_all", "default_1bit", "int8_rpr64_ideal",
                                  "int4_rpr64_ideal", "int8_noisy", "int8_read_pair", "bfp16_rpr64_all",
                                  "int8_read_output"])
def test_column_shards_and_row_prefixes_are_exact(mf, name):
    config = config_of(mf, name)
    a, b = operands(300, 512, 640, 4)
    full = product(mf, config, a, b, 0)
    p = -(-640 // config.array_size[1])
    cols = config.array_size[1]
    for t0, t1 in [(0, 1), (1, p), (p - 1, p)]:
        shard = product(mf, config, a, b, 0, tiles=(t0, t1))
        assert torch.equal(shard, full[:, t0 * cols:min(t1 * cols, 640)])
    rows = product(mf, config, a[100:], b, 0, offset=100)
    assert torch.equal(rows, full[100:])


def test_against_the_oracle(mf):
    from oracle import oracle as O

    config = config_of(mf, "int8_rpr64_all")
    a, b = operands(64, 512, 256, 5)
    got = mf.Simulator(config).mm(a, b).cpu().numpy()
    want = O.mm(a.cpu().numpy(), b.cpu().numpy(), config)
    assert_close_nonideal(got, want, "oracle")


@pytest.mark.parametrize("name", ["int8_read_shared", "int8_read_pair", "int8_read_output"])
def test_read_events_draw_new_noise(mf, name):
    config = config_of(mf, name)
    a, b = operands(128, 256, 256, 6)
    sim = mf.Simulator(config)
    first, second = sim.mm(a, b), sim.mm(a, b)
    assert not torch.equal(first, second)
    again = mf.Simulator(config)
    assert torch.equal(again.mm(a, b), first)


def test_ineligible_configs_keep_the_simt_path(mf):
    # Voltage noise runs on the tensor cores for 32-row reads only (the voltage tiles of a
    # 64-row read do not fit a pipeline stage); so does output-mode read noise, without
    # voltage noise.
    voltage64 = mf.Config(**dict(MATRIX, input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2)),
                          nonidealities=mf.Nonidealities(write_variation=0.02, voltage_variation=0.02))
    output_mode = mf.Config(**dict(MATRIX, input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2)),
                            nonidealities=mf.Nonidealities(write_variation=0.02, read_variation=0.05,
                                                           read_mode="output"))
    # Slice-pair read noise: 32-row reads without voltage noise only (every input slice's
    # conductance tiles must fit a pipeline stage).
    pair64 = mf.Config(**dict(MATRIX, input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2)),
                       nonidealities=mf.Nonidealities(write_variation=0.02, read_variation=0.02,
                                                      read_mode="slice_pair"))
    pair_voltage = mf.Config(**INT8, nonidealities=mf.Nonidealities(read_variation=0.02, voltage_variation=0.02,
                                                                    read_mode="slice_pair"))
    for config in (voltage64, output_mode, pair64, pair_voltage):
        assert threads_of(mf, config, 2, 2) == 256
    voltage = mf.Config(**INT8, nonidealities=mf.Nonidealities(write_variation=0.02, voltage_variation=0.02))
    assert threads_of(mf, voltage, 2, 2) == 640
    output32 = mf.Config(**INT8, nonidealities=mf.Nonidealities(write_variation=0.02, read_variation=0.05,
                                                                read_mode="output"))
    assert threads_of(mf, output32, 2, 2) == 640
