"""Config / Nonidealities mirror the reference's validation and derived tables."""

import pytest

from memfast_b200 import Config, Nonidealities


def test_defaults_and_layouts():
    c = Config()
    assert c.array_size == (64, 64) and c.adc_bits == 6 and c.seed == 135
    assert c.nonidealities.write_variation == 0.02
    assert c.input_layout[0] == (0, 1, 1) and c.input_layout[-1] == (7, 1, -128)
    assert c.read_rows == 64 and c.reads_per_array == 1 and not c.wide


def test_multibit_slices_and_adc_order():
    c = Config(weight_slice=(1, 1, 2, 2, 2), adc_bits=(6, 7, 8, 9, 10))
    assert c.weight_layout == ((0, 3, 1), (2, 3, 4), (4, 3, 16), (6, 1, 64), (7, 1, -128))
    assert c.adc_maxima == (1023, 511, 255, 127, 63)


def test_unsigned_weights():
    c = Config(weight_signed=False, weight_slice=(2, 2, 2, 2))
    assert all(f > 0 for _, _, f in c.weight_layout)
    with pytest.raises(ValueError):
        Config(weight_signed=False, bw_e=8)


@pytest.mark.parametrize("kwargs", [
    dict(activation_bits=1), dict(input_slice=(2, 2, 2, 2)), dict(input_slice=(1, 1, 1)),
    dict(adc_bits=(6, 6)), dict(array_size=(64, 62)), dict(rows_per_read=65),
    dict(input_quant_gran=(1, 48), rows_per_read=32), dict(high_conductance=1e-8),
    dict(seed=-1), dict(weight_slice=(1, 17, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1), weight_bits=32),
])
def test_invalid_configs(kwargs):
    with pytest.raises(ValueError):
        Config(**kwargs)


def test_nonidealities_validation():
    with pytest.raises(ValueError):
        Nonidealities(read_mode="other")
    with pytest.raises(ValueError):
        Nonidealities(stuck_at_low=0.7, stuck_at_high=0.5)
    assert Nonidealities(write_variation=0).ideal
    assert not Nonidealities(write_variation=0, drift_coefficient=0.1, drift_time=5.0).ideal
    assert Nonidealities(write_variation=0, drift_coefficient=0.1, drift_time=0.0).ideal


def test_wide_and_precise():
    assert Config(activation_bits=12, input_slice=(1, 3, 4, 4)).wide
    assert Config(bw_e=8).wide
    assert Config(weight_slice=(1, 7, 1, 1, 1, 1, 1, 1, 1, 1), weight_bits=16,
                  activation_bits=16, input_slice=(1, 15)).precise_currents
