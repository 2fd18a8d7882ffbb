"""Checkpoint compatibility with the reference (simulator.py:452-534; needs a GPU).

The golden case holds a reference layer's state dict (buffers and extra state)
after one read event and the reference's outputs of reads 0 and 1.
"""

import numpy as np
import pytest
import torch

from helpers import assert_parity, load_case

pytestmark = pytest.mark.gpu

TUPLE_FIELDS = ("array_size", "weight_quant_gran", "input_quant_gran", "input_slice", "weight_slice", "adc_bits")


@pytest.fixture(scope="module")
def mf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import memfast_b200

    return memfast_b200


def _reference_state(arrays, meta):
    """The reference state dict (JSON turned the config's tuples into lists)."""
    extra = dict(meta["extra_state"])
    config = dict(extra["config"])
    for key in TUPLE_FIELDS:
        if isinstance(config.get(key), list):
            config[key] = tuple(config[key])
    extra["config"] = config
    state = {key.split("::", 1)[1]: torch.from_numpy(arrays[key]) for key in arrays if key.startswith("state::")}
    state["_extra_state"] = extra
    return state


def test_programming_matches_reference_checkpoint(mf):
    """Mapping the same weights gives the reference's buffers and extra state."""
    config, arrays, meta = load_case("checkpoint")
    layer = mf.Simulator(config).map(torch.from_numpy(arrays["W"]).cuda(),
                                     bias=torch.from_numpy(arrays["bias"]).cuda(), name=meta["name"])
    reference = _reference_state(arrays, meta)
    ours = layer.state_dict()
    assert set(ours) == set(reference)
    for key in ("packed", "weight_scale", "bias"):
        assert ours[key].dtype == reference[key].dtype and ours[key].shape == reference[key].shape, key
        assert torch.equal(ours[key].cpu(), reference[key]), key
    extra = ours["_extra_state"]
    for key in ("config", "in_features", "out_features", "name", "seed"):
        assert extra[key] == reference["_extra_state"][key], key
    assert_parity(layer(torch.from_numpy(arrays["x"]).cuda()).cpu().numpy(), arrays["out0"], config, "read 0")


def test_reference_checkpoint_loads_and_continues(mf):
    """A layer loaded from the reference's checkpoint resumes at the saved read event."""
    config, arrays, meta = load_case("checkpoint")
    layer = mf.Simulator(config).map(torch.ones(96, 256, device="cuda"), bias=torch.zeros(96, device="cuda"),
                                     name="other")
    layer.load_state_dict(_reference_state(arrays, meta))
    assert layer.name == "ckpt" and layer._event == 1 and layer.seed == meta["extra_state"]["seed"]
    got = layer(torch.from_numpy(arrays["x"]).cuda()).cpu().numpy()
    assert_parity(got, arrays["out1"], config, "read 1 after loading")
    assert layer._event == 2


def test_checkpoint_rejects_other_physics(mf):
    config, arrays, meta = load_case("checkpoint")
    state = _reference_state(arrays, meta)
    state["_extra_state"]["config"] = dict(state["_extra_state"]["config"], adc_bits=6)
    layer = mf.Simulator(config).map(torch.ones(96, 256, device="cuda"), bias=torch.zeros(96, device="cuda"),
                                     name="other")
    with pytest.raises(ValueError):
        layer.load_state_dict(state)
