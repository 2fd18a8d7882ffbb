"""AnalogConv2d as an implicit GEMM (needs a B200).

The patches are quantised straight from the NCHW input (``mf_quantize_conv_input``)
instead of through ``F.unfold`` (memfast/nn/convolution.py:49-55).  Checked
against the reference's own outputs (golden cases), against the unfolded path
through the same programmed matrices (bit-identical codes and outputs over
geometry, padding modes, groups, dtypes, layouts and quantisation groups), and
for the reference's non-finite behaviour.
"""

import numpy as np
import pytest
import torch
from torch.nn import functional as F

from helpers import assert_parity, cases_of, load_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import memfast_b200

    return memfast_b200


@pytest.mark.parametrize("case", cases_of("conv"))
def test_conv_matches_reference_golden(mf, case):
    config, arrays, meta = load_case(case)
    source = torch.nn.Conv2d(**meta["conv"])
    with torch.no_grad():
        source.weight.copy_(torch.from_numpy(arrays["weight"]))
        if source.bias is not None:
            source.bias.copy_(torch.from_numpy(arrays["bias"]))
    layer = mf.nn.AnalogConv2d(source, mf.Simulator(config, device="cuda"), name=meta["name"])
    x = torch.from_numpy(arrays["x"]).cuda()
    for call in range(meta["calls"]):
        got = layer(x).cpu().numpy()
        assert_parity(got, arrays[f"out{call}"], config, f"{case} call {call}")


def unfolded(layer, x):
    """The unfolded reference lowering through the layer's own programmed matrices."""
    if layer.padding_mode != "zeros":
        ph, pw = layer.padding
        x = F.pad(x, (pw, pw, ph, ph), mode=layer.padding_mode)
        padding = (0, 0)
    else:
        padding = layer.padding
    patches = F.unfold(x, layer.kernel_size, layer.dilation, padding, layer.stride)
    size = patches.shape[1] // layer.groups
    parts = [matrix(patches[:, g * size:(g + 1) * size].transpose(1, 2)) for g, matrix in enumerate(layer.matrices)]
    out = torch.cat(parts, dim=-1).transpose(1, 2)
    return out


def layer_pair(mf, config, conv_kwargs, seed):
    torch.manual_seed(seed)
    source = torch.nn.Conv2d(**conv_kwargs)
    return source, mf.nn.AnalogConv2d(source, mf.Simulator(config, device="cuda"), name="conv")


def compare(layer, x):
    got = layer(x)
    for matrix in layer.matrices:
        matrix.reset_read()
    want = unfolded(layer, x)
    torch.cuda.synchronize()
    assert torch.equal(got.reshape(want.shape), want)
    assert got.shape == (x.shape[0], layer.out_channels, *got.shape[2:])


INT8 = dict(array_size=(128, 128), rows_per_read=32, weight_quant_gran=(32, 1), input_quant_gran=(1, 32),
            input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=(6, 7, 7, 8, 8))

GEOMETRIES = [
    dict(in_channels=16, out_channels=32, kernel_size=3, padding=1),
    dict(in_channels=8, out_channels=16, kernel_size=(3, 5), stride=(2, 1), padding=(2, 1), dilation=(2, 1)),
    dict(in_channels=12, out_channels=12, kernel_size=3, padding=1, groups=3, padding_mode="reflect"),
    dict(in_channels=6, out_channels=6, kernel_size=3, padding=2, groups=6, padding_mode="circular"),
    dict(in_channels=10, out_channels=8, kernel_size=3, stride=2, padding=1, padding_mode="replicate"),
    dict(in_channels=64, out_channels=48, kernel_size=1, stride=2, bias=False),
    dict(in_channels=3, out_channels=16, kernel_size=7, stride=2, padding=3),
]


@pytest.mark.parametrize("geometry", range(len(GEOMETRIES)))
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.float64])
def test_implicit_equals_unfolded(mf, geometry, dtype):
    config = mf.Config(**INT8, nonidealities=mf.Nonidealities(write_variation=0.0))
    source, layer = layer_pair(mf, config, GEOMETRIES[geometry], 40 + geometry)
    x = torch.randn(2, source.in_channels, 13, 11).to(dtype).cuda()
    compare(layer, x)


CONFIGS = {
    "default": dict(),
    "row_groups": dict(INT8, input_quant_gran=(4, 32)),
    "tensor_groups": dict(INT8, input_quant_gran=(None, 32)),
    "whole_vector": dict(INT8, input_quant_gran=(1, None), weight_quant_gran=(None, 1)),
    "int12": dict(INT8, activation_bits=12, weight_bits=12, input_slice=(1, 3, 4, 4), weight_slice=(1, 3, 4, 4),
                  adc_bits=10),
    "bfp16": dict(array_size=(256, 256), rows_per_read=64, input_quant_gran=(1, 64), weight_quant_gran=(64, 1),
                  activation_bits=16, weight_bits=16, input_slice=(1, 3, 4, 4, 4), weight_slice=(1, 3, 4, 4, 4),
                  bw_e=8, adc_bits=8),
    "noisy": dict(INT8, nonidealities=dict(write_variation=0.02, read_variation=0.02, voltage_variation=0.02)),
}


@pytest.mark.parametrize("name", list(CONFIGS))
def test_implicit_equals_unfolded_across_configs(mf, name):
    kwargs = dict(CONFIGS[name])
    effects = kwargs.pop("nonidealities", dict(write_variation=0.0))
    config = mf.Config(**kwargs, nonidealities=mf.Nonidealities(**effects))
    source, layer = layer_pair(mf, config, dict(in_channels=24, out_channels=40, kernel_size=3, padding=1,
                                                stride=(1, 2), groups=2), 50)
    x = torch.randn(3, 24, 10, 17).cuda()
    compare(layer, x)


def test_channels_last_and_sliced_inputs(mf):
    config = mf.Config(**INT8, nonidealities=mf.Nonidealities(write_variation=0.0))
    source, layer = layer_pair(mf, config, dict(in_channels=16, out_channels=24, kernel_size=3, padding=1), 60)
    x = torch.randn(4, 16, 12, 12).cuda()
    want = layer(x)
    for matrix in layer.matrices:
        matrix.reset_read()
    assert torch.equal(layer(x.to(memory_format=torch.channels_last)), want)
    for matrix in layer.matrices:
        matrix.reset_read()
    wide = torch.randn(4, 20, 12, 15).cuda()
    wide[:, 2:18, :, 1:13] = x
    assert torch.equal(layer(wide[:, 2:18, :, 1:13]), want)


def test_fixed_input_scale(mf):
    config = mf.Config(**INT8, nonidealities=mf.Nonidealities(write_variation=0.0))
    source, layer = layer_pair(mf, config, dict(in_channels=8, out_channels=16, kernel_size=3, padding=1), 70)
    for matrix in layer.matrices:
        matrix.set_input_scale(torch.full((1, 72), 0.03))
    compare(layer, torch.randn(2, 8, 9, 9).cuda())


def test_events_advance_once_per_forward(mf):
    config = mf.Config(**INT8, nonidealities=mf.Nonidealities(write_variation=0.02, read_variation=0.05))
    source, layer = layer_pair(mf, config, dict(in_channels=8, out_channels=8, kernel_size=3, groups=2), 80)
    x = torch.randn(2, 8, 7, 7).cuda()
    first, second = layer(x), layer(x)
    assert [matrix._event for matrix in layer.matrices] == [2, 2]
    assert not torch.equal(first, second)   # read noise is drawn per event
    for matrix in layer.matrices:
        matrix.reset_read(1)
    assert torch.equal(layer(x), second)


def test_nonfinite_inputs(mf):
    config = mf.Config(**INT8, nonidealities=mf.Nonidealities(write_variation=0.0))
    source, layer = layer_pair(mf, config, dict(in_channels=4, out_channels=8, kernel_size=1, stride=3), 90)
    x = torch.randn(1, 4, 7, 7).cuda()
    baseline = layer(x)
    # A value no window reads (row 1 with stride 3) is not quantised: no error, as with unfold.
    x_unread = x.clone()
    x_unread[0, 2, 1, 1] = float("nan")
    for matrix in layer.matrices:
        matrix.reset_read()
    assert torch.equal(layer(x_unread), baseline)
    x_read = x.clone()
    x_read[0, 1, 3, 3] = float("inf")
    events = [matrix._event for matrix in layer.matrices]
    with pytest.raises(ValueError, match="finite"):
        layer(x_read)
    assert [matrix._event for matrix in layer.matrices] == events
    # FP64 values beyond FP32 range are not finite in the FP32 quantiser.
    big = x.double()
    big[0, 0, 0, 0] = 1e300
    with pytest.raises(ValueError, match="finite"):
        layer(big)


def test_empty_batch_and_bad_geometry(mf):
    config = mf.Config(**INT8, nonidealities=mf.Nonidealities(write_variation=0.0))
    source, layer = layer_pair(mf, config, dict(in_channels=4, out_channels=8, kernel_size=5), 95)
    assert layer(torch.randn(0, 4, 9, 9).cuda()).shape == (0, 8, 5, 5)
    with pytest.raises(RuntimeError):
        layer(torch.randn(1, 4, 3, 3).cuda())
    with pytest.raises(ValueError):
        layer(torch.randn(1, 3, 9, 9).cuda())


def test_tuned_mode_conv(mf, tmp_path):
    config = mf.Config(**INT8, nonidealities=mf.Nonidealities(write_variation=0.0))
    torch.manual_seed(96)
    source = torch.nn.Conv2d(16, 16, 3, padding=1)
    sim = mf.Simulator(config, device="cuda", mode="tuned", cache_dir=tmp_path)
    layer = mf.nn.AnalogConv2d(source, sim, name="conv")
    x = torch.randn(2, 16, 8, 8).cuda()
    tuned = layer(x)
    for matrix in layer.matrices:
        matrix.reset_read()
    assert torch.equal(tuned, unfolded(layer, x).reshape(tuned.shape))
    assert sim.records and sim.records[-1]["shape"] == [2, 64, 144]


def test_resnet_block_shapes_match_oracle(mf):
    """A ResNet-50 bottleneck's 3x3 stage at a reduced batch against the CPU oracle."""
    from helpers import conv_arguments
    from oracle import oracle as O

    config = mf.Config(nonidealities=mf.Nonidealities(write_variation=0.0))
    torch.manual_seed(97)
    source = torch.nn.Conv2d(64, 64, 3, padding=1, bias=False)
    layer = mf.nn.AnalogConv2d(source, mf.Simulator(config, device="cuda"), name="conv")
    x = torch.randn(2, 64, 14, 14)
    got = layer(x.cuda()).cpu().numpy()
    geometry = conv_arguments(dict(kernel_size=3, padding=1))
    geometry.pop("kernel")
    want = O.conv2d(x.numpy(), source.weight.detach().numpy(), None, config, name="conv", **geometry)
    assert_parity(got, want, config, "resnet 3x3")
    assert np.isfinite(got).all()
