"""Regenerate the golden vectors in this directory from the reference MemFast.

Run in a container where the reference package is importable (it is not needed
at test time); name cases after the path to regenerate only those:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py /path/to/MemFast [case ...]

Every case stores its operands, its Config keyword arguments (JSON) and the
reference's outputs, plus the reference's quantised buffers where the case is
used to pin quantisation.  The CPU test suite checks the oracle against these
files; the GPU suite checks the CUDA engine against them and the oracle.
"""

import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path[:0] = [str(HERE.parent), str(HERE.parents[1])]
from helpers import digest, seed_operands  # noqa: E402


def _jsonable(kwargs):
    out = {}
    for key, value in kwargs.items():
        if key == "nonidealities":
            out[key] = dict(value)
        elif isinstance(value, tuple):
            out[key] = list(value)
        else:
            out[key] = value
    return out


def main(reference_root, only=()):
    sys.path.insert(0, str(reference_root))
    sys.dont_write_bytecode = True
    import memfast
    from memfast import Config, Nonidealities, Simulator

    torch.set_num_threads(8)
    base = dict(
        array_size=(128, 128), rows_per_read=32, weight_quant_gran=(32, 1),
        input_quant_gran=(1, 32), input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2),
    )
    matrix = dict(
        array_size=(256, 256), rows_per_read=64, input_quant_gran=(1, 64), weight_quant_gran=(64, 1),
    )
    effects3 = dict(write_variation=0.05, adc_nonlinearity=0.02, stuck_at_low=5e-4,
                    stuck_at_high=5e-4, drift_coefficient=0.05, drift_time=100.0)

    def make(kwargs):
        effects = kwargs.get("nonidealities", {})
        return Config(**{k: v for k, v in kwargs.items() if k != "nonidealities"},
                      nonidealities=Nonidealities(**effects))

    def save(case, kwargs, arrays, **meta):
        if only and case not in only:
            return
        payload = {k: np.asarray(v) for k, v in arrays.items()}
        payload["config_json"] = np.array(json.dumps(_jsonable(kwargs)))
        payload["meta_json"] = np.array(json.dumps(meta))
        np.savez_compressed(HERE / f"{case}.npz", **payload)
        size = (HERE / f"{case}.npz").stat().st_size
        print(f"{case:28s} {size/1024:7.1f} KiB")

    def mm_case(name, kwargs, n, k, o, seed, *, a=None, b=None, calls=1, buffers=False, seeded=False):
        """``seeded``: operands from numpy's generator (seed_operands), stored as the
        seed and a digest instead of the arrays (large reduction dimensions)."""
        if only and name not in only:
            return
        cfg = make(kwargs)
        meta = {}
        if seeded:
            a, b = (torch.from_numpy(v) for v in seed_operands(n, k, o, seed))
            meta = dict(seeded=seed, shape=[n, k, o], digest=digest(a.numpy(), b.numpy()))
        g = torch.Generator().manual_seed(seed)
        a = torch.randn(n, k, generator=g) if a is None else a
        b = torch.randn(k, o, generator=g) if b is None else b
        sim = Simulator(cfg, device="cpu")
        outs = [sim.mm(a, b) for _ in range(calls)]
        arrays = {} if seeded else {"A": a.numpy(), "B": b.numpy()}
        for i, out in enumerate(outs):
            arrays[f"out{i}"] = out.numpy()
        if buffers:
            matrix_obj = sim._matrix_for(b)
            arrays["packed"] = matrix_obj.packed.numpy()
            arrays["weight_scale"] = matrix_obj.weight_scale.numpy()
            q, xs = memfast.quantization.input_tiles(a, cfg)
            arrays["q"] = q.numpy()
            arrays["xscale"] = xs.numpy()
        save(name, kwargs, arrays, kind="mm", calls=calls, name="matrix.0", **meta)

    ideal = dict(write_variation=0.0)
    # BASELINE config #1 exactly: CPU Simulator.mm, torch.manual_seed(0), randn(4,128) @ randn(128,32).
    torch.manual_seed(0)
    a1, b1 = torch.randn(4, 128), torch.randn(128, 32)
    mm_case("config1", dict(base, adc_bits=7, nonidealities=dict(write_variation=0.02)),
            4, 128, 32, 0, a=a1, b=b1, buffers=True)
    int8 = dict(base, adc_bits=(6, 7, 7, 8, 8))
    mm_case("int8_ideal", dict(int8, nonidealities=ideal), 64, 256, 192, 1, buffers=True)
    mm_case("int8_ideal_ragged", dict(int8, nonidealities=ideal), 5, 200, 130, 2, buffers=True)
    mm_case("int8_ideal_single", dict(int8, nonidealities=ideal), 1, 384, 256, 3)
    g = torch.Generator().manual_seed(4)
    a_clip = 1.0 + 0.05 * torch.rand(16, 256, generator=g)
    b_clip = 1.0 + 0.05 * torch.rand(256, 128, generator=g)
    b_clip[:, 64:] *= -1
    mm_case("int8_ideal_clip", dict(int8, nonidealities=ideal), 16, 256, 128, 4,
            a=a_clip, b=b_clip, buffers=True)
    mm_case("int8_ideal_rpr48", dict(int8, rows_per_read=48, input_quant_gran=(1, None),
                                     weight_quant_gran=(None, 1), nonidealities=ideal),
            6, 300, 140, 5)
    mm_case("int8_nonideal", dict(int8, nonidealities=dict(write_variation=0.02, read_variation=0.02,
                                                           voltage_variation=0.02)),
            16, 256, 256, 6, calls=2)
    mm_case("int8_write_only", dict(int8, nonidealities=dict(write_variation=0.02)), 32, 256, 256, 7)
    mm_case("int4_matrix", dict(matrix, activation_bits=4, weight_bits=4, input_slice=(1, 1, 2),
                                weight_slice=(1, 1, 2), nonidealities=effects3), 8, 512, 256, 8)
    mm_case("int8_matrix", dict(matrix, input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2),
                                nonidealities=effects3), 8, 512, 256, 9)
    mm_case("bfp16_matrix", dict(matrix, activation_bits=16, weight_bits=16, input_slice=(1, 3, 4, 4, 4),
                                 weight_slice=(1, 3, 4, 4, 4), bw_e=8, adc_bits=8,
                                 nonidealities=effects3), 4, 512, 256, 10, buffers=True)
    mm_case("bfp16_ideal", dict(matrix, activation_bits=16, weight_bits=16, input_slice=(1, 3, 4, 4, 4),
                                weight_slice=(1, 3, 4, 4, 4), bw_e=8, adc_bits=8,
                                nonidealities=ideal), 4, 512, 256, 11)
    mm_case("int12_ideal", dict(base, activation_bits=12, weight_bits=12, input_slice=(1, 3, 4, 4),
                                weight_slice=(1, 3, 4, 4), adc_bits=10, nonidealities=ideal),
            4, 256, 128, 12)
    mm_case("default_config", {}, 8, 100, 70, 13)
    mm_case("default_ideal", dict(nonidealities=ideal), 8, 100, 70, 14)
    mm_case("slice_pair", dict(int8, nonidealities=dict(write_variation=0.02, read_variation=0.05,
                                                        read_mode="slice_pair")), 4, 256, 128, 15)
    mm_case("output_mode", dict(int8, nonidealities=dict(write_variation=0.02, read_variation=0.05,
                                                         read_mode="output")), 4, 256, 128, 16)
    mm_case("shared_read_events", dict(int8, nonidealities=dict(write_variation=0.0, read_variation=0.05)),
            4, 256, 128, 17, calls=3)
    # More than 256 reads per output (m * reads = 512 and 272): the cascade sum
    # over reads reaches its second level (16 blocks of 16 reads per level-2 step).
    mm_case("int8_ideal_deep", dict(int8, nonidealities=ideal), 3, 16384, 128, 40, seeded=True)
    mm_case("int8_ideal_deep_ragged", dict(int8, nonidealities=ideal), 2, 8700, 160, 41, seeded=True)
    mm_case("int8_write_deep", dict(int8, nonidealities=dict(write_variation=0.02)), 2, 16384, 128, 42, seeded=True)

    # The benchmark's own 4096 x 4096 x 4096 operands (bench.operands: seeded numpy
    # N(0,1), reproducible on any host): the first rows of A against the whole B,
    # for the ideal headline and the nonideal variants of the sweep.  Only the
    # outputs and a digest of the operands are stored; tests regenerate the
    # operands from the seed and check the digest first.
    def headline_case(name, effects, rows=8, size=4096, seed=2024):
        if only and name not in only:
            return
        from bench import EFFECTS, operand_digest, operands

        kwargs = dict(int8, nonidealities=dict(EFFECTS[effects]))
        a, b = operands(size, seed)
        out = Simulator(make(kwargs), device="cpu").mm(torch.from_numpy(a[:rows]), torch.from_numpy(b))
        save(name, kwargs, dict(out0=out.numpy()), kind="headline", name="matrix.0", size=size, seed=seed,
             rows=rows, effects=effects, digest=operand_digest(a[:rows], b))

    headline_case("headline_ideal", "ideal")
    headline_case("headline_write", "write")
    headline_case("headline_shared", "shared")
    headline_case("headline_noisy", "noisy")

    # Unsigned imported weights with zero points (simulator.py:173-185, 587-611).
    kwargs = dict(int8, weight_signed=False, nonidealities=ideal)
    cfg = make(kwargs)
    g = torch.Generator().manual_seed(18)
    codes = torch.randint(0, 256, (96, 256), generator=g)
    scales = torch.rand(96, 1, generator=g) * 0.01 + 0.001
    zeros = torch.randint(100, 156, (96, 1), generator=g).float()
    x = torch.randn(12, 256, generator=g)
    sim = Simulator(cfg, device="cpu")
    layer = sim.map_quantized(codes, scales, zero_points=zeros, name="imported")
    save("map_quantized", kwargs, dict(codes=codes.numpy(), scales=scales.numpy(), zeros=zeros.numpy(),
                                       x=x.numpy(), out0=layer(x).numpy()), kind="map_quantized",
         name="imported")

    # Fixed input scale (simulator.py:432-450).
    kwargs = dict(int8, nonidealities=ideal)
    cfg = make(kwargs)
    g = torch.Generator().manual_seed(19)
    w = torch.randn(64, 256, generator=g)
    x = torch.randn(8, 256, generator=g)
    sim = Simulator(cfg, device="cpu")
    layer = sim.map(w, name="fixed")
    layer.set_input_scale(torch.full((1, 256), 0.02))
    save("fixed_input_scale", kwargs, dict(W=w.numpy(), x=x.numpy(), scale=np.float32(0.02),
                                           out0=layer(x).numpy()), kind="fixed_scale", name="fixed")

    # Checkpoint of a programmed layer (simulator.py:452-534): the reference's buffers
    # and extra state after one read event, and the output of the next read.
    if not only or "checkpoint" in only:
        kwargs = dict(int8, adc_bits=7, nonidealities=dict(write_variation=0.02, read_variation=0.02))
        cfg = make(kwargs)
        g = torch.Generator().manual_seed(21)
        w = torch.randn(96, 256, generator=g)
        bias = torch.randn(96, generator=g)
        x = torch.randn(6, 256, generator=g)
        layer = Simulator(cfg, device="cpu").map(w, bias=bias, name="ckpt")
        out0 = layer(x)
        state = layer.state_dict()
        extra = state.pop("_extra_state")
        out1 = layer(x)
        save("checkpoint", kwargs, dict(W=w.numpy(), bias=bias.numpy(), x=x.numpy(), out0=out0.numpy(),
                                        out1=out1.numpy(),
                                        **{f"state::{k}": v.numpy() for k, v in state.items()}),
             kind="checkpoint", name="ckpt", extra_state=extra)

    # convert_model on a small Conv2d + Linear network (nn/conversion.py, nn/convolution.py).
    kwargs = dict(int8, adc_bits=7, nonidealities=dict(write_variation=0.02))
    cfg = make(kwargs)
    torch.manual_seed(20)
    net = torch.nn.Sequential(
        torch.nn.Conv2d(4, 6, 3, padding=1, stride=1, groups=2), torch.nn.ReLU(),
        torch.nn.Conv2d(6, 8, 3, padding=0, stride=2), torch.nn.Flatten(), torch.nn.Linear(8 * 3 * 3, 10),
    )
    x = torch.randn(3, 4, 8, 8)
    analog = memfast.convert_model(net, Simulator(cfg, device="cpu"))
    out0 = analog(x)
    out1 = analog(x)
    state = {k: v.numpy() for k, v in net.state_dict().items()}
    save("convert_model", kwargs, dict(x=x.numpy(), out0=out0.numpy(), out1=out1.numpy(),
                                       **{f"param::{k}": v for k, v in state.items()}),
         kind="convert_model")

    # AnalogConv2d (nn/convolution.py) on its own: geometry, groups, padding modes,
    # input groups spanning vectors, noise addressed by the patch-row index.
    def conv_case(name, kwargs, conv_kwargs, x_shape, seed, calls=2):
        if only and name not in only:
            return
        cfg = make(kwargs)
        torch.manual_seed(seed)
        source = torch.nn.Conv2d(**conv_kwargs)
        x = torch.randn(*x_shape)
        layer = memfast.nn.AnalogConv2d(source, Simulator(cfg, device="cpu"), name="conv")
        arrays = dict(x=x.numpy(), weight=source.weight.detach().numpy())
        if source.bias is not None:
            arrays["bias"] = source.bias.detach().numpy()
        for i in range(calls):
            arrays[f"out{i}"] = layer(x).numpy()
        conv = {key: list(value) if isinstance(value, tuple) else value for key, value in conv_kwargs.items()}
        save(name, kwargs, arrays, kind="conv", calls=calls, name="conv", conv=conv)

    conv_case("conv_int8", dict(int8, nonidealities=ideal),
              dict(in_channels=16, out_channels=24, kernel_size=3, stride=1, padding=1), (2, 16, 9, 11), 30)
    conv_case("conv_dilated_reflect", dict(nonidealities=dict(write_variation=0.02, read_variation=0.02,
                                                              voltage_variation=0.02)),
              dict(in_channels=8, out_channels=12, kernel_size=(3, 5), stride=(2, 1), padding=(2, 1),
                   dilation=(2, 1), groups=2, padding_mode="reflect"), (2, 8, 10, 9), 31)
    conv_case("conv_row_groups", dict(int8, input_quant_gran=(4, 32), nonidealities=dict(write_variation=0.02)),
              dict(in_channels=12, out_channels=8, kernel_size=3, stride=2, bias=False), (3, 12, 9, 9), 32)
    conv_case("conv_depthwise_circular", dict(matrix, activation_bits=4, weight_bits=4, input_slice=(1, 1, 2),
                                              weight_slice=(1, 1, 2), nonidealities=effects3),
              dict(in_channels=6, out_channels=6, kernel_size=3, padding=1, groups=6, padding_mode="circular"),
              (2, 6, 7, 7), 33)
    conv_case("conv_pointwise_strided", dict(base, adc_bits=7, input_quant_gran=(1, None),
                                             weight_quant_gran=(None, 1), nonidealities=dict(write_variation=0.02,
                                                                                             read_variation=0.05,
                                                                                             read_mode="output")),
              dict(in_channels=40, out_channels=20, kernel_size=1, stride=3), (2, 40, 8, 10), 34)


if __name__ == "__main__":
    main(Path(sys.argv[1] if len(sys.argv) > 1 else "../MemFast").resolve(), tuple(sys.argv[2:]))
