"""Programming paths and the persistent tensor-core workspace (needs a B200).

* ``mf_program_rhs`` (the right-hand matrix of ``mm`` programmed in place, with
  the K-major copy of the tensor-core kernels written in the same pass) gives the
  same buffers as ``mf_program_weights`` on the materialised transpose and as the
  CPU oracle (memfast/quantization.py:82-112).
* The one-pass FP32 row-group input quantiser gives the oracle's codes and scales
  (memfast/quantization.py:115-137).
* A matrix's workspace keeps the K-major copy between calls; reprogramming,
  checkpoint loads and device moves drop it, and every call stays bit-exact.
"""

import numpy as np
import pytest
import torch

from oracle import quantize as Q

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import memfast_b200

    return memfast_b200


CONFIGS = {
    # fused column-group pass, 32-row groups
    "int8_g32": dict(array_size=(128, 128), rows_per_read=32, weight_quant_gran=(32, 1), input_quant_gran=(1, 32),
                     input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=(6, 7, 7, 8, 8)),
    # fused column-group pass, 64-row groups
    "int8_g64": dict(array_size=(256, 256), rows_per_read=64, weight_quant_gran=(64, 1), input_quant_gran=(1, 64),
                     adc_bits=8),
    # whole-column groups: the general pass
    "int8_col": dict(array_size=(128, 128), weight_quant_gran=(None, 1), input_quant_gran=(1, None), adc_bits=8),
    # 4-bit codes, unsigned weights
    "int4_unsigned": dict(activation_bits=4, weight_bits=4, array_size=(128, 128), rows_per_read=32,
                          weight_quant_gran=(32, 1),
                          input_quant_gran=(1, 32), weight_signed=False, adc_bits=6),
    # 12-bit (wide) codes: no K-major copy
    "int12": dict(activation_bits=12, weight_bits=12, array_size=(128, 128), rows_per_read=32,
                  weight_quant_gran=(32, 1),
                  input_quant_gran=(1, 32), adc_bits=8),
    # block floating point: FP64 quantiser
    "bfp16": dict(activation_bits=16, weight_bits=16, array_size=(256, 256), rows_per_read=64,
                  weight_quant_gran=(64, 1), input_quant_gran=(1, 64), bw_e=8, adc_bits=8,
                  input_slice=(1, 3, 4, 4, 4), weight_slice=(1, 3, 4, 4, 4)),
}

SHAPES = [(256, 192), (200, 130), (96, 40), (513, 257)]


def make_config(mf, name):
    return mf.Config(**CONFIGS[name], nonidealities=mf.Nonidealities(write_variation=0.0))


def operand(shape, seed, *, nonnegative=False):
    gen = torch.Generator().manual_seed(seed)
    value = torch.randn(shape, generator=gen, dtype=torch.float64)
    if nonnegative:
        value = value.abs().round()
    return value


def kmajor_of(packed):
    """[m, p, R, C] packed codes -> the [p*C, m*R] K-major copy."""
    m, p, r, c = packed.shape
    return packed.permute(1, 3, 0, 2).reshape(p * c, m * r)


@pytest.mark.parametrize("name", list(CONFIGS))
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.float64])
def test_program_rhs_matches_program_weights_and_oracle(mf, name, shape, dtype):
    from memfast_b200.quantization import weight_tiles

    config = make_config(mf, name)
    k, o = shape
    b = operand((k, o), 7 + k + o, nonnegative=not config.weight_signed).to(dtype)
    rhs = b.cuda()
    m, p = -(-k // config.array_size[0]), -(-o // config.array_size[1])
    kmajor = None
    if not config.wide_codes:
        kmajor = torch.full((p * config.array_size[1] * m * config.array_size[0],), 0xAB, dtype=torch.uint8,
                            device="cuda")
    packed, wscale, written = weight_tiles(rhs.T, config, kmajor=kmajor)
    ref_packed, ref_wscale, ref_written = weight_tiles(rhs.T.contiguous(), config)
    torch.cuda.synchronize()
    assert written == (kmajor is not None) and not ref_written
    assert torch.equal(packed, ref_packed)
    assert torch.equal(wscale.view(torch.uint8) if wscale.dtype != torch.float64 else wscale.view(torch.int64),
                       ref_wscale.view(torch.uint8) if ref_wscale.dtype != torch.float64
                       else ref_wscale.view(torch.int64))
    if kmajor is not None:
        assert torch.equal(kmajor.view(p * config.array_size[1], m * config.array_size[0]), kmajor_of(packed))
    want_packed, want_wscale = Q.weight_tiles(b.T.numpy(), config)
    assert np.array_equal(packed.cpu().numpy().astype(np.int64), want_packed)
    assert np.array_equal(wscale.cpu().numpy(), want_wscale)


@pytest.mark.parametrize("name", ["int8_g32", "int8_g64", "int4_unsigned", "int8_col"])
@pytest.mark.parametrize("shape", [(64, 256), (5, 200), (130, 96), (1, 513)])
def test_input_quantiser_matches_oracle(mf, name, shape):
    from memfast_b200.quantization import input_tiles

    config = make_config(mf, name)
    a = operand(shape, 11 + shape[0] * 3 + shape[1]).float()
    codes, xscale = input_tiles(a.cuda(), config)
    torch.cuda.synchronize()
    want_codes, want_xscale = Q.input_tiles(a.numpy(), config)
    assert np.array_equal(codes.cpu().numpy().astype(np.int64), want_codes)
    assert np.array_equal(xscale.cpu().numpy().view(np.uint32), want_xscale.view(np.uint32))


def test_input_quantiser_on_a_row_view(mf):
    """Rows with a stride wider than K (a slice of a larger buffer) take the same codes."""
    from memfast_b200.quantization import input_tiles

    config = make_config(mf, "int8_g32")
    wide = operand((48, 320), 5).float().cuda()
    view = wide[:, 32:288]
    codes, xscale = input_tiles(view, config)
    ref_codes, ref_xscale = input_tiles(view.contiguous(), config)
    torch.cuda.synchronize()
    assert torch.equal(codes, ref_codes) and torch.equal(xscale, ref_xscale)


def generic(mf, config, a, b):
    """The same product through the generic SIMT kernel (schedule kernel 1)."""
    from memfast_b200.quantization import input_tiles

    sim = mf.Simulator(config)
    matrix = sim.map(b.T.contiguous(), name="matrix.0")
    q, xscale = input_tiles(a, config)
    out = matrix._execute(q, xscale, dict(kernel=1, tile_n=32, tile_o=64, arrays=2), 0)
    return out


def test_mm_writes_the_kmajor_copy_at_programming(mf):
    config = make_config(mf, "int8_g32")
    a = operand((512, 1024), 1).float().cuda()
    b = operand((1024, 384), 2).float().cuda()
    sim = mf.Simulator(config)
    matrix = sim._matrix_for(b, rows=512)
    assert matrix._ws is not None and matrix._ws_ready
    got = matrix._forward(a)
    want = generic(mf, config, a, b)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert torch.equal(sim.mm(a, b), want)


def test_workspace_is_reused_and_invalidated(mf):
    from memfast_b200.simulator import check_device_error

    config = make_config(mf, "int8_g32")
    a = operand((300, 512), 3).float().cuda()
    b = operand((512, 256), 4).float().cuda()
    b2 = operand((512, 256), 5).float().cuda()
    sim = mf.Simulator(config)
    matrix = sim.map(b.T.contiguous(), name="matrix.0")   # [O, K] rows: the copy is built on the first call
    assert not matrix._ws_ready
    first = matrix(a)
    assert matrix._ws_ready
    workspace = matrix._ws
    matrix.reset_read()
    assert torch.equal(matrix(a), first) and matrix._ws is workspace
    # more vectors than the workspace was sized for: a larger one keeps the copy
    big = operand((4096, 512), 6).float().cuda()
    matrix.reset_read()
    grown = matrix(big)
    assert matrix._ws is not workspace and matrix._ws_ready
    assert torch.equal(grown, generic(mf, config, big, b))
    # reprogramming drops the copy; the next call rebuilds it from the new codes
    matrix.update_weight(b2)
    assert not matrix._ws_ready
    assert torch.equal(matrix(a), generic(mf, config, a, b2))
    # a checkpoint load does too
    state = mf.Simulator(config).map(b.T.contiguous(), name="matrix.0").state_dict()
    matrix.load_state_dict(state)
    assert not matrix._ws_ready
    matrix.reset_read()
    assert torch.equal(matrix(a), first)
    # another stream gets its own workspace
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        matrix.reset_read()
        other = matrix(a)
    stream.synchronize()
    assert torch.equal(other, first)
    check_device_error()


def near_half_integers(groups, seed):
    """[groups, 32] FP32 values whose quotients by their group's scale sit on or next
    to half-integers: element 0 fixes the group maximum M = 127 s, the others are
    fl((k + 1/2) * fl(M / 127)) and their FP32 neighbours, so that rounding the
    quotient to an integer depends on its last bits (the quantisers' exact path)."""
    rng = np.random.default_rng(seed)
    s = np.float32(2.0) ** rng.integers(-12, 4, size=groups).astype(np.float32)
    s = (s * (1 + rng.random(groups, dtype=np.float32))).astype(np.float32)
    top = (np.float32(127) * s).astype(np.float32)
    scale = (top / np.float32(127)).astype(np.float32)
    k = rng.integers(-127, 127, size=(groups, 31)).astype(np.float32)
    x = ((k + np.float32(0.5)) * scale[:, None]).astype(np.float32)
    step = rng.integers(-1, 2, size=x.shape)
    x = np.where(step < 0, np.nextafter(x, np.float32(-np.inf)),
                 np.where(step > 0, np.nextafter(x, np.float32(np.inf)), x))
    x = np.clip(x, -top[:, None], top[:, None]).astype(np.float32)
    return np.concatenate([top[:, None], x], axis=1)


def test_quantisers_round_near_half_integers_like_the_oracle(mf):
    """The one-pass FP32 quantisers multiply by the reciprocal scale and divide exactly
    only near half-integers; values placed there round as the reference's division."""
    from memfast_b200.quantization import input_tiles, weight_tiles

    config = make_config(mf, "int8_g32")
    rows, k = 96, 256
    a = near_half_integers(rows * k // 32, 21).reshape(rows, k)
    codes, xscale = input_tiles(torch.from_numpy(a).cuda(), config)
    want_codes, want_xscale = Q.input_tiles(a, config)
    assert np.array_equal(codes.cpu().numpy().astype(np.int64), want_codes)
    assert np.array_equal(xscale.cpu().numpy().view(np.uint32), want_xscale.view(np.uint32))
    o = 160
    b = near_half_integers(o * k // 32, 22).reshape(o, k // 32, 32).transpose(1, 2, 0).reshape(k, o)
    b = np.ascontiguousarray(b)
    packed, wscale, _ = weight_tiles(torch.from_numpy(b).cuda().T, config)
    want_packed, want_wscale = Q.weight_tiles(b.T, config)
    assert np.array_equal(packed.cpu().numpy().astype(np.int64), want_packed)
    assert np.array_equal(wscale.cpu().numpy(), want_wscale)
