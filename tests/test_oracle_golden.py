"""The CPU oracle reproduces the reference's own outputs (golden vectors)."""

import numpy as np
import pytest

from helpers import assert_parity, cases_of, conv_arguments, load_case, mm_cases
from oracle import oracle as O
from oracle import quantize as Q


@pytest.mark.parametrize("case", mm_cases())
def test_oracle_mm_matches_reference(case):
    config, arrays, meta = load_case(case)
    for call in range(meta["calls"]):
        got = O.mm(arrays["A"], arrays["B"], config, event=call)
        assert_parity(got, arrays[f"out{call}"], config, f"{case} call {call}")


@pytest.mark.parametrize("case", ["config1", "int8_ideal", "int8_ideal_ragged", "int8_ideal_clip", "bfp16_matrix"])
def test_oracle_quantisation_matches_reference(case):
    config, arrays, _ = load_case(case)
    packed, wscale = Q.weight_tiles(arrays["B"].T, config)
    q, xscale = Q.input_tiles(arrays["A"], config)
    assert np.array_equal(packed, arrays["packed"].astype(np.int64))
    assert np.array_equal(wscale.view(np.uint8), arrays["weight_scale"].view(np.uint8))
    assert np.array_equal(q, arrays["q"].astype(np.int64))
    assert np.array_equal(xscale.view(np.uint8), arrays["xscale"].view(np.uint8))


@pytest.mark.parametrize("case", cases_of("conv"))
def test_oracle_conv_matches_reference(case):
    config, arrays, meta = load_case(case)
    geometry = conv_arguments(meta["conv"])
    geometry.pop("kernel")
    for call in range(meta["calls"]):
        got = O.conv2d(arrays["x"], arrays["weight"], arrays.get("bias"), config, name=meta["name"], event=call,
                       **geometry)
        assert_parity(got, arrays[f"out{call}"], config, f"{case} call {call}")

def test_ideal_integer_path_equals_physical_fp32_path():
    """In ideal mode the physical FP32 currents round to the exact integer counts."""
    config, arrays, _ = load_case("int8_ideal_clip")
    packed, _ = Q.weight_tiles(arrays["B"].T, config)
    q, _ = Q.input_tiles(arrays["A"], config)
    exact = O.partial(q, packed, config, 1, 0, 0, packed.shape[1], physical=False)
    physical = O.partial(q, packed, config, 1, 0, 0, packed.shape[1], physical=True)
    assert np.array_equal(exact, physical)


def test_clip_case_really_clips():
    config, arrays, _ = load_case("int8_ideal_clip")
    packed, _ = Q.weight_tiles(arrays["B"].T, config)
    q, _ = Q.input_tiles(arrays["A"], config)
    totals = O.partial(q, packed, config, 1, 0, 0, packed.shape[1], physical=False)
    # Without ADC clipping the total would be the plain integer product of the codes.
    x = ((q + 128) % 256 - 128).reshape(q.shape[0], -1)
    w = ((packed + 128) % 256 - 128).transpose(0, 2, 1, 3).reshape(-1, packed.shape[1] * packed.shape[3])
    linear = x[:, :32] @ w[:32]
    assert not np.array_equal(totals[:, 0].reshape(q.shape[0], -1), linear)


def test_rng_streams_pinned():
    """mix/uniform/normal restatement (random.py:8-33) against fixed values."""
    lib = O.lib()
    # uniform is ((mix(...) >> 8) + 0.5) / 2^24: strictly inside (0, 1)
    values = [lib.rng_uniform(a, 135, 10) for a in range(1000)]
    assert 0 < min(values) and max(values) < 1
    assert abs(np.mean(values) - 0.5) < 0.03
    normals = np.array([lib.rng_normal(a, 12345, 10) for a in range(20000)])
    assert abs(normals.mean()) < 0.03 and abs(normals.std() - 1) < 0.03
    assert lib.rng_event_seed(135, 0) != lib.rng_event_seed(135, 1)


def test_cascade_matches_torch_for_aligned_tiles():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(0)
    for rows in (1, 5, 16, 17, 128, 255, 256, 257, 1030):
        v = (rng.standard_normal((2, rows, 128)) * np.exp(3 * rng.standard_normal((2, rows, 128)))).astype(np.float32)
        want = torch.from_numpy(v).sum(1).numpy()
        lib = O.lib()
        import ctypes as ct
        got = np.empty((2, 128), np.float32)
        for b in range(2):
            for c in range(128):
                col = np.ascontiguousarray(v[b, :, c])
                got[b, c] = np.float32(0) + lib.orc_cascade_f32(col.ctypes.data_as(ct.POINTER(ct.c_float)), rows, 1)
        assert np.array_equal(got.view(np.int32), want.view(np.int32)), rows


@pytest.mark.parametrize("case", cases_of("headline"))
def test_oracle_headline_rows_match_reference(case):
    """The benchmark's own 4096^3 operands: the reference's first rows, reproduced by
    the oracle (bit for bit in ideal mode, within the stated tolerance otherwise)."""
    import bench

    config, arrays, meta = load_case(case)
    a, b = bench.operands(meta["size"], meta["seed"])
    rows = meta["rows"]
    assert bench.operand_digest(a[:rows], b) == meta["digest"], "regenerated operands differ from the reference's"
    got = O.mm(a[:rows], b, config, name=meta["name"])
    assert_parity(got, arrays["out0"], config, case)
