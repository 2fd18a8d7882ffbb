"""The C ABI library loads, exports every declared symbol, and validates on the host."""

import ctypes as ct
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "memfast_b200.h").read_text()
    return sorted(set(re.findall(r"\b(mf_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    from memfast_b200 import _lib

    handle = ct.CDLL(str(_lib.LIBRARY))
    for name in declared_symbols():
        assert hasattr(handle, name), name
    assert set(declared_symbols()) == set(_lib.exported_symbols())
    assert _lib.load().mf_abi_version() == _lib.ABI_VERSION


def test_invalid_config_is_reported_not_raised_across_abi():
    from memfast_b200 import Config, _lib

    c = _lib.native_config(Config())
    bad = _lib.MFConfig.from_buffer_copy(c)
    bad.abi_version = 999
    size = ct.c_size_t()
    status = _lib.load().mf_quantize_workspace(ct.byref(bad), 0, 4, 4, ct.byref(size))
    assert status == _lib.MF_ERR_INVALID
    assert "ABI version" in _lib.last_error()
    with pytest.raises(ValueError):
        _lib.check(status, "probe")


def test_workspace_queries_need_no_gpu():
    from memfast_b200 import Config, Nonidealities, _lib

    ideal = Config(nonidealities=Nonidealities(write_variation=0.0))
    noisy = Config()
    size = ct.c_size_t()
    sched = _lib.schedule()
    lib = _lib.load()
    simt = _lib.schedule(kernel=1)
    assert lib.mf_sliced_mm_workspace(_lib.native_config(ideal), ct.byref(simt), 64, 2, 3, 0, 3, ct.byref(size)) == 0
    assert size.value == 0
    assert lib.mf_sliced_mm_workspace(_lib.native_config(ideal), ct.byref(sched), 64, 2, 3, 0, 3, ct.byref(size)) == 0
    # tensor-core digit dots: FP16 weight digits of 8 slices x 16-column blocks of the
    # 3 tiles (128 rows per block) over K = 128
    assert size.value == (3 * 64 // 16) * 128 * 128 * 2 + 256
    assert lib.mf_sliced_mm_workspace(_lib.native_config(noisy), ct.byref(simt), 64, 2, 3, 0, 3, ct.byref(size)) == 0
    # one group of `arrays` tiles of restored FP32 conductances: m * width * W * R * C * 4
    assert size.value == 2 * 2 * 8 * 64 * 64 * 4
    assert lib.mf_sliced_mm_workspace(_lib.native_config(noisy), ct.byref(sched), 64, 2, 3, 0, 3, ct.byref(size)) == 0
    # tensor-core currents: two FP16 parts of G - LOW for 8 weight slices x 4-column
    # blocks of the 3 tiles (NPAD = 32 rows per block and part) over K = 128
    assert size.value == (3 * 64 // 4) * 2 * 32 * 128 * 2 + 256
    assert lib.mf_quantize_workspace(_lib.native_config(noisy), 0, 10, 300, ct.byref(size)) == 0
    assert size.value >= 10 * 4


def test_native_config_mirrors_layouts():
    from memfast_b200 import Config, _lib

    cfg = Config(input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=(6, 7, 7, 8, 8),
                 array_size=(128, 128), rows_per_read=32)
    c = _lib.native_config(cfg)
    assert (c.n_in, c.n_w) == (5, 5)
    assert [c.in_shift[i] for i in range(5)] == [0, 2, 4, 6, 7]
    assert [c.w_factor[i] for i in range(5)] == [1, 4, 16, 64, -128]
    assert [c.adc_max[i] for i in range(5)] == [255, 255, 127, 127, 63]
    assert (c.rows, c.cols, c.read_rows, c.reads) == (128, 128, 32, 4)


def test_simulator_refuses_cpu():
    import memfast_b200 as mf

    with pytest.raises(ValueError):
        mf.Simulator(device="cpu")


def test_debug_stall_hook_validates_its_arguments():
    """The failure-detection test hook refuses a negative stage or an out-of-range budget
    (and so arms nothing) without touching a GPU."""
    from memfast_b200 import _lib

    lib = _lib.load()
    for stage, cycles in ((-1, 10_000), (0, 10), (0, 5_000_000_000)):
        assert lib.mf_debug_stall_next_launch(stage, cycles) == _lib.MF_ERR_INVALID
        assert "mf_debug_stall_next_launch" in _lib.last_error()


def test_schedule_grid_lists_each_execution_once():
    """The tuned-mode domain of the headline configuration covers all three ideal kernel
    families and both raster orders of the tensor-core ones, each execution once
    (mf_query resolves schedules on the host)."""
    from memfast_b200 import Config, Nonidealities
    from memfast_b200.tuning import _PATH_AXES, resolve, schedule_grid

    config = Config(array_size=(128, 128), rows_per_read=32, weight_quant_gran=(32, 1), input_quant_gran=(1, 32),
                    input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=(6, 7, 7, 8, 8),
                    nonidealities=Nonidealities(write_variation=0.0))
    domain = list(schedule_grid(config, 4096, 32, 32))
    identities = []
    for schedule in domain:
        path, _ = resolve(config, schedule, 4096, 32, 32)
        identities.append((path,) + tuple(schedule[axis] for axis in _PATH_AXES[path]))
    assert len(identities) == len(set(identities))
    paths = {identity[0] for identity in identities}
    assert paths == {"generic_ideal", "packed", "fp8_planes"}
    assert {i[:2] for i in identities if i[0] in ("packed", "fp8_planes")} == {
        ("packed", 0), ("packed", 1), ("fp8_planes", 0), ("fp8_planes", 1)}
    # Nonideal: SIMT currents over restore-group sizes, tensor-core currents in both orders.
    noisy = Config(array_size=(128, 128), rows_per_read=32, weight_quant_gran=(32, 1), input_quant_gran=(1, 32),
                   input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=(6, 7, 7, 8, 8),
                   nonidealities=Nonidealities(write_variation=0.02))
    paths = [resolve(noisy, s, 64, 4, 4)[0] for s in schedule_grid(noisy, 64, 4, 4)]
    assert paths.count("tc_currents") == 2 and paths.count("simt_currents") == 3   # arrays 1, 2, 4


def test_mf_mm_validates_on_the_host():
    """mf_mm refuses missing buffers and undersized workspaces before enqueuing anything."""
    from memfast_b200 import Config, Nonidealities, _lib

    config = Config(array_size=(128, 128), rows_per_read=32, weight_quant_gran=(32, 1), input_quant_gran=(1, 32),
                    input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=(6, 7, 7, 8, 8),
                    nonidealities=Nonidealities(write_variation=0.0))
    lib = _lib.load()
    cfg = _lib.native_config(config)
    sched = _lib.schedule()
    fake = ct.c_void_p(256)
    buffers = _lib.MFMMBuffers(fake, fake, fake, fake, fake, fake, fake, 1, fake, 1, fake, 1)
    args = (ct.byref(cfg), ct.byref(sched), fake, fake, 0, 64, 256, 128, 0, 0)
    assert lib.mf_mm(*args, None, 0, 0, 0, None, None) == _lib.MF_ERR_INVALID
    missing = _lib.MFMMBuffers.from_buffer_copy(buffers)
    missing.flags = None
    assert lib.mf_mm(*args, ct.byref(missing), 0, 0, 0, None, None) == _lib.MF_ERR_INVALID
    assert lib.mf_mm(*args, ct.byref(buffers), 0, 0, 0, None, None) == _lib.MF_ERR_RESOURCE
    assert "workspaces too small" in _lib.last_error()


def test_read_modes_resolve_to_their_current_kernels():
    """Every read mode of 32-row reads takes the tensor-core current kernel; output-mode
    read noise with 64-row reads or with voltage noise keeps the SIMT kernels.  The
    output mode's conductance operand carries, per 16-column block, the two halves of
    G' (160 rows for five weight slices), a row of ones padded to 16 rows, and two
    FP16 parts of G^2 (160 rows): 336 rows against the shared mode's 160.  Resolved on
    the host (mf_query, mf_sliced_mm_workspace), no GPU needed."""
    from memfast_b200 import Config, Nonidealities, _lib
    from memfast_b200.tuning import default_schedule, resolve

    int8 = dict(array_size=(128, 128), rows_per_read=32, weight_quant_gran=(32, 1), input_quant_gran=(1, 32),
                input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=(6, 7, 7, 8, 8))
    rpr64 = dict(array_size=(256, 256), rows_per_read=64, weight_quant_gran=(64, 1), input_quant_gran=(1, 64),
                 input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=(6, 7, 7, 8, 8))

    def config(shape, **effects):
        return Config(**shape, nonidealities=Nonidealities(write_variation=0.02, **effects))

    def path(c):
        return resolve(c, default_schedule(c), 64, 2, 3)[0]

    shared = config(int8, read_variation=0.02)
    pair = config(int8, read_variation=0.02, read_mode="slice_pair")
    output = config(int8, read_variation=0.02, read_mode="output")
    assert path(shared) == path(pair) == path(output) == "tc_currents"
    assert path(config(int8, read_variation=0.02, read_mode="output", voltage_variation=0.02)) == "simt_currents"
    assert path(config(rpr64, read_variation=0.02, read_mode="output")) == "simt_currents"

    lib = _lib.load()
    size = ct.c_size_t()
    blocks, k = 3 * 128 // 16, 2 * 128            # 16-column blocks of 3 tiles; K of 2 arrays
    for c, rows in ((shared, 160), (output, 336)):
        sched = _lib.schedule(**default_schedule(c))
        assert lib.mf_sliced_mm_workspace(_lib.native_config(c), ct.byref(sched), 64, 2, 3, 0, 3, ct.byref(size)) == 0
        assert size.value == blocks * rows * k * 2 + 256
