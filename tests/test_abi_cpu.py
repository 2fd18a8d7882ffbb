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
