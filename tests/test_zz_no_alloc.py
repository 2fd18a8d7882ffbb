"""mf_quantize_input_static: input quantisation with the library's own scratch.

Collected last on purpose (file name), so it also runs after every other test
has used the library on the same device.
"""

import ctypes as ct

import pytest
import torch

from memfast_b200 import Config, _lib


def _config(**kwargs):
    base = dict(array_size=(128, 128), rows_per_read=32, weight_quant_gran=(32, 1), input_quant_gran=(1, 32),
                input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=(6, 7, 7, 8, 8))
    base.update(kwargs)
    return Config(**base)


def _sizes(config, n, k):
    m = -(-k // config.array_size[0])
    wide = config.wide_codes
    return m, (torch.int64 if wide else torch.uint8), (torch.float64 if config.wide else torch.float32)


def _fixed(config, x, fixed):
    return None if fixed is None else _lib.ptr(fixed)


def _with_workspace(config, x, fixed=None):
    n, k = x.shape
    ldx = x.stride(0)
    m, code_dtype, scale_dtype = _sizes(config, n, k)
    codes = torch.full((n, m * config.array_size[0]), 0x5A, dtype=code_dtype, device=x.device)
    xscale = torch.full((n, m * config.reads_per_array), -1.0, dtype=scale_dtype, device=x.device)
    size = ct.c_size_t()
    native = _lib.native_config(config)
    _lib.check(_lib.load().mf_quantize_workspace(ct.byref(native), 0, n, k, ct.byref(size)), "workspace")
    workspace = torch.empty(size.value, dtype=torch.uint8, device=x.device)
    _lib.check(_lib.load().mf_quantize_input(ct.byref(native), _lib.ptr(x), _lib.DTYPES[x.dtype], n, k, ldx,
                                             _fixed(config, x, fixed), _lib.ptr(codes), _lib.ptr(xscale),
                                             _lib.ptr(workspace), size.value, _lib.stream_of(x.device)),
               "mf_quantize_input")
    return codes, xscale


def _static(config, x, fixed=None):
    n, k = x.shape
    ldx = x.stride(0)
    m, code_dtype, scale_dtype = _sizes(config, n, k)
    codes = torch.full((n, m * config.array_size[0]), 0xA5, dtype=code_dtype, device=x.device)
    xscale = torch.full((n, m * config.reads_per_array), -2.0, dtype=scale_dtype, device=x.device)
    native = _lib.native_config(config)
    _lib.check(_lib.load().mf_quantize_input_static(ct.byref(native), _lib.ptr(x), _lib.DTYPES[x.dtype], n, k, ldx,
                                                    _fixed(config, x, fixed), _lib.ptr(codes), _lib.ptr(xscale),
                                                    _lib.stream_of(x.device)), "mf_quantize_input_static")
    return codes, xscale


def test_static_quantize_rejects_oversize_without_a_gpu_call():
    """Group maxima beyond the static capacity are refused before any device work."""
    config = _config()
    native = _lib.native_config(config)
    # (1, 32) groups, FP32 maxima: n * k / 32 * 4 bytes; 4096 x 65536 needs 32 MiB.
    n, k = 4096, 65536
    status = _lib.load().mf_quantize_input_static(ct.byref(native), ct.c_void_p(16), _lib.DTYPES[torch.float32],
                                                  n, k, k, None, ct.c_void_p(16), ct.c_void_p(16), None)
    assert status == _lib.MF_ERR_RESOURCE
    message = _lib.last_error()
    assert "static scratch" in message and str(_lib.STATIC_QUANTIZE_SCRATCH_BYTES) in message
    with pytest.raises(_lib.ResourceError):
        _lib.check(status, "mf_quantize_input_static")


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["one_pass", "bfp16", "row_pairs", "odd_ldx", "fixed_scale"])
def test_static_quantize_matches_workspace_entry_point(case):
    """Two calls in a row: the second must not see the first call's group maxima.

    The cases reach each path of the shared quantiser: the FP32 one-pass row-group
    kernel (which writes every maximum it reads), the FP64 maxima of BFP16 and the
    FP32 atomic maxima of groups spanning two rows (both cleared before the max
    pass), an odd row stride (the general kernels), and a fixed input scale (no
    maxima at all)."""
    kwargs = dict(bfp16=dict(bw_e=8, input_slice=(1, 3, 4, 4, 4), weight_slice=(1, 3, 4, 4, 4), activation_bits=16,
                             weight_bits=16, adc_bits=6),
                  row_pairs=dict(input_quant_gran=(2, 32))).get(case, {})
    config = _config(**kwargs)
    g = torch.Generator().manual_seed(31)
    # Large values first, then small ones on a different shape: stale maxima
    # from call one would shrink every code of call two.
    first = (torch.randn(512, 1000, generator=g) * 100.0).cuda()
    second = (torch.randn(300, 2048, generator=g) * 0.01).cuda()
    if case == "odd_ldx":
        first = torch.nn.functional.pad(first, (0, 3))[:, :1000]
        second = torch.nn.functional.pad(second, (0, 5))[:, :2048]
        assert first.stride(0) == 1003 and second.stride(0) == 2053
    for x in (first, second):
        fixed = None
        if case == "fixed_scale":
            # Per-column scales, constant along each 32-column read (as set_input_scale requires).
            peak = torch.nn.functional.pad(x.abs().amax(0), (0, -x.shape[1] % 32)).view(-1, 32).amax(1)
            fixed = (peak / 127.0).clamp_min(1e-6).repeat_interleave(32)[: x.shape[1]].contiguous()
        expected = _with_workspace(config, x, fixed)
        got = _static(config, x, fixed)
        torch.cuda.synchronize()
        assert torch.equal(got[0], expected[0])
        assert torch.equal(got[1].view(torch.int32 if got[1].dtype == torch.float32 else torch.int64),
                           expected[1].view(torch.int32 if expected[1].dtype == torch.float32 else torch.int64))
