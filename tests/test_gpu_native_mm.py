"""The one-call product path: ``mf_mm`` behind ``AnalogMatrix._native_mm``.

From the second ``mm`` call on one right-hand tensor, the operand checks, the
in-place reprogramming of B, the quantisation of A, the fused product and the
output check are enqueued by one native call instead of one per step.  These
tests run the same call sequences with that path switched off and require the
outputs to agree bit for bit (read events and sampling seeds included), the
errors to be the same, in the reference's order (functional.py:50-53, then the
quantisers' dtype checks), and the FP64 rerun of a product whose FP32 epilogue
overflows (simulator.py:614-615) to happen as before.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import memfast_b200

    return memfast_b200


def _config(mf, case):
    int8 = dict(array_size=(128, 128), rows_per_read=32, weight_quant_gran=(32, 1), input_quant_gran=(1, 32),
                input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=(6, 7, 7, 8, 8))
    effects = {"ideal": dict(write_variation=0.0), "write": dict(write_variation=0.02),
               "noisy": dict(write_variation=0.02, read_variation=0.02, voltage_variation=0.02)}
    if case == "defaults":
        return mf.Config()
    if case == "bfp16":
        return mf.Config(array_size=(256, 256), rows_per_read=64, weight_quant_gran=(64, 1),
                         input_quant_gran=(1, 64), activation_bits=16, weight_bits=16, bw_e=8, adc_bits=8,
                         input_slice=(1, 3, 4, 4, 4), weight_slice=(1, 3, 4, 4, 4),
                         nonidealities=mf.Nonidealities(write_variation=0.05))
    return mf.Config(**int8, nonidealities=mf.Nonidealities(**effects[case]))


class _Spy:
    """Counts the products that went through the native path."""

    def __init__(self, original):
        self.original, self.calls = original, 0

    def __call__(self, matrix, *args, **kwargs):
        self.calls += 1
        return self.original(matrix, *args, **kwargs)


def _runs(mf, monkeypatch, config, a, b, steps=3):
    """``steps`` calls of Simulator.mm(a, b): with the native path, then without it."""
    from memfast_b200 import functional
    from memfast_b200.simulator import AnalogMatrix

    spy = _Spy(AnalogMatrix._native_mm)
    with monkeypatch.context() as patch:
        patch.setattr(AnalogMatrix, "_native_mm", lambda self, *args, **kw: spy(self, *args, **kw))
        sim = mf.Simulator(config)
        native = [sim.mm(a, b) for _ in range(steps)]
    with monkeypatch.context() as patch:
        patch.setattr(functional, "_native_product", lambda *args, **kwargs: None)
        sim = mf.Simulator(config)
        plain = [sim.mm(a, b) for _ in range(steps)]
    return native, plain, spy.calls


def _same(x, y):
    return x.dtype == y.dtype and x.shape == y.shape and torch.equal(x.view(torch.uint8), y.view(torch.uint8))


@pytest.mark.parametrize("case", ["ideal", "write", "noisy", "defaults", "bfp16"])
def test_native_mm_matches_the_step_by_step_path(mf, monkeypatch, case):
    """Every call after the first takes the native path; all calls agree bit for bit
    (events 0, 1, 2: nonideal draws differ per event, so the seeds and events match)."""
    config = _config(mf, case)
    g = torch.Generator().manual_seed(7)
    a, b = torch.randn(200, 600, generator=g).cuda(), torch.randn(600, 333, generator=g).cuda()
    native, plain, calls = _runs(mf, monkeypatch, config, a, b)
    assert calls == 2
    for x, y in zip(native, plain):
        assert _same(x, y)
    if case == "noisy":
        assert not torch.equal(native[1], native[2])   # read noise: the read event advanced


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float64])
def test_native_mm_other_dtypes(mf, monkeypatch, dtype):
    """Half, bfloat16 and double operands: the checks run as separate passes before the
    quantisers (no folded check), results cast back to the operands' dtype."""
    config = _config(mf, "write")
    g = torch.Generator().manual_seed(11)
    a = torch.randn(130, 300, generator=g).to(dtype).cuda()
    b = torch.randn(300, 260, generator=g).to(dtype).cuda()
    native, plain, calls = _runs(mf, monkeypatch, config, a, b, steps=2)
    assert calls == 1
    for x, y in zip(native, plain):
        assert x.dtype == dtype and _same(x, y)


def test_native_mm_launches_fewer_kernels(mf, monkeypatch):
    """FP32 operands of the one-pass quantisers: no separate operand-check passes."""
    from memfast_b200 import _lib, functional

    config = _config(mf, "ideal")
    g = torch.Generator().manual_seed(3)
    a, b = torch.randn(512, 1024, generator=g).cuda(), torch.randn(1024, 512, generator=g).cuda()
    sim = mf.Simulator(config)
    lib = _lib.load()
    first = sim.mm(a, b)
    with monkeypatch.context() as patch:
        patch.setattr(functional, "_native_product", lambda *args, **kwargs: None)
        before = lib.mf_launch_count()
        second = sim.mm(a, b)
        step_by_step = lib.mf_launch_count() - before
    before = lib.mf_launch_count()
    third = sim.mm(a, b)
    native = lib.mf_launch_count() - before
    assert torch.equal(first, second) and torch.equal(first, third)
    # Quantise A, program B (K-major copy included), the packed kernel, its rerun
    # filter, the output check; the step-by-step path adds two operand-check passes.
    assert native == 5 and step_by_step == native + 2, (native, step_by_step)
    assert _lib.PATHS[lib.mf_last_path()] == "packed"


@pytest.mark.parametrize("bad", ["A", "B", "both"])
def test_native_mm_operand_errors(mf, bad):
    """Non-finite operands raise the reference's error, A's first, and leave the
    simulator usable: the next clean call equals a fresh simulator's."""
    config = _config(mf, "write")
    g = torch.Generator().manual_seed(5)
    a, b = torch.randn(64, 256, generator=g).cuda(), torch.randn(256, 128, generator=g).cuda()
    sim = mf.Simulator(config)
    first = sim.mm(a, b)
    a_bad, b_bad = a.clone(), b.clone()
    if bad in ("A", "both"):
        a_bad[3, 17] = float("nan")
    if bad in ("B", "both"):
        b_bad[9, 4] = float("inf")
    # B is programmed by tensor object: write the bad values into b itself.
    saved = b.clone()
    b.copy_(b_bad)
    with pytest.raises(ValueError, match="A must be finite" if bad != "B" else "B must be finite"):
        sim.mm(a_bad, b)
    b.copy_(saved)
    again = sim.mm(a, b)
    fresh = mf.Simulator(config)
    expected = [fresh.mm(a, b) for _ in range(2)]
    assert torch.equal(first, expected[0])
    # The failed call raised before its read event counted, as on the step-by-step path.
    assert torch.equal(again, expected[1])


def test_native_mm_narrowing_error(mf):
    """Double operands that overflow FP32 in the quantiser raise its dtype error."""
    config = _config(mf, "ideal")
    g = torch.Generator().manual_seed(2)
    a = torch.randn(32, 128, generator=g, dtype=torch.float64).cuda()
    b = torch.randn(128, 64, generator=g, dtype=torch.float64).cuda()
    sim = mf.Simulator(config)
    sim.mm(a, b)
    a[0, 0] = 1e300
    with pytest.raises(ValueError, match="finite in torch.float32"):
        sim.mm(a, b)


def test_native_mm_fp64_rerun(mf, monkeypatch):
    """An FP32 epilogue overflow on the native path reruns in FP64 like the step-by-step path."""
    rng = np.random.default_rng(23)
    a = rng.standard_normal((256, 512), dtype=np.float32)
    b = rng.standard_normal((512, 384), dtype=np.float32)
    a[200] *= np.float32(3e37)
    b *= np.float32(1e-30)
    a, b = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    native, plain, calls = _runs(mf, monkeypatch, _config(mf, "ideal"), a, b, steps=2)
    assert calls == 1
    for x, y in zip(native, plain):
        assert _same(x, y) and bool(torch.isfinite(x).all())


def test_native_mm_row_shard_offset(mf, monkeypatch):
    """A row shard (sharded_mm with a vector offset) on the native path equals the same
    rows of the whole product, nonideal noise included."""
    from memfast_b200.sharding import sharded_mm

    config = _config(mf, "noisy")
    g = torch.Generator().manual_seed(19)
    a, b = torch.randn(256, 384, generator=g).cuda(), torch.randn(384, 256, generator=g).cuda()
    whole = mf.Simulator(config)
    full = [whole.mm(a, b) for _ in range(2)]
    shard = mf.Simulator(config)
    rows = [sharded_mm(a[96:160].contiguous(), b, simulator=shard, row_offset=96) for _ in range(2)]
    for got, want in zip(rows, full):
        assert torch.equal(got, want[96:160])


def test_native_mm_plans_follow_row_count_changes(mf, monkeypatch):
    """Alternating vector counts on one right-hand tensor (plans per row count, a
    workspace that grows) give the step-by-step path's results call for call."""
    from memfast_b200 import functional

    config = _config(mf, "ideal")
    g = torch.Generator().manual_seed(29)
    b = torch.randn(512, 256, generator=g).cuda()
    inputs = [torch.randn(rows, 512, generator=g).cuda() for rows in (64, 640, 64, 200, 640)]
    sim = mf.Simulator(config)
    native = [sim.mm(a, b) for a in inputs]
    with monkeypatch.context() as patch:
        patch.setattr(functional, "_native_product", lambda *args, **kwargs: None)
        sim = mf.Simulator(config)
        plain = [sim.mm(a, b) for a in inputs]
    for x, y in zip(native, plain):
        assert _same(x, y)
