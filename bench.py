#!/usr/bin/env python
"""Benchmark of the sliced analog matrix product (BASELINE metric).

Metric: simulated MAC/s of ``Simulator.mm`` on the 4096x4096x4096 sliced INT8
workload (array 128x128, rows_per_read 32, groups
(32,1)/(1,32), slices (1,1,2,2,2), adc_bits (6,7,7,8,8), ideal device) on
seeded N(0,1) FP32 operands.  One step = one ``Simulator.mm(A, B)`` call
(quantise A, reprogram B, sliced product with fused epilogue), operands
resident in HBM.  ``e2e`` times the host-operand call ``streaming.host_mm`` on
pinned A and B: both copied in and the product copied out inside the timed
region, the copies overlapped with the product row chunk by row chunk.  With --gpus N (one process per GPU
under torchrun) the batch has 4096 rows per GPU: every rank runs the 4096^3
product on its own row block of one (4096 N)-row batch with B replicated, its
vectors keeping their global indices (noise addresses), and keeps its output
rows (weak scaling; the path has no data exchange).  --gather adds an NCCL
all-gather of the output rows to every step.

``--impl reference`` times the reference algorithm's CPU restatement (the
oracle: restored conductances, FP32 currents, ADC, signed reconstruction,
scale epilogue) on the host cores, on bounded row prefixes of the same
workload; the full-batch time is extrapolated linearly in rows.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

UNIT = "MAC/s"


def metric_name(size):
    return f"simulated MAC/s on {size}^3 sliced INT8 Simulator.mm"


def parse():
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["engine", "reference"], default="engine")
    p.add_argument("--size", type=int, default=4096, help="N = K = O")
    p.add_argument("--skip-cpu", action="store_true", help="omit the cpu_baseline leg")
    p.add_argument("--cpu-seconds", type=float, default=15.0, help="CPU work budget of the baseline sample")
    p.add_argument("--gather", action="store_true",
                   help="with --gpus N > 1, also all-gather every rank's output rows inside each step")
    p.add_argument("--kernel", type=int, default=0, choices=[0, 1, 2, 3],
                   help="schedule kernel of the kernel-only timing (0 automatic, 1 generic SIMT, "
                        "2 tcgen05 (packed counts / nonideal currents), 3 tcgen05 FP8 digit planes)")
    p.add_argument("--effects", choices=sorted(EFFECTS), default="ideal",
                   help="device effects of the configs[1] sweep: ideal (the headline), write "
                        "(write variation 0.02), shared (write + shared read variation 0.02), "
                        "noisy (write + read + voltage variation 0.02, BASELINE's noisy run)")
    return p.parse_args()


EFFECTS = {
    "ideal": dict(write_variation=0.0),
    "write": dict(write_variation=0.02),
    "shared": dict(write_variation=0.02, read_variation=0.02),
    "noisy": dict(write_variation=0.02, read_variation=0.02, voltage_variation=0.02),
}


def bench_config(mf_module, effects="ideal"):
    return mf_module.Config(
        array_size=(128, 128), rows_per_read=32, weight_quant_gran=(32, 1), input_quant_gran=(1, 32),
        input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=(6, 7, 7, 8, 8),
        nonidealities=mf_module.Nonidealities(**EFFECTS[effects]),
    )


def operands(size, seed=2024, rank=0):
    """Seeded N(0,1) operands: B is the same on every rank; rank 0's A is the 1-GPU A and
    rank r > 0 draws its own rows from a seed of its own."""
    import torch

    g = torch.Generator().manual_seed(seed)
    a = torch.randn(size, size, generator=g)
    b = torch.randn(size, size, generator=g)
    if rank > 0:
        a = torch.randn(size, size, generator=torch.Generator().manual_seed(seed + 7919 * rank))
    return a, b


def workload(args):
    n = k = o = args.size
    gpus = args.gpus
    effects = getattr(args, "effects", "ideal")
    label = "ideal" if effects == "ideal" else "nonideal: " + ", ".join(
        f"{name.replace('_variation', '')} {value}" for name, value in EFFECTS[effects].items())
    return dict(workload=f"Simulator.mm {n}x{k}x{o} INT8 (1,1,2,2,2) {label} per GPU", n=n, k=k, o=o,
                batch=f"{gpus} row block(s) of {n}: one {n * gpus}-row batch, rows sharded, B replicated"
                      + (", output rows all-gathered" if getattr(args, "gather", False) and gpus > 1 else
                         ", each rank keeps its output rows"),
                array=[128, 128], rows_per_read=32, adc_bits=[6, 7, 7, 8, 8],
                input_groups=[1, 32], weight_groups=[32, 1], operands="seeded N(0,1) fp32",
                l2=f"inputs 2x{4 * n * k / 2**20:.0f} MiB fp32; L2 (126 MB) flushed by a 256 MiB write "
                   f"before every timed step")


# ------------------------------------------------------------------ CPU leg --
class OracleSample:
    """The oracle (the reference CPU algorithm restated in C) on a row prefix.

    One call programs B (restores every conductance) and then runs the rows, so
    time = fixed + rows * per_row.  Both terms are measured from two prefixes and
    the full-batch time is extrapolated linearly (work is exactly linear in the
    rows: every vector is independent).
    """

    def __init__(self, size, config, budget_s):
        from oracle import oracle as O

        self.O = O
        self.size, self.config = size, config
        self.threads = os.cpu_count() or 1
        O.set_threads(self.threads)
        O.lib()
        a, b = operands(size)
        self.a, self.b = a.numpy(), b.numpy()
        t1 = self.time(1)
        t9 = self.time(9)
        per_row = max((t9 - t1) / 8, 1e-6)
        fixed = max(t1 - per_row, 0.0)
        self.rows = int(max(9, min(size, (budget_s - fixed) / per_row)))
        self.t1 = t1

    def time(self, rows):
        start = time.perf_counter()
        self.O.mm(self.a[:rows], self.b, self.config, physical=True)
        return time.perf_counter() - start

    def rate(self, t_rows):
        """Extrapolated full-batch MAC/s from one timing of self.rows rows."""
        per_row = max((t_rows - self.t1) / (self.rows - 1), 1e-9)
        fixed = max(self.t1 - per_row, 0.0)
        full = fixed + per_row * self.size
        return float(self.size) ** 3 / full, full

    def describe(self, elapsed):
        return (f"oracle C restatement of the reference CPU algorithm (physical FP32 currents, ADC, "
                f"reconstruction, scale epilogue) on {self.threads} threads; prefixes of 1 and {self.rows} of "
                f"{self.size} rows timed ({elapsed:.1f} s), B programmed once per call, full-batch time "
                f"extrapolated linearly in rows")


def cpu_sample(size, budget_s, config):
    sample = OracleSample(size, config, budget_s)
    elapsed = sample.time(sample.rows)
    value, full = sample.rate(elapsed)
    return dict(value=value, unit=UNIT, cores=sample.threads, kind="port", sample=sample.describe(elapsed),
                extrapolated_full_batch_s=full, rows=sample.rows)


def reference_arm(args):
    import memfast_b200 as mf

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    config = bench_config(mf, args.effects)
    budget = max(2.0, 150.0 / max(1, args.steps + args.warmup))
    sample = OracleSample(args.size, config, budget)
    rates, times = [], []
    for step in range(args.warmup + args.steps):
        elapsed = sample.time(sample.rows)
        if step >= args.warmup:
            rates.append(sample.rate(elapsed)[0])
            times.append(elapsed)
    value = statistics.mean(rates)
    line = dict(metric=metric_name(args.size), value=value, unit=UNIT, n_gpus=args.gpus, steps=args.steps, warmup=args.warmup,
                ms_per_step=float(args.size) ** 3 / value * 1e3, higher_is_better=True, scaling="weak",
                vs_baseline=None, dtype="f32 currents / int64 totals", data="synthetic", config=workload(args),
                impl="reference",
                cpu_baseline=dict(value=value, unit=UNIT, cores=sample.threads, kind="port",
                                  sample=sample.describe(sum(times)) + "; each step one prefix call"),
                e2e=dict(value=value, unit=UNIT, h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ clock sampler --
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.samples = []
        self.proc = None
        self.device_index = device_index

    def __enter__(self):
        try:
            import torch

            ident = str(torch.cuda.get_device_properties(self.device_index).uuid)
            ident = ident if ident.startswith("GPU-") else f"GPU-{ident}"
        except Exception:
            ident = str(self.device_index)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={ident}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.samples.append(parts)

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=["no samples"], samples=0)
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[5 + i] == "Active"})
        return dict(sm_mhz=statistics.median(sm) if sm else None, sm_max_mhz=max(mx) if mx else None,
                    reasons=reasons, samples=len(self.samples))


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return data.get("bf16_tflops"), data.get("hbm_gbs"), "measured"
    return 1590.0, 6650.0, "fallback"


def profiled_traffic():
    """dram bytes per launch of the sliced-mm kernel from the committed ncu summary, if any."""
    path = ROOT / "profiles" / "sliced_mm_4096_ideal.md"
    if path.exists():
        for line in path.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                try:
                    return float(line.split(":", 1)[1].split()[0])
                except ValueError:
                    return None
    return None


# --------------------------------------------------------------- engine arm --
def engine_arm(args):
    import torch
    import torch.distributed as dist

    import memfast_b200 as mf
    from memfast_b200 import _lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    from memfast_b200.sharding import gather_rows, row_range, sharded_mm

    config = bench_config(mf, args.effects)
    size = args.size
    # Weak scaling: every rank owns `size` rows of a (size * world)-row batch; its rows
    # carry their global vector indices (noise addresses), so each rank's output rows
    # equal those rows of a single-device run.
    a_cpu, b_cpu = operands(size, rank=rank)
    total_rows = size * world
    r0, r1 = rank * size, (rank + 1) * size
    rows = r1 - r0
    a_host = a_cpu.contiguous().pin_memory()
    b_host = b_cpu.contiguous().pin_memory()
    a = a_host.to(device)
    b = b_host.to(device)
    sim = mf.Simulator(config, device=device)
    out_host = torch.empty((r1 - r0, size), pin_memory=True)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    def step(x, y):
        # This rank's rows with global vector indices; optionally the rows of every rank.
        out = sharded_mm(x, y, simulator=sim, row_offset=r0) if world > 1 else sim.mm(x, y)
        if world > 1 and args.gather:
            gather_rows(out, total_rows)
        return out

    def timed(fn, count):
        times = []
        for _ in range(count):
            flush.zero_()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize(device)
            start.record(stream)
            fn()
            end.record(stream)
            torch.cuda.synchronize(device)
            times.append(start.elapsed_time(end) / 1e3)
        return times

    for _ in range(args.warmup):
        step(a, b)
    torch.cuda.synchronize(device)
    launches0 = _lib.load().mf_launch_count()
    with ClockSampler(local) as clocks:
        t_wall = time.perf_counter()
        times = timed(lambda: step(a, b), args.steps)
        launches = _lib.load().mf_launch_count() - launches0
        # Keep the GPU loaded long enough for the clock sampler (not part of the measurement).
        while time.perf_counter() - t_wall < 1.0:
            step(a, b)
            torch.cuda.synchronize(device)
    per_step = sum(times) / len(times)

    # End to end through the host-operand API: pinned A and B copied in and the
    # product copied out every step, overlapped chunk by chunk with the compute.
    from memfast_b200.streaming import host_mm

    def e2e_step():
        host_mm(a_host, b_host, simulator=sim, out=out_host, row_offset=r0)
        if world > 1 and args.gather:
            gather_rows(out_host.to(device), total_rows)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    e2e_times = timed(e2e_step, args.steps)
    e2e_step_s = sum(e2e_times) / len(e2e_times)

    # Dominant kernel alone: one mf_sliced_mm call on pre-quantised operands with a
    # preallocated workspace and output (no Python work inside the timed region).
    import ctypes as ct

    from memfast_b200.quantization import input_tiles
    from memfast_b200.simulator import default_schedule

    matrix = sim._matrix_for(b)
    q, xscale = input_tiles(a, config)
    schedule = dict(default_schedule(config), kernel=args.kernel)
    n_rows = q.shape[0]
    ws_bytes = matrix._workspace_size(n_rows, schedule)
    workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=device)
    out_k = torch.empty((n_rows, size), device=device)
    native = _lib.schedule(**schedule)
    lib = _lib.load()
    cfg = _lib.native_config(config)

    def sliced_mm():
        _lib.check(lib.mf_sliced_mm(
            cfg, ct.byref(native), _lib.ptr(q), _lib.ptr(xscale), _lib.ptr(matrix.packed),
            _lib.ptr(matrix.weight_scale), None, _lib.ptr(out_k), n_rows, matrix.packed.shape[0], matrix.p,
            size, size, 0, matrix.p, matrix.seed & 0xFFFFFFFF, 0, 0, 0, _lib.ptr(workspace), ws_bytes,
            _lib.stream_of(device)), "mf_sliced_mm")

    for _ in range(2):
        sliced_mm()
    kernel_times = timed(sliced_mm, max(3, args.steps))
    kernel_s = sum(kernel_times) / len(kernel_times)
    from memfast_b200.simulator import check_device_error

    check_device_error()   # a bounded device-side wait that gave up invalidates the timing

    def reduce_max(value):
        if world == 1:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    per_step = reduce_max(per_step)
    e2e_step_s = reduce_max(e2e_step_s)
    kernel_s = reduce_max(kernel_s)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    macs = float(size) ** 3 * world
    pairs = len(config.input_layout) * len(config.weight_layout)
    bf16, hbm, peak_kind = measured_peaks()
    ideal = args.effects == "ideal"
    # Ideal: int8 digit MMAs against the int8 dense rate (2 x bf16).  Nonideal: FP16 digit x
    # conductance MMAs against the f16 dense rate (= bf16); each current's two FP16 halves
    # double the issued MMA work over this algorithmic count.
    peak_tops = 2.0 * bf16 if ideal else bf16
    kernel_ops = 2.0 * (rows * size * size) * pairs
    achieved_tops = kernel_ops / kernel_s / 1e12
    traffic = profiled_traffic() if ideal else None
    path = ("the tensor-core kernel plus its K-major weight copy and rare-tile filter launch" if ideal else
            "the conductance restore and the current kernel")
    line = dict(
        metric=metric_name(args.size), value=macs / per_step, unit=UNIT, n_gpus=world, steps=args.steps, warmup=args.warmup,
        ms_per_step=per_step * 1e3, higher_is_better=True, scaling="weak", vs_baseline=None,
        dtype="u8 digits / int32 totals / f32 epilogue" if ideal else
              "f16 digits x f16 conductance halves / f32 currents, ADC and epilogue",
        data="synthetic", config=workload(args),
        slice_pair_macs_per_s=macs * pairs / per_step,
        roofline=dict(bound="tensor", achieved=achieved_tops, peak=peak_tops, unit="TFLOP/s",
                      frac=achieved_tops / peak_tops, traffic=traffic,
                      note=f"one mf_sliced_mm call (schedule kernel {args.kernel}: {path}), "
                           f"{rows}x{size}x{size}; algorithmic {pairs} slice-pair MAC streams x2 ops; peak = "
                           + (f"2 x {peak_kind} dense bf16 ({bf16} TFLOP/s), the int8 dense rate of B200" if ideal
                              else f"{peak_kind} dense bf16 ({bf16} TFLOP/s), the f16 dense rate of B200"),
                      kernel_ms=kernel_s * 1e3),
        e2e=dict(value=macs / e2e_step_s, unit=UNIT,
                 h2d_bytes_per_step=int(2 * size * size * world * 4),
                 d2h_bytes_per_step=int(size * size * world * 4), ms_per_step=e2e_step_s * 1e3),
        gpu_launches=int(launches),
        clocks=clocks.summary(),
    )
    if world == 1 and not args.skip_cpu:
        line["cpu_baseline"] = cpu_sample(size, args.cpu_seconds, config)
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
    else:
        engine_arm(args)


if __name__ == "__main__":
    main()
