#!/usr/bin/env python
"""Benchmark of the sliced analog matrix product (BASELINE metric).

Metric: simulated MAC/s of ``Simulator.mm`` on the 4096x4096x4096 sliced INT8
workload (array 128x128, rows_per_read 32, groups
(32,1)/(1,32), slices (1,1,2,2,2), adc_bits (6,7,7,8,8), ideal device) on
seeded N(0,1) FP32 operands.  One step = one ``Simulator.mm(A, B)`` call
(quantise A, reprogram B, sliced product with fused epilogue), operands
resident in HBM.  ``e2e`` times the host-operand call ``streaming.host_mm`` on
pinned A and B: both copied in and the product copied out inside the timed
region, the copies overlapped with the product row chunk by row chunk.

With --gpus N (one process per GPU under torchrun) the default is strong
scaling: the one 4096^3 product is split into N row blocks (``row_range``);
each rank computes its block (``sharding.row_parallel_mm``: quantise its rows
of A, program B, the fused product, written straight into its rows of the full
output) and an NCCL all-gather, enqueued before the step's one host
synchronisation, fills every rank's copy of the full output in place.  Both are inside every timed step; ``breakdown`` reports the kernel,
the gather and the rest per step (max over ranks).  ``--scaling weak`` keeps
the earlier measurement instead: 4096 rows per rank, each rank keeping its
output rows (``--gather`` adds the all-gather).

``--impl reference`` times the reference algorithm's CPU restatement (the
oracle: restored conductances, FP32 currents, ADC, signed reconstruction,
scale epilogue) on the host cores, on a bounded row prefix of the same
workload per step.

``parity`` in the line: rows of the step's own output (the first call, read
event 0) checked against the oracle outside the timed region.
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

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

UNIT = "MAC/s"

EFFECTS = {
    "ideal": dict(write_variation=0.0),
    "write": dict(write_variation=0.02),
    "shared": dict(write_variation=0.02, read_variation=0.02),
    "noisy": dict(write_variation=0.02, read_variation=0.02, voltage_variation=0.02),
    # Read noise drawn per (input slice, weight slice, cell) instead of per cell.
    "pair": dict(write_variation=0.02, read_variation=0.02, read_mode="slice_pair"),
    # Read noise drawn per ADC event from the read's second moments.
    "output": dict(write_variation=0.02, read_variation=0.02, read_mode="output"),
}


WORKLOADS = ("sweep", "matrix-int4", "matrix-int8", "matrix-bfp16", "resnet50", "llama7b")

# the format/nonideality matrix at 2048^3 (array 256x256, 64-row reads,
# groups (64,1)/(1,64)) with every effect on together.  The configuration leaves the ADC
# resolution open; Config's default (6 bits; 8 for the 16-bit format) is used, as in the
# golden cases of the same configurations (tests/golden/*_matrix.npz).
MATRIX_EFFECTS = dict(write_variation=0.05, adc_nonlinearity=0.02, stuck_at_low=5e-4, stuck_at_high=5e-4,
                      drift_coefficient=0.05, drift_time=100.0)
MATRIX_FORMATS = {
    "int4": dict(activation_bits=4, weight_bits=4, input_slice=(1, 1, 2), weight_slice=(1, 1, 2)),
    "int8": dict(input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2)),
    "bfp16": dict(activation_bits=16, weight_bits=16, input_slice=(1, 3, 4, 4, 4), weight_slice=(1, 3, 4, 4, 4),
                  bw_e=8, adc_bits=8),
}


def metric_name(size, label="INT8"):
    return f"simulated MAC/s on {size}^3 sliced {label} Simulator.mm"


def matrix_config(mf_module, fmt):
    return mf_module.Config(array_size=(256, 256), rows_per_read=64, input_quant_gran=(1, 64),
                            weight_quant_gran=(64, 1), nonidealities=mf_module.Nonidealities(**MATRIX_EFFECTS),
                            **MATRIX_FORMATS[fmt])


def product_spec(mf_module, args):
    """(config, size, format label, effects label) of a matrix-product workload."""
    if args.workload == "sweep":
        return bench_config(mf_module, args.effects), args.size, "INT8", effects_label(args.effects)
    fmt = args.workload.split("-", 1)[1]
    effects = "nonideal: write 0.05, S-curve ADC 0.02, stuck-at 1e-3 (half low, half high), drift c=0.05 t=100 s"
    return matrix_config(mf_module, fmt), 2048, {"int4": "INT4", "int8": "INT8", "bfp16": "BFP16"}[fmt], effects


def parse(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["engine", "reference", "reference-cuda"], default="engine",
                   help="reference: the reference algorithm's CPU restatement on the host cores; reference-cuda: "
                        "the unmodified reference package (installed in baseline/_ref) on its own CUDA path")
    p.add_argument("--workload", choices=WORKLOADS, default="sweep",
                   help="sweep: BASELINE configs[1] at --size (the headline at 4096); matrix-*: configs[2] at "
                        "2048^3; resnet50: configs[3]; llama7b: configs[4]")
    p.add_argument("--size", type=int, default=4096, help="N = K = O of the sweep")
    p.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                   help="with --gpus N > 1: split the one product over the ranks and all-gather its output "
                        "(strong, default) or give every rank a product of its own (weak)")
    p.add_argument("--skip-cpu", action="store_true", help="omit the cpu_baseline leg")
    p.add_argument("--llama-layers", type=int, default=32, help="decoder layers of the llama7b line")
    p.add_argument("--cpu-seconds", type=float, default=15.0, help="CPU work budget of the baseline sample")
    p.add_argument("--parity-rows", type=int, default=16,
                   help="rows checked against the oracle when the cpu_baseline leg does not run")
    p.add_argument("--exchange", choices=["nccl", "peers"], default="nccl",
                   help="strong scaling: how every rank's output rows reach the others -- an NCCL all-gather "
                        "after the product (default; faster at 8 GPUs) or peer stores from the packed kernel's "
                        "epilogue over NVLink (falls back to NCCL where unavailable)")
    p.add_argument("--gather", action="store_true",
                   help="--scaling weak only: also all-gather every rank's output rows inside each step")
    p.add_argument("--kernel", type=int, default=0, choices=[0, 1, 2, 3],
                   help="schedule kernel of the kernel-only timing (0 automatic, 1 generic SIMT, "
                        "2 tcgen05 (packed counts / nonideal currents), 3 tcgen05 FP8 digit planes)")
    p.add_argument("--effects", choices=sorted(EFFECTS), default="ideal",
                   help="device effects of the configs[1] sweep: ideal (the headline), write "
                        "(write variation 0.02), shared (write + shared read variation 0.02), "
                        "noisy (write + read + voltage variation 0.02, BASELINE's noisy run), pair (write + "
                        "read variation 0.02 drawn per slice pair), output (write + read variation 0.02 drawn per ADC event)")
    return p.parse_args(argv)


def bench_config(mf_module, effects="ideal"):
    return mf_module.Config(
        array_size=(128, 128), rows_per_read=32, weight_quant_gran=(32, 1), input_quant_gran=(1, 32),
        input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=(6, 7, 7, 8, 8),
        nonidealities=mf_module.Nonidealities(**EFFECTS[effects]),
    )


def operands(size, seed=2024, rank=0):
    """Seeded N(0,1) FP32 operands as numpy arrays, A [size, size] then B [size, size].

    numpy's PCG64 generator is scalar C code, so every host draws the same values
    (the golden outputs of the reference in tests/golden are keyed to them).  B is
    the same on every rank; rank 0's A is the one-GPU A, and rank r > 0 of the
    weak-scaling run draws its own rows from a seed of its own."""
    import numpy as np

    rng = np.random.default_rng(seed)
    a = rng.standard_normal((size, size), dtype=np.float32)
    b = rng.standard_normal((size, size), dtype=np.float32)
    if rank > 0:
        a = np.random.default_rng(seed + 7919 * rank).standard_normal((size, size), dtype=np.float32)
    return a, b


def operand_digest(*arrays):
    """Short SHA-256 of the arrays' bytes (C order): identifies a set of operands."""
    import hashlib

    import numpy as np

    digest = hashlib.sha256()
    for array in arrays:
        digest.update(np.ascontiguousarray(array).tobytes())
    return digest.hexdigest()[:24]


def effects_label(effects):
    if effects == "ideal":
        return "ideal"
    return "nonideal: " + ", ".join(f"{name.replace('_variation', '')} {value}"
                                    for name, value in EFFECTS[effects].items() if name != "read_mode") + \
        (f", read mode {EFFECTS[effects]['read_mode']}" if "read_mode" in EFFECTS[effects] else "")


def workload(args, world, spec=None):
    import memfast_b200 as mf

    config, size, fmt, effects = spec or product_spec(mf, args)
    n = k = o = size
    strong = world > 1 and args.scaling == "strong"
    if world == 1:
        batch = f"one {n}-row batch on one GPU"
    elif strong:
        batch = (f"one {n}-row batch split into {world} row blocks of {n // world}, B replicated; the output "
                 f"rows all-gathered (NCCL, in place) into every rank's full output inside each step")
    else:
        batch = (f"{world} row blocks of {n}: one {n * world}-row batch, B replicated, "
                 + ("output rows all-gathered" if args.gather else "each rank keeps its output rows"))
    slices = list(config.input_slice or ())
    return dict(workload=f"Simulator.mm {n}x{k}x{o} {fmt} {tuple(slices)} {effects}"
                         + ("" if strong or world == 1 else " per GPU"),
                n=n * (world if world > 1 and not strong else 1), k=k, o=o, batch=batch,
                array=list(config.array_size), rows_per_read=config.read_rows,
                adc_bits=list(config.adc_bits) if isinstance(config.adc_bits, tuple) else config.adc_bits,
                input_groups=list(config.input_quant_gran), weight_groups=list(config.weight_quant_gran),
                operands="seeded N(0,1) fp32 (numpy PCG64, seed 2024)",
                l2=f"inputs 2x{4 * n * k / 2**20:.0f} MiB fp32; L2 (126 MB) flushed by a 256 MiB write "
                   f"before every timed step")


# ------------------------------------------------------------------ CPU leg --
class OracleSample:
    """The oracle (the reference CPU algorithm restated in C) on a row prefix.

    One call programs B (restores every conductance) and then runs the rows, as
    the reference's ``Simulator.mm`` does on every call.  The prefix is sized from
    two short timings so that one call takes about ``budget_s`` seconds.
    """

    def __init__(self, size, config, budget_s):
        from oracle import oracle as O

        self.O = O
        self.size, self.config = size, config
        self.threads = os.cpu_count() or 1
        O.set_threads(self.threads)
        O.lib()
        self.a, self.b = operands(size)
        # Rows run in parallel over the threads: time one and two rows per thread.
        t1 = self.time(self.threads)[0]
        t2 = self.time(2 * self.threads)[0]
        per_row = max((t2 - t1) / self.threads, 0.25 * t2 / self.threads)
        self.fixed = max(t1 - per_row * self.threads, 0.0)
        rows = int((budget_s - self.fixed) / per_row)
        self.rows = max(self.threads, min(size, rows - rows % self.threads))
        self.output = None

    def time(self, rows):
        start = time.perf_counter()
        out = self.O.mm(self.a[:rows], self.b, self.config, physical=True)
        return time.perf_counter() - start, out

    def run(self):
        """One timed call on the prefix; keeps its output (read event 0, matrix.0)."""
        elapsed, self.output = self.time(self.rows)
        return elapsed

    def rate(self, elapsed):
        return float(self.rows) * self.size * self.size / elapsed

    def describe(self, elapsed):
        return (f"oracle C restatement of the reference CPU algorithm (B programmed and every conductance "
                f"restored per call, physical FP32 currents, ADC, reconstruction, scale epilogue) on "
                f"{self.threads} threads; one call = the first {self.rows} of {self.size} rows against the full "
                f"{self.size}x{self.size} B ({elapsed:.1f} s, of which about {self.fixed:.2f} s is the per-call "
                f"programming of B)")


def cpu_sample(size, budget_s, config):
    sample = OracleSample(size, config, budget_s)
    elapsed = sample.run()
    extrapolated = sample.fixed + (elapsed - sample.fixed) * size / sample.rows
    return sample, dict(value=sample.rate(elapsed), unit=UNIT, cores=sample.threads, kind="port",
                        sample=sample.describe(elapsed), rows=sample.rows,
                        extrapolated_full_batch_s=extrapolated)


def parity_report(got, want, ideal, label):
    """Bit-exactness (ideal) or the element-error statistics (nonideal) of got vs want."""
    import numpy as np

    got = np.ascontiguousarray(got, np.float32)
    want = np.ascontiguousarray(want, np.float32)
    line = dict(rows=int(got.shape[0]), against=label)
    if ideal:
        line["bit_exact"] = bool(np.array_equal(got.view(np.uint32), want.view(np.uint32)))
        if not line["bit_exact"]:
            scale = float(max(np.abs(want).max(), 1e-30))
            line.update(mismatch_fraction=float(np.mean(got != want)),
                        max_err_of_range=float(np.abs(got.astype(np.float64) - want).max() / scale))
        return line
    diff = got.astype(np.float64) - want
    scale = float(max(np.abs(want).max(), 1e-30))
    line.update(mismatch_fraction=float(np.mean(diff != 0)), max_err_of_range=float(np.abs(diff).max() / scale),
                rms_err_of_range=float(np.sqrt(np.mean(diff**2)) / scale))
    return line


def reference_arm(args):
    import memfast_b200 as mf

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    if args.workload in ("resnet50", "llama7b"):
        # The reference's per-layer algorithm on one layer-shaped product of the model's
        # configuration (a whole forward of either model takes hours on the host).
        config, k, o = (resnet_config(mf), 576, 64) if args.workload == "resnet50" else (llama_config(mf), 4096, 512)
        sample = oracle_layer_sample(config, k, o, max(2.0, 150.0 / max(1, args.steps + args.warmup)))
        line = dict(metric=f"simulated MAC/s, {args.workload} layer sample", value=sample["value"], unit=UNIT,
                    n_gpus=args.gpus, steps=1, warmup=0, ms_per_step=None, higher_is_better=True,
                    scaling="strong", vs_baseline=None, dtype="f32 currents / int64 totals", data="synthetic",
                    config=dict(workload=f"{args.workload}: one layer-shaped product, oracle"), impl="reference",
                    cpu_baseline=sample, e2e=dict(value=sample["value"], unit=UNIT, h2d_bytes_per_step=0,
                                                  d2h_bytes_per_step=0))
        print(json.dumps(line), flush=True)
        return
    spec = product_spec(mf, args)
    config, size = spec[0], spec[1]
    budget = max(2.0, 150.0 / max(1, args.steps + args.warmup))
    sample = OracleSample(size, config, budget)
    rates, times = [], []
    for step in range(args.warmup + args.steps):
        elapsed = sample.run()
        if step >= args.warmup:
            rates.append(sample.rate(elapsed))
            times.append(elapsed)
    value = statistics.mean(rates)
    line = dict(metric=metric_name(size, spec[2]), value=value, unit=UNIT, n_gpus=args.gpus, steps=args.steps,
                warmup=args.warmup, ms_per_step=statistics.mean(times) * 1e3, higher_is_better=True,
                scaling=args.scaling if world > 1 else "strong", vs_baseline=None,
                dtype="f32 currents / int64 totals", data="synthetic", config=workload(args, 1, spec),
                impl="reference",
                cpu_baseline=dict(value=value, unit=UNIT, cores=sample.threads, kind="port",
                                  sample=sample.describe(statistics.mean(times)) + "; each step one such call"),
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
    from memfast_b200.sharding import gather_rows, peer_outputs, row_parallel_mm, row_range, sharded_mm

    spec = product_spec(mf, args)
    config, size = spec[0], spec[1]
    strong = world > 1 and args.scaling == "strong"
    if strong:
        a_np, b_np = operands(size)
        r0, r1 = row_range(size, world, rank)
        total_rows = size
        a_np = a_np[r0:r1]
    else:
        # Weak scaling: every rank owns `size` rows of a (size * world)-row batch; its rows
        # carry their global vector indices (noise addresses).
        a_np, b_np = operands(size, rank=rank)
        r0, r1 = rank * size, (rank + 1) * size
        total_rows = size * world
    rows = r1 - r0
    a_host = torch.from_numpy(a_np).contiguous().pin_memory()
    b_host = torch.from_numpy(b_np).contiguous().pin_memory()
    a = a_host.to(device)
    b = b_host.to(device)
    sim = mf.Simulator(config, device=device)
    gather = world > 1 and (strong or args.gather)
    full = torch.empty((total_rows, size), device=device) if gather else None
    own = full[r0:r1] if (gather and strong) else None
    # Strong scaling with --exchange peers: the kernel stores its rows into every rank's
    # copy of the output over NVLink (peer stores) instead of an all-gather after it.
    peers = peer_outputs(full) if strong and args.exchange == "peers" else None
    out_host = torch.empty((rows, size), pin_memory=True)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    def step():
        # Strong scaling: this rank's rows with global vector indices, written straight
        # into its rows of the full output, and the in-place all-gather enqueued before
        # the call's one host synchronisation.  Weak scaling: each rank's own product.
        if world == 1:
            return sim.mm(a, b)
        if strong:
            return row_parallel_mm(a, b, simulator=sim, row_offset=r0, rows=total_rows, out=full, peers=peers)
        out = sharded_mm(a, b, simulator=sim, row_offset=r0)
        if gather:
            return gather_rows(out, total_rows, out=full)
        return out

    def timed(fn, count, barrier=True):
        times = []
        for _ in range(count):
            flush.zero_()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if world > 1 and barrier:
                dist.barrier()
            torch.cuda.synchronize(device)
            start.record(stream)
            fn()
            end.record(stream)
            torch.cuda.synchronize(device)
            times.append(start.elapsed_time(end) / 1e3)
        return times

    # The first call (read event 0) is the one the parity check reads.
    first = step()
    torch.cuda.synchronize(device)
    check_rows = first[:min(first.shape[0], 4096)].cpu() if rank == 0 else None
    for _ in range(max(0, args.warmup - 1)):
        step()
    torch.cuda.synchronize(device)
    def reduce_max(value):
        if world == 1:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    launches0 = _lib.load().mf_launch_count()
    with ClockSampler(local) as clocks:
        t_wall = time.perf_counter()
        times = timed(step, args.steps)
        launches = _lib.load().mf_launch_count() - launches0
        # Keep the GPU loaded for about a second in all for the clock sampler (not part
        # of the measurement); every rank runs the same number of steps (collectives).
        left = 1.0 - (time.perf_counter() - t_wall)
        extra = int(reduce_max(max(0, int(left / max(min(times), 1e-4)) + 1) if left > 0 else 0))
        for _ in range(extra):
            step()
        torch.cuda.synchronize(device)
    per_step = sum(times) / len(times)

    # End to end through the host-operand API: pinned A rows and B copied in and the
    # product rows copied out every step, overlapped chunk by chunk with the compute.
    from memfast_b200.streaming import host_mm

    def e2e_step():
        host_mm(a_host, b_host, simulator=sim, out=out_host, row_offset=r0)
        if world > 1 and args.gather and not strong:
            gather_rows(out_host.to(device), total_rows)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    e2e_times = timed(e2e_step, args.steps)
    e2e_step_s = sum(e2e_times) / len(e2e_times)

    # Dominant kernel alone: one mf_sliced_mm call on pre-quantised operands with a
    # preallocated workspace and output (no Python work inside the timed region).
    import ctypes as ct

    from memfast_b200.quantization import input_tiles
    from memfast_b200.simulator import check_device_error, default_schedule

    matrix = sim._matrix_for(b)
    q, xscale = input_tiles(a, config)
    schedule = dict(default_schedule(config), kernel=args.kernel)
    n_rows = q.shape[0]
    ws_bytes = matrix._workspace_size(n_rows, schedule)
    workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=device)
    # Wide configurations (BFP, more than 8 bits) reconstruct and write FP64 outputs.
    out_k = torch.empty((n_rows, size), device=device, dtype=torch.float64 if config.wide else torch.float32)
    native = _lib.schedule(**schedule)
    lib = _lib.load()
    cfg = _lib.native_config(config)

    def sliced_mm():
        _lib.check(lib.mf_sliced_mm(
            cfg, ct.byref(native), _lib.ptr(q), _lib.ptr(xscale), _lib.ptr(matrix.packed),
            _lib.ptr(matrix.weight_scale), None, _lib.ptr(out_k), n_rows, matrix.packed.shape[0], matrix.p,
            size, size, 0, matrix.p, matrix.seed & 0xFFFFFFFF, 0, r0, 0, _lib.ptr(workspace), ws_bytes,
            _lib.stream_of(device)), "mf_sliced_mm")

    for _ in range(2):
        sliced_mm()
    kernel_times = timed(sliced_mm, max(3, args.steps), barrier=False)
    kernel_s = sum(kernel_times) / len(kernel_times)
    gather_s = 0.0
    if gather:
        source = own if own is not None else torch.zeros((rows, size), device=device)
        gather_times = timed(lambda: gather_rows(source, total_rows, out=full), max(3, args.steps))
        gather_s = sum(gather_times) / len(gather_times)
    check_device_error()   # a bounded device-side wait that gave up invalidates the timing

    per_step = reduce_max(per_step)
    e2e_step_s = reduce_max(e2e_step_s)
    kernel_s = reduce_max(kernel_s)
    gather_s = reduce_max(gather_s)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    macs = float(total_rows) * size * size
    pairs = len(config.input_layout) * len(config.weight_layout)
    bf16, hbm, peak_kind = measured_peaks()
    ideal = config.nonidealities.ideal
    kernel_path = _lib.PATHS[lib.mf_last_path()]
    # Ideal: int8 digit MMAs against the int8 dense rate (2 x bf16).  Nonideal: FP16 digit x
    # conductance MMAs against the f16 dense rate (= bf16); each current's two FP16 halves
    # double the issued MMA work over this algorithmic count.
    peak_tops = 2.0 * bf16 if ideal else bf16
    kernel_ops = 2.0 * (rows * size * size) * pairs
    achieved_tops = kernel_ops / kernel_s / 1e12
    traffic = profiled_traffic() if ideal and rows == size else None
    path = {"packed": "the packed tcgen05 kernel plus its K-major weight copy and rare-tile filter launch",
            "fp8_planes": "the FP8 digit-plane tcgen05 kernel plus its K-major weight copy",
            "tc_currents": "the conductance-operand build and the tcgen05 current kernel",
            "simt_currents": "the conductance restore and the SIMT FP32 current kernel (no tensor cores)",
            "generic_ideal": "the dp4a SIMT digit kernel (no tensor cores)"}[kernel_path]
    line = dict(
        metric=metric_name(size, spec[2]), value=macs / per_step, unit=UNIT, n_gpus=world, steps=args.steps,
        warmup=args.warmup, ms_per_step=per_step * 1e3, higher_is_better=True,
        scaling="strong" if world == 1 or strong else "weak", vs_baseline=None,
        dtype="u8 digits / int32 totals / f32 epilogue" if ideal else
              "f16 digits x f16 conductance halves / f32 currents, ADC and epilogue",
        data="synthetic", config=workload(args, world, spec),
        slice_pair_macs_per_s=macs * pairs / per_step,
        roofline=dict(bound="tensor", achieved=achieved_tops, peak=peak_tops, unit="TFLOP/s",
                      frac=achieved_tops / peak_tops, traffic=traffic,
                      kernel_path=kernel_path,
                      note=f"one mf_sliced_mm call per rank (schedule kernel {args.kernel}: {path}), "
                           f"{rows}x{size}x{size}; algorithmic {pairs} slice-pair MAC streams x2 ops; peak = "
                           + (f"2 x {peak_kind} dense bf16 ({bf16} TFLOP/s), the int8 dense rate of B200" if ideal
                              else f"{peak_kind} dense bf16 ({bf16} TFLOP/s), the f16 dense rate of B200"),
                      kernel_ms=kernel_s * 1e3),
        e2e=dict(value=macs / e2e_step_s, unit=UNIT,
                 h2d_bytes_per_step=int((total_rows * size + size * size * world) * 4),
                 d2h_bytes_per_step=int(total_rows * size * 4), ms_per_step=e2e_step_s * 1e3,
                 note="streaming.host_mm per rank: its rows of A and all of B from pinned host memory, its "
                      "output rows back to pinned host memory"),
        gpu_launches=int(launches),
        clocks=clocks.summary(),
    )
    if world > 1:
        line["breakdown"] = dict(
            step_ms=per_step * 1e3, kernel_ms=kernel_s * 1e3, gather_ms=gather_s * 1e3,
            rest_ms=max(0.0, per_step - kernel_s - (0.0 if peers is not None and peers.enabled else gather_s)) * 1e3,
            output_exchange="peer stores from the packed kernel's epilogue over NVLink" if peers is not None
                            and peers.enabled else "in-place NCCL all-gather",
            note="max over ranks of each part timed alone: the rank's mf_sliced_mm launch (no peer stores), the "
                 "in-place NCCL all-gather of the output rows (which the step replaces by peer stores when "
                 "output_exchange says so), and the step's remainder")
    oracle_rows = None
    if world == 1 and not args.skip_cpu:
        sample, line["cpu_baseline"] = cpu_sample(size, args.cpu_seconds, config)
        oracle_rows = sample.output
    if oracle_rows is None:
        from oracle import oracle as O

        a_full, b_full = operands(size)
        oracle_rows = O.mm(a_full[:args.parity_rows], b_full, config)
    got = check_rows[:oracle_rows.shape[0]].numpy()
    line["parity"] = parity_report(got, oracle_rows, ideal, "oracle (reference CPU algorithm), read event 0")
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- model arms --
def resnet_config(mf_module):
    """INT8 (1,1,2,2,2) slices, 7-bit ADCs, write variation 0.02; the
    rest (64x64 arrays, whole-array reads, per-vector input groups) are Config's defaults."""
    return mf_module.Config(input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=7,
                            nonidealities=mf_module.Nonidealities(write_variation=0.02))


def llama_config(mf_module):
    """INT8 (1,1,2,2,2) slices, ADC bits (6,7,7,8,8), dynamic input
    quantisation; everything else (including write variation 0.02) is Config's default."""
    return mf_module.Config(input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=(6, 7, 7, 8, 8))


def analog_macs(model, run):
    """MACs of every analog layer in one ``run()`` (counted by forward hooks)."""
    from memfast_b200.nn import AnalogConv2d
    from memfast_b200.simulator import AnalogMatrix

    total = [0]

    def conv_hook(module, inputs, output):
        per_output = module.in_channels // module.groups * module.kernel_size[0] * module.kernel_size[1]
        total[0] += output.numel() * per_output

    def matrix_hook(module, inputs, output):
        total[0] += inputs[0].numel() // module.in_features * module.in_features * module.out_features

    handles = []
    for module in model.modules():
        if isinstance(module, AnalogConv2d):
            handles.append(module.register_forward_hook(conv_hook))
        elif isinstance(module, AnalogMatrix) and not any(
                isinstance(parent, AnalogConv2d) and module in parent.modules() for parent in model.modules()):
            handles.append(module.register_forward_hook(matrix_hook))
    try:
        run()
    finally:
        for handle in handles:
            handle.remove()
    return total[0]


def oracle_layer_sample(config, k, o, budget_s, seed=11):
    """cpu_baseline of a model line: the oracle on a row prefix of one [rows, k] x [k, o]
    product of the model's configuration (its layers run the same per-row algorithm)."""
    from oracle import oracle as O

    threads = os.cpu_count() or 1
    O.set_threads(threads)
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((4 * threads, k), dtype=np.float32)
    b = rng.standard_normal((k, o), dtype=np.float32)
    start = time.perf_counter()
    O.mm(a[:threads], b, config, physical=True)
    t1 = time.perf_counter() - start
    rows = int(max(threads, min(4 * threads, budget_s / max(t1, 1e-3) * threads)))
    start = time.perf_counter()
    O.mm(a[:rows], b, config, physical=True)
    elapsed = time.perf_counter() - start
    return dict(value=rows * k * o / elapsed, unit=UNIT, cores=threads, kind="port",
                sample=f"oracle C restatement of the reference CPU algorithm on {threads} threads: {rows} rows of a "
                       f"[rows, {k}] x [{k}, {o}] product of the model's configuration ({elapsed:.1f} s, B programmed "
                       f"per call as the reference does)")


class ModelRun:
    """Shared plumbing of the model lines: process group, timing, clocks, max over ranks."""

    def __init__(self, args):
        import torch
        import torch.distributed as dist

        self.torch, self.dist, self.args = torch, dist, args
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != args.gpus:
            raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={self.world}")
        torch.cuda.set_device(self.local)
        self.device = torch.device("cuda", self.local)
        if self.world > 1:
            import datetime

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=self.device)

    def timed(self, fn, count):
        torch, dist = self.torch, self.dist
        stream = torch.cuda.current_stream(self.device)
        times = []
        for _ in range(count):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if self.world > 1:
                dist.barrier()
            torch.cuda.synchronize(self.device)
            start.record(stream)
            fn()
            end.record(stream)
            torch.cuda.synchronize(self.device)
            times.append(start.elapsed_time(end) / 1e3)
        return times

    def reduce_max(self, value):
        if self.world == 1:
            return value
        t = self.torch.tensor([value], dtype=self.torch.float64, device=self.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def measure(self, step):
        from memfast_b200 import _lib

        for _ in range(self.args.warmup):
            step()
        self.torch.cuda.synchronize(self.device)
        launches0 = _lib.load().mf_launch_count()
        with ClockSampler(self.local) as clocks:
            times = self.timed(step, self.args.steps)
        launches = _lib.load().mf_launch_count() - launches0
        return self.reduce_max(sum(times) / len(times)), launches, clocks.summary()

    def close(self):
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


def resnet_arm(args):
    """ResNet-50 (torchvision architecture, Kaiming-init random weights) converted with
    convert_model, forward on 256 synthetic 3x224x224 images; with N GPUs the batch is
    split into N data-parallel shards (each rank converts its own model copy with the same
    seeds) and the logits are all-gathered inside every step."""
    import torch
    import torchvision

    import memfast_b200 as mf
    from memfast_b200.sharding import gather_rows, row_range

    run = ModelRun(args)
    config = resnet_config(mf)
    batch = 256
    r0, r1 = row_range(batch, run.world, run.rank)
    images = np.random.default_rng(2024).standard_normal((batch, 3, 224, 224), dtype=np.float32)
    x = torch.from_numpy(images[r0:r1]).to(run.device)
    torch.manual_seed(0)
    model = torchvision.models.resnet50(weights=None)
    conv1_weight = model.conv1.weight.detach().numpy().copy()
    sim = mf.Simulator(config, device=run.device)
    analog = mf.convert_model(model, sim)
    logits = torch.empty((batch, 1000), device=run.device)

    # Parity (rank 0): the first analog layer on the first image against the oracle.
    conv1 = analog.conv1
    first = conv1(x[:1]).cpu().numpy()
    mf.reset_read_events(analog)

    def step():
        with torch.no_grad():
            out = analog(x)
        if run.world > 1:
            gather_rows(out, batch, out=logits)

    macs_local = analog_macs(analog, lambda: analog(x))
    macs = run.reduce_max(macs_local) * batch / max(1, r1 - r0) if run.world > 1 else macs_local
    per_step, launches, clocks = run.measure(step)
    run.close()
    if run.rank != 0:
        return
    from oracle import oracle as O

    want = O.conv2d(images[:1], conv1_weight, None, config, stride=(2, 2), padding=(3, 3), dilation=(1, 1), groups=1,
                    name="conv1")
    line = dict(
        metric="simulated MAC/s of a ResNet-50 forward, batch 256 x 3 x 224 x 224, converted with convert_model",
        value=macs / per_step, unit=UNIT, n_gpus=run.world, steps=args.steps, warmup=args.warmup,
        ms_per_step=per_step * 1e3, higher_is_better=True, scaling="strong", vs_baseline=None,
        dtype="f16 digits x f16 conductance halves / f32 currents, ADC and epilogue (analog layers); f32 digital",
        data="synthetic", images_per_s=batch / per_step, analog_macs_per_forward=macs,
        config=dict(workload="ResNet-50 forward (BASELINE configs[3])", batch=batch, image=[3, 224, 224],
                    model="torchvision resnet50, weights=None (Kaiming init), seed 0",
                    analog="every Conv2d and Linear: INT8 (1,1,2,2,2), adc 7, write variation 0.02, array 64x64, "
                           "64-row reads, per-vector input groups",
                    parallelism=f"data parallel x{run.world}: {batch // run.world} images per rank, logits "
                                "all-gathered every step; each rank's vectors are indexed from its own first image"),
        gpu_launches=int(launches), clocks=clocks,
        parity=parity_report(first.reshape(-1), want.reshape(-1), False, "oracle conv2d of conv1 on image 0, event 0"),
    )
    if run.world == 1 and not args.skip_cpu:
        line["cpu_baseline"] = oracle_layer_sample(config, 576, 64, args.cpu_seconds)
    print(json.dumps(line), flush=True)


def build_llama(torch, device, layers=32):
    """Llama-2-7B architecture with random N(0, 0.02) weights, built straight on the device."""
    from transformers import LlamaConfig, LlamaForCausalLM
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    cfg = LlamaConfig(vocab_size=32000, hidden_size=4096, intermediate_size=11008, num_hidden_layers=layers,
                      num_attention_heads=32, num_key_value_heads=32, max_position_embeddings=4096,
                      rms_norm_eps=1e-5, tie_word_embeddings=False)
    cfg._attn_implementation = "sdpa"
    with torch.device("meta"):
        model = LlamaForCausalLM(cfg)
    model.to_empty(device=device)
    generator = torch.Generator(device).manual_seed(2024)
    with torch.no_grad():
        for parameter in model.parameters():
            if parameter.ndim == 2:
                parameter.normal_(0.0, 0.02, generator=generator)
            else:
                parameter.fill_(1.0)   # RMSNorm gains
    model.model.rotary_emb = LlamaRotaryEmbedding(cfg, device=device)
    return model.eval()


def llama_arm(args):
    """Llama-2-7B architecture forward on 8 x 512 uniform-random token ids with every
    nn.Linear analog; with N GPUs every AnalogLinear is column-sharded over the ranks
    (sharding.tensor_parallel) and its output tiles all-gathered over NCCL."""
    import torch

    import memfast_b200 as mf
    from memfast_b200.sharding import tensor_parallel

    run = ModelRun(args)
    config = llama_config(mf)
    layers = args.llama_layers
    model = build_llama(torch, run.device, layers)
    probe_weight = model.model.layers[0].self_attn.q_proj.weight.detach().clone()
    sim = mf.Simulator(config, device=run.device)
    analog = mf.convert_model(model, sim, inplace=True)
    if run.world > 1:
        tensor_parallel(analog)
    tokens = torch.from_numpy(np.random.default_rng(2024).integers(0, 32000, (8, 512))).to(run.device)

    # Parity (rank 0): q_proj of layer 0 on a few hidden vectors against the oracle.
    q_proj = analog.model.layers[0].self_attn.q_proj
    probe = torch.from_numpy(np.random.default_rng(7).standard_normal((16, 4096), dtype=np.float32)).to(run.device)
    got = q_proj(probe).cpu().numpy()
    mf.reset_read_events(analog)

    def step():
        with torch.no_grad():
            analog(input_ids=tokens, use_cache=False)

    macs = analog_macs(analog, step)
    mf.reset_read_events(analog)
    per_step, launches, clocks = run.measure(step)
    run.close()
    if run.rank != 0:
        return
    from oracle import oracle as O

    want = O.linear(probe.cpu().numpy(), probe_weight.cpu().numpy(), None, config,
                    name="model.layers.0.self_attn.q_proj")
    tokens_n = 8 * 512
    line = dict(
        metric="simulated MAC/s of a Llama-2-7B-architecture forward, batch 8 x 512 tokens, every nn.Linear analog",
        value=macs / per_step, unit=UNIT, n_gpus=run.world, steps=args.steps, warmup=args.warmup,
        ms_per_step=per_step * 1e3, higher_is_better=True, scaling="strong", vs_baseline=None,
        dtype="f16 digits x f16 conductance halves / f32 currents, ADC and epilogue (analog linears); f32 digital",
        data="synthetic", tokens_per_s=tokens_n / per_step, analog_macs_per_forward=macs,
        config=dict(workload="Llama-2-7B-architecture forward (BASELINE configs[4])", batch=8, seq_len=512,
                    layers=layers, model="transformers LlamaForCausalLM (d 4096, 32 heads, SwiGLU 11008, vocab 32000), "
                                         "random N(0, 0.02) weights",
                    analog="every nn.Linear including lm_head: INT8 (1,1,2,2,2), adc (6,7,7,8,8), write variation "
                           "0.02 (Config default), array 64x64, 64-row reads, dynamic per-vector input groups",
                    parallelism=(f"tensor parallel x{run.world}: every AnalogLinear column-sharded by output tiles, "
                                 "NCCL all-gather of the column slabs" if run.world > 1 else "one GPU")),
        gpu_launches=int(launches), clocks=clocks,
        parity=parity_report(got, want, False, "oracle q_proj of layer 0 on 16 vectors, event 0"),
    )
    if run.world == 1 and not args.skip_cpu:
        line["cpu_baseline"] = oracle_layer_sample(config, 4096, 512, args.cpu_seconds)
    print(json.dumps(line), flush=True)


def reference_cuda_arm(args):
    """The reference's own GPU path on the same operands: ``Simulator(cfg, device="cuda").mm``
    of the unmodified reference package (NVRTC-compiled SIMT kernels, default schedule,
    memfast/cuda.py:322-373), installed from the reference sources into baseline/_ref.
    Rank 0 only; prints ``unavailable`` when the package is not installed."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    package = ROOT / "baseline" / "_ref"
    if not (package / "memfast" / "__init__.py").exists():
        print(json.dumps(dict(impl="reference-cuda", unavailable="reference package not installed in baseline/_ref")))
        return
    import torch

    sys.path.insert(0, str(package))
    import memfast as ref

    if args.workload != "sweep":
        raise SystemExit("--impl reference-cuda times the sweep workload")
    config = bench_config(ref, args.effects)
    a_np, b_np = operands(args.size)
    a, b = torch.from_numpy(a_np).cuda(), torch.from_numpy(b_np).cuda()
    sim = ref.Simulator(config, device="cuda")
    for _ in range(max(1, args.warmup)):
        first = sim.mm(a, b)
    torch.cuda.synchronize()
    times = []
    with ClockSampler(0) as clocks:
        for _ in range(args.steps):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            sim.mm(a, b)
            end.record()
            torch.cuda.synchronize()
            times.append(start.elapsed_time(end) / 1e3)
    per_step = sum(times) / len(times)
    size = args.size
    line = dict(metric=metric_name(size), value=float(size) ** 3 / per_step, unit=UNIT, n_gpus=1, steps=args.steps,
                warmup=args.warmup, ms_per_step=per_step * 1e3, higher_is_better=True, scaling="strong",
                vs_baseline=None, dtype="f32 currents / int64 totals (reference SIMT kernels)", data="synthetic",
                config=workload(args, 1, (config, size, "INT8", effects_label(args.effects))),
                impl="reference-cuda", clocks=clocks.summary(),
                note="unmodified reference memfast 0.3.0 from baseline/_ref, Simulator(device='cuda').mm, default "
                     "mode: B reprogrammed per call, restore + consume NVRTC kernels per tile group, partials "
                     "scaled and summed in PyTorch")
    # Its rows against the oracle, as the engine's line does.
    from oracle import oracle as O

    rows = args.parity_rows
    line["parity"] = parity_report(first[:rows].cpu().numpy(), O.mm(a_np[:rows], b_np, config),
                                   args.effects == "ideal", "oracle (reference CPU algorithm)")
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
    elif args.impl == "reference-cuda":
        reference_cuda_arm(args)
    elif args.workload == "resnet50":
        resnet_arm(args)
    elif args.workload == "llama7b":
        llama_arm(args)
    else:
        engine_arm(args)


if __name__ == "__main__":
    main()
