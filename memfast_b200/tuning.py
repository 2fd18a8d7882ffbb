"""Tuned mode: per-shape schedule selection over this engine's declared grid.

User-visible behaviour follows the reference's tuned mode
(memfast/simulator.py:27-45 and 195-347, docs/user-guide.md:464-478):

* the first call of a programmed matrix for an input shape and dtype computes
  the output of the default schedule, the reference that every candidate must
  reproduce bit for bit;
* a winner saved by an earlier process (one JSON file per key: the hash of the
  configuration, the device, the shape, the engine's source fingerprint and
  the grid) is used after a bitwise re-check, without timing anything;
* otherwise every candidate that ``mf_query`` admits and that fits the
  simulator's workspace budget runs once for the bitwise check and once under
  CUDA events, the fastest is kept, and the file is written atomically;
* ``Simulator.report()`` lists each selection with its candidates.

What differs is the grid.  The reference enumerates thread shapes of its SIMT
kernel (arrays x vectors x columns x workers).  This engine's axes are the
choices its sm_100a kernels take at run time:

* ``kernel``: 1 = SIMT (dp4a digit dots, or restored-conductance FP32
  currents), 2 = tcgen05 (packed integer counts, or FP16 digit x conductance
  currents), 3 = tcgen05 FP8 digit planes (ideal 8-bit configurations);
* ``raster``: the order in which the tensor-core kernels launch their
  128-vector x column-block CTAs (vector blocks first or column blocks first,
  which decides which operand the CTAs in flight share through L2);
* ``arrays``: output tiles whose conductances the SIMT current kernels
  restore per group (workspace size against launch count).

The schedule's ``tile_n``/``tile_o`` fields are kept for the ABI but no kernel
reads them, so they are not axes.

Each candidate is reduced to the execution it resolves to (``mf_query``'s
path plus the axes that path reads), so equivalent schedules run once.  For
ideal devices every path is bit-identical; for nonideal devices the SIMT and
tensor-core currents sum in different orders, so the bitwise check keeps only
schedules of the default's path.
"""

import ctypes as ct
import hashlib
import itertools
import json
import os
import tempfile
import time
from dataclasses import asdict
from pathlib import Path

import torch

from . import _lib

KERNELS = (1, 2, 3)
RASTERS = (0, 1)
ARRAYS = (1, 2, 4, 8, 16, 32, 64)

# Axes each kernel family reads (the others do not change its execution).
_PATH_AXES = {
    "generic_ideal": (),
    "simt_currents": ("arrays",),
    "packed": ("raster",),
    "fp8_planes": ("raster",),
    "tc_currents": ("raster",),
}


def default_schedule(config):
    """Schedule used outside tuned mode: kernel 0 lets the library choose."""
    return dict(kernel=0, tile_n=32, tile_o=64, arrays=2, raster=0)


def declared_grid():
    """The grid's axes and values (part of the cache key)."""
    return dict(kernel=list(KERNELS), raster=list(RASTERS), arrays=list(ARRAYS))


def resolve(config, schedule, n, m, p):
    """(path name, resources) that ``schedule`` runs as for an n x (m arrays) x (p tiles) product."""
    resources = _lib.MFResources()
    native = _lib.schedule(**schedule)
    _lib.check(_lib.load().mf_query(_lib.native_config(config), ct.byref(native), n, m, p, ct.byref(resources)),
               "mf_query")
    return _lib.PATHS[resources.path], resources


def schedule_grid(config, n, partitions, m=1):
    """Every distinct execution of the declared grid for this product, in a fixed order."""
    seen = set()
    for kernel, raster, arrays in itertools.product(KERNELS, RASTERS, ARRAYS):
        # More restore groups than output tiles act as one group per tile.
        candidate = dict(kernel=kernel, tile_n=32, tile_o=64, arrays=min(arrays, partitions), raster=raster)
        path, _ = resolve(config, candidate, max(n, 1), m, partitions)
        identity = (path,) + tuple(candidate[axis] for axis in _PATH_AXES[path])
        if identity in seen:
            continue
        seen.add(identity)
        yield candidate


def cache_root():
    base = os.environ.get("MEMFAST_CACHE_DIR")
    if base:
        return Path(base).expanduser()
    return Path(os.environ.get("XDG_CACHE_HOME", Path.home() / ".cache")) / "memfast_b200"


def atomic_write(path, content):
    """Write bytes to ``path`` through a temporary file in the same directory and a rename."""
    path.parent.mkdir(parents=True, exist_ok=True)
    handle, name = tempfile.mkstemp(dir=path.parent, prefix=path.name, suffix=".tmp")
    try:
        with os.fdopen(handle, "wb") as stream:
            stream.write(content)
        os.replace(name, path)
    except BaseException:
        Path(name).unlink(missing_ok=True)
        raise


def source_hash():
    """Fingerprint of the engine: its Python and CUDA sources."""
    root = Path(__file__).parent
    digest = hashlib.sha256()
    for path in sorted([*root.rglob("*.py"), *root.rglob("*.cu"), *root.rglob("*.cuh")]):
        if "_build" in path.parts:
            continue
        digest.update(path.relative_to(root).as_posix().encode())
        digest.update(path.read_bytes())
    return digest.hexdigest()


def device_identity(device):
    properties = torch.cuda.get_device_properties(device)
    return dict(name=properties.name, capability=list(torch.cuda.get_device_capability(device)),
                multiprocessors=properties.multi_processor_count, memory=properties.total_memory,
                torch=torch.__version__, cuda=torch.version.cuda)


def _bits(tensor):
    return tensor.view(torch.int32 if tensor.dtype == torch.float32 else torch.int64)


class Search:
    """One tuned-mode selection: a programmed matrix, one input shape and dtype."""

    def __init__(self, simulator, matrix, shape, dtype, q, xscale, event):
        self.simulator, self.matrix = simulator, matrix
        self.shape, self.dtype = tuple(shape), dtype
        self.q, self.xscale, self.event = q, xscale, event
        self.started = time.perf_counter()
        self.fingerprint = json.loads(json.dumps(dict(
            config=asdict(simulator.config), hardware=device_identity(simulator.device), shape=list(self.shape),
            output=matrix.out_features, dtype=str(dtype), sources=simulator._fingerprint,
            workspace_bytes=simulator.workspace_bytes, grid=declared_grid())))
        self.key = hashlib.sha256(json.dumps(self.fingerprint, sort_keys=True).encode()).hexdigest()
        self.path = simulator.cache_dir / f"{self.key}.json"
        self.domain = list(schedule_grid(simulator.config, q.shape[0], matrix.p, q.shape[1]))
        self.record = dict(key=self.key, layer=matrix.name, shape=list(self.shape), cache_hit=False, candidates=[],
                           selected=None, complete=False)

    # -- pieces
    def admit(self, schedule):
        """Resources of ``schedule``, or ResourceError when it cannot run within the budget."""
        n, m = self.q.shape[0], self.q.shape[1]
        _, resources = resolve(self.simulator.config, schedule, n, m, self.matrix.p)
        need = self.matrix._workspace_size(n, schedule)
        if need > self.simulator.workspace_bytes:
            raise _lib.ResourceError("workspace budget")
        return dict(workspace_bytes=need, threads=resources.threads)

    def run(self, schedule):
        return self.matrix._execute(self.q, self.xscale, schedule, self.event)

    def reference_output(self, default):
        """The default schedule's output (the first admitted schedule when it does not fit)."""
        for schedule in [default, *self.domain]:
            try:
                self.admit(schedule)
                output = self.run(schedule)
            except (_lib.ResourceError, torch.cuda.OutOfMemoryError):
                torch.cuda.empty_cache()
                continue
            if not torch.isfinite(output).all():
                raise FloatingPointError("nonfinite default output during tuning")
            return _bits(output)
        raise RuntimeError("no feasible reference schedule in the declared grid")

    def saved_winner(self):
        """The schedule stored under this key by an earlier process, if the file is valid."""
        try:
            content = json.loads(self.path.read_text(encoding="utf-8"))
        except (OSError, ValueError):
            return None
        if not isinstance(content, dict) or content.get("fingerprint") != self.fingerprint:
            return None
        winner = content.get("selected")
        return winner if content.get("complete") is True and winner in self.domain else None

    def measure(self, schedule, reference):
        """Admit, check bit for bit, time one run; the candidate's report entry.

        Ideal devices: every schedule must reproduce the default bit for bit, and one
        that does not is an engine fault (RuntimeError, as in the reference).
        Nonideal devices: the SIMT and tensor-core currents sum in different orders,
        so a schedule of another path may round an ADC count differently; it is
        rejected and the search goes on."""
        entry = dict(schedule=schedule, status="rejected", timed_samples=0)
        try:
            entry["resources"] = self.admit(schedule)
            if not torch.equal(self.run(schedule).view(reference.dtype), reference):
                if self.simulator.config.nonidealities.ideal:
                    raise RuntimeError("schedule changes output")
                entry["reason"] = "output differs from the default schedule (another current summation order)"
                return entry
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            self.run(schedule)
            end.record()
            end.synchronize()
            entry.update(status="accepted", seconds=start.elapsed_time(end) / 1e3, timed_samples=1)
        except _lib.ResourceError as error:
            entry["reason"] = str(error)
        except torch.cuda.OutOfMemoryError:
            entry["reason"] = "CUDA out of memory"
            torch.cuda.empty_cache()
        return entry

    def finish(self, schedule, **fields):
        self.record.update(selected=schedule, complete=True,
                           preparation_seconds=time.perf_counter() - self.started, **fields)
        self.simulator._selections[self.key] = schedule
        return schedule

    # -- the selection
    def select(self, default):
        reference = self.reference_output(default)
        self.simulator.records.append(self.record)
        known = self.simulator._selections.get(self.key) or self.saved_winner()
        if known is not None:
            try:
                self.admit(known)
                if not torch.equal(self.run(known).view(reference.dtype), reference):
                    raise RuntimeError("cached schedule changes output")
                return self.finish(known, cache_hit=True)
            except (_lib.ResourceError, torch.cuda.OutOfMemoryError):
                torch.cuda.empty_cache()
        entries = [self.measure(schedule, reference) for schedule in self.domain]
        self.record["candidates"] = entries
        timed = [entry for entry in entries if entry["status"] == "accepted"]
        if not timed:
            raise RuntimeError("no feasible schedule in the declared grid")
        winner = min(timed, key=lambda entry: entry["seconds"])["schedule"]
        atomic_write(self.path, json.dumps(dict(fingerprint=self.fingerprint, complete=True, selected=winner,
                                                candidates=entries), sort_keys=True).encode())
        return self.finish(winner, domain_count=len(self.domain))


__all__ = ["default_schedule", "schedule_grid", "declared_grid", "resolve", "Search", "cache_root", "source_hash",
           "atomic_write", "device_identity"]
