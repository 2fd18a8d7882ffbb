"""Build libmemfast_b200.so in-tree with nvcc for sm_100a (B200).

    python -m memfast_b200.build          # or: python memfast_b200/build.py

The library is a plain shared object with a C ABI (include/memfast_b200.h); it
is loaded with ctypes, so the build needs nvcc and the CUDA runtime only.
"""

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
LIBRARY = PACKAGE / "libmemfast_b200.so"
SOURCES = ["capi.cu", "quantize.cu", "generic.cu", "tc_common.cu", "tc_ideal.cu", "tc_packed.cu",
           "tc_physical.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build memfast_b200")


def _stale():
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    inputs = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + [ROOT / "include" / "memfast_b200.h"]
    return any(p.stat().st_mtime > built for p in inputs if p.exists())


def build(force=False, verbose=False):
    if not force and not _stale():
        return LIBRARY
    compiler = nvcc()
    objects = []
    build_dir = PACKAGE / "_build"
    build_dir.mkdir(exist_ok=True)
    procs = []
    for source in SOURCES:
        obj = build_dir / (Path(source).stem + ".o")
        cmd = [
            compiler, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-fmad=false",
            "-Xcompiler", "-fPIC", "-Xptxas", "-warn-spills",
            "-I", str(ROOT / "include"), "-I", str(CSRC),
            "-c", str(CSRC / source), "-o", str(obj),
        ]
        objects.append(obj)
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failed = False
    for cmd, proc in procs:
        out, _ = proc.communicate()
        if verbose or proc.returncode:
            sys.stderr.write(" ".join(cmd) + "\n" + out)
        failed |= proc.returncode != 0
    if failed:
        raise RuntimeError("nvcc failed while building memfast_b200")
    tmp = LIBRARY.with_suffix(".so.tmp")
    link = [compiler, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objects)]
    subprocess.run(link, check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIBRARY)
