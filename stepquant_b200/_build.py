"""Build libstepquant_b200.so in-tree with nvcc for sm_100a.

``python -m stepquant_b200._build`` (or ``__graft_entry__.build()``) compiles
every CUDA source under ``csrc/`` into ``stepquant_b200/_lib/``.  The build is
skipped when the library is newer than every source and header.
"""
import os
import shutil
import subprocess
import sys

PACKAGE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PACKAGE)
CSRC = os.path.join(PACKAGE, "csrc")
LIBDIR = os.path.join(PACKAGE, "_lib")
LIBRARY = os.path.join(LIBDIR, "libstepquant_b200.so")
HEADER = os.path.join(ROOT, "include", "stepquant_b200.h")
SOURCES = ["sq_abi.cu", "sq_tile.cu", "sq_fast.cu", "sq_pack.cu", "sq_fp32.cu", "sq_noalloc.cu", "sq_prefill.cu",
           "sq_fast_kda.cu", "sq_streams.cu", "sq_fast_two.cu", "sq_prefill_kda.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-diag-suppress", "128",
    "-Xcompiler", "-fPIC",
]
# The quantizer must not contract a*b+c into FMAs (bit-exactness with the
# reference fit_state; intended FMAs are written as fmaf()).  The chunked
# prefill passes are toleranced and are built with contraction.
CONTRACT = {"sq_prefill.cu", "sq_prefill_kda.cu"}


def _nvcc():
    for candidate in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and os.path.exists(candidate):
            return candidate
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build stepquant_b200")


def _inputs():
    paths = [os.path.join(CSRC, s) for s in SOURCES] + [HEADER]
    paths += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return paths


def up_to_date():
    if not os.path.exists(LIBRARY):
        return False
    built = os.path.getmtime(LIBRARY)
    return all(os.path.getmtime(p) <= built for p in _inputs())


def build(force=False, verbose=False):
    """Compile the native library; returns its path."""
    if not force and up_to_date():
        return LIBRARY
    objdir = os.path.join(LIBDIR, "obj")
    os.makedirs(objdir, exist_ok=True)
    nvcc = _nvcc()
    jobs = []
    for src in SOURCES:
        obj = os.path.join(objdir, src[:-3] + ".o")
        fmad = "-fmad=true" if src in CONTRACT else "-fmad=false"
        cmd = [nvcc, *NVCC_FLAGS, fmad, "-c", "-o", obj, os.path.join(CSRC, src)]
        if verbose:
            print(" ".join(cmd), flush=True)
        jobs.append((cmd, obj, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failures = []
    for cmd, obj, proc in jobs:
        out, _ = proc.communicate()
        if proc.returncode != 0:
            failures.append(" ".join(cmd) + "\n" + out)
    if failures:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failures))
    tmp = LIBRARY + ".tmp"
    link = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp, *[obj for _, obj, _ in jobs]]
    result = subprocess.run(link, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError("nvcc link failed:\n" + result.stdout + result.stderr)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
