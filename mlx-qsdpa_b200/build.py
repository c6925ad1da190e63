"""Build libqsdpa.so (the sm_100a kernels behind the C ABI in include/qsdpa.h).

    python mlx-qsdpa_b200/build.py [--force] [--verbose] [--trace]

Compiles every ``csrc/*.cu`` with nvcc for sm_100a (cross-compiles without a
GPU) and links them, with the CUDA runtime linked statically, into
``mlx_qsdpa/libqsdpa.so`` next to the Python package that loads it.  Objects
go to ``_build/`` (git-ignored); a source is recompiled only when it or a
header is newer than its object.  ``--trace`` builds the instrumented
variant ``mlx_qsdpa/libqsdpa_trace.so`` (objects in ``_build_trace/``): the
decode kernel's per-tile hand-off clocks and the sharded step's per-CTA
timeline (``python -m mlx_qsdpa.shard_timeline``); the package loads it only
when ``QSDPA_LIB`` names it.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "mlx_qsdpa", "libqsdpa.so")
TRACE_LIB = os.path.join(HERE, "mlx_qsdpa", "libqsdpa_trace.so")
TRACE_FLAGS = ["-DQSDPA_TC_TRACE", "-DQSDPA_SHARD_TRACE"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
              "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libqsdpa.so")


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra_flags=(), trace: bool = False) -> str:
    """Compile (if needed) and return the path of libqsdpa.so (or of the trace variant)."""
    nvcc = _nvcc()
    build_dir, lib = (BUILD + "_trace", TRACE_LIB) if trace else (BUILD, LIB)
    extra_flags = list(extra_flags) + (TRACE_FLAGS if trace else [])
    os.makedirs(build_dir, exist_ok=True)
    sources = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    headers = _headers()
    jobs = []
    objs = []
    for src in sources:
        s = os.path.join(CSRC, src)
        o = os.path.join(build_dir, src[:-3] + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            cmd = [nvcc, *ARCH, *NVCC_FLAGS, *extra_flags, "-c", s, "-o", o]
            jobs.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, flush=True)

    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            list(ex.map(run, jobs))
    if force or jobs or _stale(lib, objs):
        cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", lib, *objs]
        run(cmd)
    return lib


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--trace", action="store_true", help="build the instrumented libqsdpa_trace.so")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose, trace=args.trace))


if __name__ == "__main__":
    sys.exit(main())
