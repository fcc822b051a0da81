"""Build the in-tree native libraries.

* ``libfd_sm100.so`` — the CUDA operator library (C ABI, include/fd_sm100.h),
  compiled by nvcc for sm_100a only; it links the CUDA runtime statically and
  reaches the driver (tensor-map encoding) through cudaGetDriverEntryPoint,
  so it has no torch dependency.
* ``libfd_synth.so`` — a host-only helper of the synthetic data generators.

Usage: ``python -m flashdiffusion_b200.build`` (or ``build()`` from Python).
Rebuilds only when a source is newer than the library.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libfd_sm100.so")
SYNTH = os.path.join(PKG, "libfd_synth.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build_cuda(verbose=False, force=False, extra=()):
    cu = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = cu + glob.glob(os.path.join(CSRC, "*.cuh")) + [os.path.join(ROOT, "include", "fd_sm100.h")]
    if not force and not _stale(LIB, deps):
        return LIB
    cmd = [_nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"), "-o", LIB + ".tmp", *cu, "-ldl", *extra]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libfd_sm100.so")
    if verbose:
        sys.stderr.write(r.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


def build_profile(force=False):
    """libfd_sm100_prof.so: the same library with the block kernel's wait-time
    counters compiled in (-DFD_PROFILE_WAITS; fd_debug_wait_cycles)."""
    prof = os.path.join(PKG, "libfd_sm100_prof.so")
    cu = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = cu + glob.glob(os.path.join(CSRC, "*.cuh")) + [os.path.join(ROOT, "include", "fd_sm100.h")]
    if not force and not _stale(prof, deps):
        return prof
    cmd = [_nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           "--expt-relaxed-constexpr", "-DFD_PROFILE_WAITS", "-I", os.path.join(ROOT, "include"),
           "-o", prof + ".tmp", *cu, "-ldl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libfd_sm100_prof.so")
    os.replace(prof + ".tmp", prof)
    return prof


def build_synth(force=False):
    src = os.path.join(CSRC, "synth_host.c")
    if not force and not _stale(SYNTH, [src]):
        return SYNTH
    subprocess.run(["gcc", "-O2", "-shared", "-fPIC", "-o", SYNTH, src, "-lm"], check=True)
    return SYNTH


def build(verbose=False, force=False):
    build_synth(force=force)
    return build_cuda(verbose=verbose, force=force)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(LIB)
