"""The persistent kernels' work split, checked on the host: tests/sched_check.cu
compiles the schedule code of flashdiffusion_b200/csrc/fd_tc_common.cuh for the
CPU and verifies unit coverage and the fix-up owner lists over many shapes
(contiguous ranges and lockstep rows with chunked remainders)."""
import os
import shutil
import subprocess
import tempfile

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def test_schedule_covers_every_unit_once():
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not available")
    with tempfile.TemporaryDirectory() as td:
        exe = os.path.join(td, "sched_check")
        subprocess.run([nvcc, "-std=c++17", "-O1", "--expt-relaxed-constexpr", "-o", exe, os.path.join(HERE, "sched_check.cu")],
                       check=True, capture_output=True)
        r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stdout + r.stderr
        assert r.stdout.startswith("OK")
