"""CPU check of the tensor-core engine's work-unit schedule and mask scanning:
tests/sched_check.cu includes the same header the kernels use
(csrc/schedule.cuh), is compiled with nvcc for the host and run here."""

import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


def test_schedule_and_mask_scan_on_host(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).exists():
        pytest.skip("nvcc not available")
    exe = tmp_path / "sched_check"
    res = subprocess.run([nvcc, "-std=c++17", "-O1", "-I", str(REPO / "mlx-cross-entropy_b200" / "csrc"),
                          "-o", str(exe), str(REPO / "tests" / "sched_check.cu")],
                         capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr[-3000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0 and "SCHEDULE_OK" in run.stdout, run.stdout[-2000:]
