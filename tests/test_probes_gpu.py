"""Hardware probes behind the single-pass findings, built with nvcc and run on the
GPU (their tables go to the test log):

  probes/mma_rate.cu      tcgen05.mma issue rate per SM for M x N tiles and 1, 2 or 4
                          issuing warps: x bytes per cycle with token rows on the
                          MMA's M dimension (M = 128) or on its N dimension (8..256)
  probes/l2_bandwidth.cu  L2 -> SM read bandwidth against the re-read footprint, and
                          DRAM read bandwidth
"""
from __future__ import annotations

import re
import shutil
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent


def _build(name, tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    exe = tmp_path / name
    subprocess.check_call([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                           "-o", str(exe), str(HERE / "probes" / f"{name}.cu")])
    return exe


def test_mma_issue_rate(tmp_path):
    out = subprocess.run([str(_build("mma_rate", tmp_path)), "256"], capture_output=True, text=True, timeout=300)
    print("\n" + out.stdout)
    assert out.returncode == 0 and "status 0" in out.stdout
    rows = {}
    for m, n, iss, cyc, bpc in re.findall(r"M +(\d+) N +(\d+) issuers (\d) cycles_per_mma +([\d.]+) "
                                          r"x_bytes_per_cycle +([\d.]+)", out.stdout):
        rows[(int(m), int(n), int(iss))] = float(bpc)
    assert rows[(128, 48, 1)] > 0 and rows[(64, 32, 1)] > 0


def test_l2_read_bandwidth(tmp_path):
    out = subprocess.run([str(_build("l2_bandwidth", tmp_path))], capture_output=True, text=True, timeout=300)
    print("\n" + out.stdout)
    assert out.returncode == 0 and "status no error" in out.stdout
    bw = [float(v) for v in re.findall(r"GBps ([\d.]+)", out.stdout)]
    assert len(bw) == 14 and min(bw) > 0
