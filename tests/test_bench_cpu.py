"""bench.py host logic on CPU: which workloads get an L2 flush between timed steps,
and the reference arm's JSON line (it runs the CPU formula, no GPU needed)."""
import json
import subprocess
import sys
from pathlib import Path

import bench
from mhcpre_review_b200.configs import CONFIGS

ROOT = Path(__file__).resolve().parents[1]


def test_flush_only_below_twice_l2():
    # config 4 on one GPU and on 8 (0.47 GB per GPU) streams more than L2: no flush
    c4 = CONFIGS["c4"]
    assert not bench.needs_flush(c4, c4.M)
    assert not bench.needs_flush(c4, c4.M // 8)
    # config 2 (84 MB of x) and config 3 at 8 GPUs (134 MB) fit in twice the L2: flushed
    c2, c3 = CONFIGS["c2"], CONFIGS["c3"]
    assert bench.needs_flush(c2, c2.M)
    assert bench.needs_flush(c3, c3.M // 8)
    assert not bench.needs_flush(c3, c3.M)
    assert bench.FLUSH_BYTES > 126 * 1000 * 1000


def test_workload_config_says_how_l2_was_handled():
    assert "flushed" in bench.workload_config(CONFIGS["c2"], 1)["l2"]
    assert "no flush" in bench.workload_config(CONFIGS["c4"], 1)["l2"]
    warm = bench.workload_config(CONFIGS["c2"], 1, flushed=False)["l2"]
    assert "warm" in warm and "not a headline" in warm


def test_reference_arm_line():
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", "c1", "--steps", "3",
                          "--warmup", "3"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0 and line["higher_is_better"] is True
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
