"""Shared pytest configuration: the ``gpu`` marker and repository paths."""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")


def pytest_collection_modifyitems(config, items):
    # GPU tests are skipped automatically when no CUDA device is visible.
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def pytest_sessionfinish(session, exitstatus):
    """With MHC_PARITY_REPORT=<path>, writes the per-case parity statistics the GPU
    parity tests collected (hIn max ulp and exact-match rate, hPost/hRes max error)
    as JSON lines."""
    path = os.environ.get("MHC_PARITY_REPORT")
    if not path:
        return
    # the parity module is imported twice (by pytest as a test file, and by the other
    # GPU test files as tests.test_parity_gpu): gather the statistics of both copies
    stats = []
    for name in ("test_parity_gpu", "tests.test_parity_gpu"):
        stats += getattr(sys.modules.get(name), "PARITY_STATS", [])
    import json
    with open(path, "w") as f:
        for st in stats:
            f.write(json.dumps(st) + "\n")
