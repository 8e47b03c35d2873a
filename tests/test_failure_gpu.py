"""Failure detection on the GPU without a fault: every wait in the kernels is
bounded.  A diagnostic kernel waits on a counter and an mbarrier that nothing ever
signals, with a 2 ms limit; both waits must give up, the device status word must
read MHC_STATUS_DEVICE_TIMEOUT (and be cleared by reading it), and the context must
stay usable: an ordinary operator call afterwards still matches the oracle."""
from __future__ import annotations

import time

import pytest
import torch

import mhcpre_review_b200 as mp
from mhcpre_review_b200.configs import CONFIGS
from tests.test_parity_gpu import check_config

pytestmark = pytest.mark.gpu


def test_bounded_waits_give_up_and_report_timeout():
    assert mp.device_status() == 0
    t0 = time.perf_counter()
    counter_gave_up, barrier_gave_up = mp.diag_wait_timeout(2000)
    elapsed = time.perf_counter() - t0
    assert counter_gave_up and barrier_gave_up
    assert elapsed < 5.0  # two 2 ms limits, not a hang
    assert mp.device_status() == -11  # MHC_STATUS_DEVICE_TIMEOUT
    assert mp.device_status() == 0    # reading clears it


def test_context_usable_after_timeout():
    mp.diag_wait_timeout(1000)
    assert mp.device_status() == -11
    check_config(CONFIGS["c1"])  # asserts device_status() == 0 afterwards
    torch.cuda.synchronize()


def test_diag_rejects_bad_limits():
    import ctypes
    c, b = ctypes.c_int32(0), ctypes.c_int32(0)
    assert mp.lib().mhcPreDiagWaitTimeout(ctypes.c_uint32(0), ctypes.byref(c), ctypes.byref(b), None) == -2
    assert mp.lib().mhcPreDiagWaitTimeout(ctypes.c_uint32(5_000_000), ctypes.byref(c), ctypes.byref(b), None) == -2
