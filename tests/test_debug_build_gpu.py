"""The debug build (libmhcpre_b200_debug.so, compile flag MHC_DEBUG): bounds checks
on every partial-record index in the kernels.  On the boundary and ragged shapes of
every path it must report nothing and give the default library's results bit for
bit; with the records buffer declared smaller than it is (mhcPreDebugSetRecordCap),
the checks must fail -- skipping the accesses they guard, so nothing outside a
buffer is touched -- and report MHC_STATUS_INTERNAL_CHECK with a source line."""
from __future__ import annotations

import ctypes

import pytest
import torch

import mhcpre_review_b200 as mp
from mhcpre_review_b200.configs import Config, make_inputs
from tests.test_parity_gpu import run_op

pytestmark = pytest.mark.gpu

CASES = [  # (B, S, n, D, gamma, dtype, path)
    (1, 3, 4, 64, True, "bf16", None),      # decode
    (1, 7, 6, 16, False, "fp16", None),     # decode, K not a multiple of 64
    (1, 129, 4, 48, True, "fp16", None),    # small batch
    (3, 100, 8, 32, True, "bf16", None),    # small batch, n = 8
    (1, 1000, 6, 80, True, "bf16", None),   # split-K, ragged tile
    (2, 700, 8, 1040, False, "fp16", None), # split-K, n = 8
    (1, 1000, 4, 1040, True, "bf16", 5),    # one pass
]


def _need_lib():
    if not mp.DEBUG_LIB_PATH.exists():
        pytest.fail("the debug library was not built (python -m mhcpre_review_b200.build --debug)")


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"B{c[0]}S{c[1]}n{c[2]}D{c[3]}{c[5]}p{c[6]}")
def test_debug_build_checks_pass_and_results_match(case, monkeypatch):
    _need_lib()
    B, S, n, D, g, dt, path = case
    if path is not None:
        monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=path))
    inp = make_inputs(Config("debug", B, S, n, D, dt, 0.02, g, seed=71))
    ref = run_op(inp, use_executor=True)
    with mp.use_library(mp.DEBUG_LIB_PATH) as L:
        got = run_op(inp, use_executor=True)
        assert mp.device_status() == 0
        line = ctypes.c_int32(-1)
        assert L.mhcPreDebugLastCheckLine(ctypes.byref(line)) == 0 and line.value == 0
    for u, v in zip(ref, got):
        assert torch.equal(u, v)


@pytest.mark.parametrize("path", [0, 2, 4, 5])
def test_debug_build_reports_a_failed_check(path, monkeypatch):
    _need_lib()
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=path))
    M = {0: 1000, 2: 8, 4: 200, 5: 1000}[path]
    inp = make_inputs(Config("debug_cap", 1, M, 4, 256, "bf16", 0.02, True, seed=72))
    with mp.use_library(mp.DEBUG_LIB_PATH) as L:
        mp.device_status()
        try:
            assert L.mhcPreDebugSetRecordCap(64) == 0  # far below any plan's records buffer
            run_op(inp, use_executor=True)
            assert mp.device_status() == -14  # MHC_STATUS_INTERNAL_CHECK
            line = ctypes.c_int32(0)
            assert L.mhcPreDebugLastCheckLine(ctypes.byref(line)) == 0 and line.value > 0
        finally:
            assert L.mhcPreDebugSetRecordCap(0) == 0
        # the context stays usable and the next call is clean
        run_op(inp, use_executor=True)
        assert mp.device_status() == 0


def _post_pre_inputs(cfg):
    inp = make_inputs(cfg)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(6)
    y = torch.randn((cfg.batch, cfg.seq, cfg.D), generator=gen, device="cuda", dtype=inp["x"].dtype)
    hPost = torch.rand((cfg.batch, cfg.seq, cfg.n), generator=gen, device="cuda")
    hRes = (0.5 * torch.randn((cfg.batch, cfg.seq, cfg.n, cfg.n), generator=gen, device="cuda")).contiguous()
    return inp, y, hPost, hRes


def _post_pre(cfg, inp, y, hPost, hRes):
    ex = mp.MhcPre(cfg.batch, cfg.seq, cfg.n, cfg.D, inp["x"].dtype, cfg.gamma)
    ex.prepare(inp["phi"], inp["gamma"])
    x_next, out = ex.post_and_run(inp["x"], y, hPost, hRes, inp["alpha"], inp["bias"])
    torch.cuda.synchronize()
    return [x_next, *out]


def test_debug_build_fused_post_pre():
    """The fused post + MhcPre kernel under the debug build: no check fires and the
    results equal the default build's; with the records buffer declared too small,
    its record writes are skipped and reported."""
    _need_lib()
    cfg = Config("debug_pp", 1, 1000, 4, 1024, "bf16", 0.02, True, seed=73)
    args = _post_pre_inputs(cfg)
    ref = _post_pre(cfg, *args)
    with mp.use_library(mp.DEBUG_LIB_PATH) as L:
        got = _post_pre(cfg, *args)
        assert mp.device_status() == 0
        line = ctypes.c_int32(-1)
        assert L.mhcPreDebugLastCheckLine(ctypes.byref(line)) == 0 and line.value == 0
        for u, v in zip(ref, got):
            assert torch.equal(u, v)
        try:
            assert L.mhcPreDebugSetRecordCap(64) == 0
            _post_pre(cfg, *args)
            assert mp.device_status() == -14  # MHC_STATUS_INTERNAL_CHECK
            assert L.mhcPreDebugLastCheckLine(ctypes.byref(line)) == 0 and line.value > 0
        finally:
            assert L.mhcPreDebugSetRecordCap(0) == 0
        _post_pre(cfg, *args)
        assert mp.device_status() == 0
