"""mhcPreRunNoAlloc: the operator for callers that cannot allocate device memory.

Some callers cannot hand the operator a workspace: a plugin that receives only its
tensors' device pointers and no allocator, a serving runtime whose device memory is
planned and locked before traffic starts, or a latency-critical loop that must not
call cudaMalloc because it can synchronize the device.  For them the library keeps
the workspace in one fixed 96 MiB device array of its own and the call allocates
nothing.

This file is named so pytest collects it last.  It checks, through the C ABI, that
two calls in a row (on two different problems, so the second one starts from the
first one's leftovers in the shared array) give the same outputs as the ordinary
entry point mhcPreRun, bit for bit (the two share the plan, the kernels and the
reduction order, so any difference would be state left over in the array); that a problem
larger than the array is rejected before anything runs; and that the calls leave
the device's free memory unchanged.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

import mhcpre_review_b200 as mp
from mhcpre_review_b200.configs import CONFIGS, make_inputs, with_shape

pytestmark = pytest.mark.gpu


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _outputs(x, n, D):
    B, S = x.shape[0], x.shape[1]
    return (torch.empty((B, S, D), dtype=x.dtype, device="cuda"),
            torch.empty((B, S, n), dtype=torch.float32, device="cuda"),
            torch.empty((B, S, n, n), dtype=torch.float32, device="cuda"))


def _desc(cfg, x):
    return mp.make_desc(cfg.batch, cfg.seq, cfg.n, cfg.D, mp.BF16 if x.dtype == torch.bfloat16 else mp.F16,
                        cfg.gamma, cfg.norm_eps, cfg.hc_eps)


def _run_no_alloc(cfg, inp, out):
    d = _desc(cfg, inp["x"])
    return mp.lib().mhcPreRunNoAlloc(ctypes.byref(d), _p(inp["x"]), _p(inp["phi"]), _p(inp["alpha"]),
                                     _p(inp["bias"]), _p(inp["gamma"]), _p(out[0]), _p(out[1]), _p(out[2]),
                                     _stream())


def _run_with_workspace(cfg, inp, out):
    d = _desc(cfg, inp["x"])
    ws_bytes = mp.workspace_size(d)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    rc = mp.lib().mhcPreRun(ctypes.byref(d), _p(inp["x"]), _p(inp["phi"]), _p(inp["alpha"]), _p(inp["bias"]),
                            _p(inp["gamma"]), _p(out[0]), _p(out[1]), _p(out[2]), _p(ws), ctypes.c_size_t(ws_bytes),
                            _stream())
    torch.cuda.synchronize()
    return rc


def _assert_same(a, b):
    # Same plan, same kernels, same fixed reduction order as mhcPreRun: the outputs
    # must be identical bit for bit (a looser rule could hide state left over in the
    # shared scratch array from the previous call).
    for g, r in zip(a, b):
        assert torch.equal(g, r)


def test_no_alloc_entry_matches_workspace_entry_twice():
    # two different problems back to back: the second starts from the first's
    # leftovers in the shared scratch array
    cases = [with_shape(CONFIGS["c2"], seq=1024), with_shape(CONFIGS["c5_m32_ng"], seed=3)]
    inputs = [make_inputs(c) for c in cases]
    outs = [_outputs(i["x"], c.n, c.D) for c, i in zip(cases, inputs)]
    refs = [_outputs(i["x"], c.n, c.D) for c, i in zip(cases, inputs)]

    # first call on this device: looks up the scratch array's address (set-up)
    assert _run_no_alloc(cases[0], inputs[0], outs[0]) == 0
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for c, i, o in zip(cases, inputs, outs):
        assert _run_no_alloc(c, i, o) == 0
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before, "the no-allocation entry point changed the device's free memory"

    for c, i, r in zip(cases, inputs, refs):
        assert _run_with_workspace(c, i, r) == 0
    for o, r in zip(outs, refs):
        _assert_same(o, r)
    assert mp.device_status() == 0


SCRATCH_BYTES = 96 * 1024 * 1024  # MHC_PRE_NOALLOC_SCRATCH_BYTES in include/mhc_pre.h


def test_no_alloc_rejects_problems_larger_than_the_scratch_array():
    # config 4 itself fits, as the header promises
    c4 = CONFIGS["c4"]
    assert mp.workspace_size(mp.make_desc(c4.batch, c4.seq, c4.n, c4.D, mp.BF16, True)) <= SCRATCH_BYTES
    # twice its rows do not: the split-K path's partial records grow with M (about
    # 126 MiB of workspace at M = 131072)
    cfg = with_shape(CONFIGS["c4"], batch=32, D=7184)
    d = mp.make_desc(cfg.batch, cfg.seq, cfg.n, cfg.D, mp.BF16, True)
    assert mp.workspace_size(d) > SCRATCH_BYTES
    rc = mp.lib().mhcPreRunNoAlloc(ctypes.byref(d), None, None, None, None, None, None, None, None, _stream())
    assert rc == -13  # MHC_STATUS_TOO_LARGE, before any pointer is touched
