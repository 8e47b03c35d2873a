"""The trace build (libmhcpre_b200_trace.so, compile flag MHC_TRACE): the same
results as the default library, and stage stamps that a reader can re-derive the
kernels' timelines from.  One small case per traced path prints its stage
summary (medians in microseconds) to the test log."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import mhcpre_review_b200 as mp
from mhcpre_review_b200.configs import CONFIGS, make_inputs, with_shape
from tests.test_parity_gpu import run_op

pytestmark = pytest.mark.gpu


def _rows(tr, ev):
    sel = tr[tr["event"] == ev]
    return {(int(a) | (int(b) << 32)): int(t) for a, b, t in zip(sel["a"], sel["b"], sel["t_ns"])}


@pytest.mark.parametrize("path", [5, 0])
def test_trace_build_matches_and_records_stages(path, monkeypatch):
    if not mp.TRACE_LIB_PATH.exists():
        pytest.fail("the trace library was not built (python -m mhcpre_review_b200.build --trace)")
    cfg = with_shape(CONFIGS["c2"], name="trace_c2")
    inp = make_inputs(cfg)
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=path))
    ref = run_op(inp, use_executor=True)
    with mp.use_library(mp.TRACE_LIB_PATH):
        mp.trace_read()  # start from an empty trace
        got = run_op(inp, use_executor=True)
        tr, n = mp.trace_read()
        assert mp.device_status() == 0
    for u, v in zip(ref, got):
        assert torch.equal(u, v), "the trace build changed a result"
    assert 0 < n == len(tr)
    assert set(np.unique(tr["cta"]) % 8) == {0}  # every 8th CTA records
    begins = tr[tr["event"] == 10]
    ends = tr[tr["event"] == 11]
    assert len(begins) > 0 and len(begins) == len(ends)
    span_us = (int(tr["t_ns"].max()) - int(tr["t_ns"].min())) / 1e3
    items = tr[tr["event"] == 1]
    records = tr[tr["event"] == 3]
    assert len(items) > 0 and len(records) > 0
    if path == 5:
        wait, ready, reduced, done = (_rows(tr, e) for e in (4, 5, 6, 7))
        assert len(wait) > 0 and set(wait) == set(ready) == set(reduced) == set(done)
        for r in wait:
            assert wait[r] <= ready[r] <= reduced[r] <= done[r]
        w = np.array([ready[r] - wait[r] for r in wait]) / 1e3
        red = np.array([reduced[r] - ready[r] for r in wait]) / 1e3
        hin = np.array([done[r] - reduced[r] for r in wait]) / 1e3
        print(f"\ntrace path 5 ({cfg.name}): {len(wait)} traced rows over {span_us:.1f} us; median us: "
              f"wait for tile {np.median(w):.2f}, records {np.median(red):.2f}, hIn stream {np.median(hin):.2f}")
    else:
        b, e = _rows(tr, 8), _rows(tr, 9)
        assert len(b) > 0 and set(b) == set(e)
        rows = np.array([e[r] - b[r] for r in b]) / 1e3
        print(f"\ntrace path 0 ({cfg.name}): {len(items)} traced GEMM items, {len(b)} traced epilogue rows over "
              f"{span_us:.1f} us; median epilogue row {np.median(rows):.2f} us")
