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


def test_trace_build_fused_post_pre_stages():
    """The fused post + MhcPre kernel under the trace build: the same results, and per
    traced CTA and stage the order loads issued (2) <= data landed (5) <= xNext
    formed (6) <= xNext stores have read it (7)."""
    if not mp.TRACE_LIB_PATH.exists():
        pytest.fail("the trace library was not built (python -m mhcpre_review_b200.build --trace)")
    cfg = with_shape(CONFIGS["c4"], batch=1, seq=2048, name="trace_pp")
    inp = make_inputs(cfg)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(7)
    y = torch.randn((cfg.batch, cfg.seq, cfg.D), generator=gen, device="cuda", dtype=inp["x"].dtype)
    hPost = torch.rand((cfg.batch, cfg.seq, cfg.n), generator=gen, device="cuda")
    hRes = (0.5 * torch.randn((cfg.batch, cfg.seq, cfg.n, cfg.n), generator=gen, device="cuda")).contiguous()

    def run():
        ex = mp.MhcPre(cfg.batch, cfg.seq, cfg.n, cfg.D, inp["x"].dtype, cfg.gamma)
        ex.prepare(inp["phi"], inp["gamma"])
        x_next, out = ex.post_and_run(inp["x"], y, hPost, hRes, inp["alpha"], inp["bias"])
        torch.cuda.synchronize()
        return [x_next, *out]

    ref = run()
    with mp.use_library(mp.TRACE_LIB_PATH):
        mp.trace_read()
        got = run()
        tr, n = mp.trace_read()
        assert mp.device_status() == 0
    for u, v in zip(ref, got):
        assert torch.equal(u, v), "the trace build changed a result"
    stamps = {}
    for ev in (2, 5, 6, 7):
        sel = tr[tr["event"] == ev]
        stamps[ev] = {(int(c), int(a)): int(t) for c, a, t in zip(sel["cta"], sel["a"], sel["t_ns"])}
    keys = set(stamps[2]) & set(stamps[5]) & set(stamps[6]) & set(stamps[7])
    assert len(keys) > 0 and set(stamps[6]) == set(stamps[7]) == keys
    for k in keys:
        assert stamps[2][k] <= stamps[5][k] <= stamps[6][k] <= stamps[7][k]
    med = lambda a, b: np.median([stamps[b][k] - stamps[a][k] for k in keys]) / 1e3
    print(f"\ntrace fused post+pre ({cfg.name}): {len(keys)} traced stages; median us: loads to landed "
          f"{med(2, 5):.2f}, post {med(5, 6):.2f}, stores read {med(6, 7):.2f}")
