"""The one-pass kernel (path 5, x read from HBM once; n = 4): plan selection,
parity with the CPU oracle (bf16 and fp16, gamma on and off, a ragged last tile, K
not a multiple of the 4-chunk work item, both CTA layouts, a record ring small
enough that the TMA producer must wait for it), determinism, independence of M
(token shards reproduce the full run bit for bit), and agreement with the split-K
path."""
from __future__ import annotations

import pytest
import torch

import mhcpre_review_b200 as mp
from mhcpre_review_b200.configs import CONFIGS, Config, make_inputs, with_shape
from tests.test_parity_gpu import RTOL, check_config, run_op

pytestmark = pytest.mark.gpu


def _plan(cfg):
    return mp.query_plan(mp.make_desc(cfg.batch, cfg.seq, cfg.n, cfg.D, mp.BF16 if cfg.dtype == "bf16" else mp.F16,
                                      cfg.gamma))


def test_onepass_plan_for_config4(monkeypatch):
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=5))
    plan = _plan(CONFIGS["c4"])
    assert plan["path"] == 5 and plan["kernels_per_run"] == 1
    assert plan["splits"] == 28672 // 64 // 4  # work items of four 64-wide chunks
    # n = 8 has no one-pass kernel: the plan falls back to split-K
    assert _plan(CONFIGS["c3"])["path"] == 0


CASES = [
    (with_shape(CONFIGS["c4"], batch=1, seq=2048, name="op_c4_2048"), {}),
    (Config("op_ragged_fp16", 1, 1000, 4, 1024, "fp16", 0.01, True, seed=51), {}),
    (Config("op_k_odd_nogamma", 3, 300, 4, 1040, "bf16", 0.01, False, seed=52), {}),  # K/64 = 65 chunks
    (with_shape(CONFIGS["c2"], name="op_c2"), {}),
    (with_shape(CONFIGS["c2"], name="op_c2_two_ctas"), {"gemm_ctas_per_sm": 2}),
    (with_shape(CONFIGS["c2"], name="op_c2_ring2"), {"ring_tiles": 2}),    # the producer waits for the ring
    (Config("op_tiny", 1, 5, 4, 64, "bf16", 0.05, True, seed=53), {}),     # one partial tile, one chunk split
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: c[0].name)
def test_onepass_parity(case, monkeypatch):
    cfg, opts = case
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=5, **opts))
    assert _plan(cfg)["path"] == 5
    check_config(cfg)


def test_onepass_full_config4(monkeypatch):
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=5))
    check_config(CONFIGS["c4"])


def test_onepass_is_deterministic_and_independent_of_m(monkeypatch):
    cfg = with_shape(CONFIGS["c4"], batch=2, seq=1536)
    inp = make_inputs(cfg)
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=5))
    a = run_op(inp, use_executor=True)
    b = run_op(inp, use_executor=True)
    for u, v in zip(a, b):
        assert torch.equal(u, v)
    # rows are independent and the plan depends on K only: each half alone gives the
    # same bits, whatever its grid and ring
    halves = [run_op(dict(inp, x=inp["x"][i:i + 1].contiguous()), use_executor=True) for i in range(2)]
    for k in range(3):
        assert torch.equal(a[k], torch.cat([h[k] for h in halves], dim=0))
    # the two CTA layouts and ring sizes give the same bits too
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=5, gemm_ctas_per_sm=2, ring_tiles=3))
    c = run_op(inp, use_executor=True)
    for u, v in zip(a, c):
        assert torch.equal(u, v)
    # agreement with the split-K path (a different K-split, so fp32 sums differ)
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=0))
    d = run_op(inp, use_executor=True)
    for u, v in zip(a[1:], d[1:]):
        err = (u.double() - v.double()).abs() / v.double().abs().clamp_min(1.0)
        assert float(err.max()) <= 2 * RTOL
    same = (a[0].view(torch.int16) == d[0].view(torch.int16)).float().mean()
    assert float(same) > 0.99
    assert mp.device_status() == 0
