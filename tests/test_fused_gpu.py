"""The fused single-kernel path (path 1): plan selection, parity with the CPU
oracle on shapes beyond the BASELINE configs, agreement with the split-K path, and
determinism.  The fused path is opt-in: plan options (path=1) select it when D is a
multiple of 64."""
from __future__ import annotations

import pytest
import torch

import mhcpre_review_b200 as mp
from mhcpre_review_b200.configs import CONFIGS, Config, make_inputs, with_shape
from tests.test_parity_gpu import RTOL, check_config, run_op

pytestmark = pytest.mark.gpu


def test_fused_plan_for_config4(monkeypatch):
    cfg = CONFIGS["c4"]
    desc = mp.make_desc(cfg.batch, cfg.seq, cfg.n, cfg.D, mp.BF16, cfg.gamma)
    assert mp.query_plan(desc)["path"] == 0  # the fused kernel is opt-in
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=1))
    plan = mp.query_plan(desc)
    assert plan["path"] == 1 and plan["kernels_per_run"] == 1
    assert plan["splits"] == 28 and plan["grid_ctas"] == 140  # 5 teams of 28: about 37 MB of tiles in flight


FORCED = [
    with_shape(CONFIGS["c2"], name="c2_fused"),                                   # n=4, S=8, 18 teams
    Config("n8_d1024", 1, 1000, 8, 1024, "fp16", 0.01, True, seed=5),           # ragged last tile, fp16
    Config("n6_d1024", 2, 700, 6, 1024, "bf16", 0.01, False, seed=6),           # n=6 (N=96)
    Config("n4_d512_tiny", 1, 130, 4, 512, "bf16", 0.02, True, seed=7),         # 2 tiles, S=8
    with_shape(CONFIGS["c3"], batch=1, seq=2048, name="c3_small"),              # n=8 with outliers
]


@pytest.mark.parametrize("cfg", FORCED, ids=lambda c: c.name)
def test_fused_parity_forced(cfg, monkeypatch):
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=1))
    plan = mp.query_plan(mp.make_desc(cfg.batch, cfg.seq, cfg.n, cfg.D, mp.BF16, cfg.gamma))
    assert plan["path"] == 1
    check_config(cfg)


def test_fused_and_split_paths_agree(monkeypatch):
    cfg = with_shape(CONFIGS["c4"], batch=1, seq=4096)
    inp = make_inputs(cfg)
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=1))
    a = run_op(inp)
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=0))
    b = run_op(inp)
    for name, u, v in (("hPost", a[1], b[1]), ("hRes", a[2], b[2])):
        err = ((u.double() - v.double()).abs() / v.double().abs().clamp_min(1.0)).max().item()
        assert err <= RTOL, (name, err)
    ua = a[0].view(torch.int16).int()
    ub = b[0].view(torch.int16).int()
    oa = torch.where(ua < 0, -(ua & 0x7FFF), ua)
    ob = torch.where(ub < 0, -(ub & 0x7FFF), ub)
    assert ((oa - ob).abs() <= 1).float().mean().item() > 0.9999


def test_fused_is_deterministic():
    cfg = with_shape(CONFIGS["c4"], batch=2)   # M = 8192: fused path by default
    inp = make_inputs(cfg)
    a = run_op(inp)
    b = run_op(inp)
    for u, v in zip(a, b):
        assert torch.equal(u, v)
    assert mp.device_status() == 0
