"""The cluster-team single-pass kernel (path 3, chosen through plan options): plan selection,
parity with the CPU oracle on shapes with 16- and 8-CTA clusters (fp16 and bf16,
n=4/6/8, ragged last tile), agreement with the split-K path, and determinism."""
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


def test_cluster_plan_for_config4(monkeypatch):
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=3))
    plan = _plan(CONFIGS["c4"])
    assert plan["path"] == 3 and plan["kernels_per_run"] == 1 and plan["splits"] == 16
    assert plan["grid_ctas"] % 16 == 0 and 16 <= plan["grid_ctas"] <= 148


CASES = [
    Config("cl_n4_d512_tiny", 1, 130, 4, 512, "bf16", 0.02, True, seed=41),      # S=8, 2 tiles, ragged
    Config("cl_n8_d1024", 1, 1000, 8, 1024, "fp16", 0.01, True, seed=42),         # S=16, N=160
    Config("cl_n6_d1024", 2, 700, 6, 1024, "bf16", 0.01, False, seed=43),         # S=16, N=96
    with_shape(CONFIGS["c2"], name="cl_c2"),                                       # S=8, D=2560
    with_shape(CONFIGS["c3"], batch=1, seq=2048, name="cl_c3_small"),             # n=8 with outliers
]


@pytest.mark.parametrize("cfg", CASES, ids=lambda c: c.name)
def test_cluster_parity(cfg, monkeypatch):
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=3))
    assert _plan(cfg)["path"] == 3
    check_config(cfg)


def test_cluster_matches_split_k_and_is_deterministic(monkeypatch):
    cfg = with_shape(CONFIGS["c4"], batch=1, seq=4096)
    inp = make_inputs(cfg)
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=3))
    a = run_op(inp, use_executor=True)
    b = run_op(inp, use_executor=True)
    for u, v in zip(a, b):
        assert torch.equal(u, v)
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=0))
    c = run_op(inp, use_executor=True)
    for u, v in zip(a[1:], c[1:]):
        err = (u.double() - v.double()).abs() / v.double().abs().clamp_min(1.0)
        assert float(err.max()) <= 2 * RTOL
    same = (a[0].view(torch.int16) == c[0].view(torch.int16)).float().mean()
    assert float(same) > 0.99
    assert mp.device_status() == 0
