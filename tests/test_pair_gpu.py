"""The split-K GEMM on CTA pairs (n = 8, plan option paired_gemm = 2): one
M = 256 tcgen05 MMA per 2-CTA cluster, each CTA staging its own 128-row x tile and
half of the 160 weight rows.  Its arithmetic per row is the one-CTA GEMM's, so the
results must equal the one-CTA path's bit for bit; parity with the oracle on n = 8
shapes (bf16 and fp16, an odd number of row tiles, K not a multiple of 64, a
ragged last tile) and all rows of config 3."""
from __future__ import annotations

import pytest
import torch

import mhcpre_review_b200 as mp
from mhcpre_review_b200.configs import CONFIGS, Config, make_inputs, with_shape
from tests.test_parity_gpu import check_config, run_op

pytestmark = pytest.mark.gpu


def _plan(cfg):
    return mp.query_plan(mp.make_desc(cfg.batch, cfg.seq, cfg.n, cfg.D, mp.BF16 if cfg.dtype == "bf16" else mp.F16,
                                      cfg.gamma))


CASES = [
    Config("pair_n8_odd_tiles", 1, 300, 8, 512, "bf16", 0.01, True, seed=81),     # 3 row tiles: one lone tile
    Config("pair_n8_fp16_kodd", 2, 700, 8, 1040, "fp16", 0.01, False, seed=82),   # K/64 = 130, ragged
    with_shape(CONFIGS["c3"], batch=1, seq=4096, name="pair_c3_4096"),           # outliers, 11 splits
]


@pytest.mark.parametrize("cfg", CASES, ids=lambda c: c.name)
def test_pair_gemm_equals_one_cta_gemm_and_matches_oracle(cfg, monkeypatch):
    inp = make_inputs(cfg)
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=0, paired_gemm=1))
    one = run_op(inp, use_executor=True)
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=0, paired_gemm=2))
    assert _plan(cfg)["path"] == 0
    two = run_op(inp, use_executor=True)
    assert mp.device_status() == 0
    for u, v in zip(one, two):
        assert torch.equal(u, v)
    check_config(cfg)


def test_pair_gemm_config3_all_rows(monkeypatch):
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(paired_gemm=2))
    check_config(CONFIGS["c3"])
