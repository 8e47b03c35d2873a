"""The split-K epilogue is compiled twice: for 12 resident rows per SM (40 registers a
thread) and for 16 (at most 32), the default up to 16384 rows.  The arithmetic is the
same, so both must give the same bits on every shape, and the default plan's choice
must pass the parity rule."""
from __future__ import annotations

import pytest
import torch

import mhcpre_review_b200 as mp
from mhcpre_review_b200.configs import CONFIGS, Config, make_inputs, with_shape
from tests.test_parity_gpu import bits, compare, np32

pytestmark = pytest.mark.gpu

CASES = [
    with_shape(CONFIGS["c2"], name="ev_c2"),
    Config("ev_fp16_ragged", 1, 1000, 4, 1024, "fp16", 0.01, True, seed=81),
    Config("ev_d1040", 1, 700, 4, 1040, "bf16", 0.01, False, seed=82),
    Config("ev_n6", 1, 900, 6, 512, "bf16", 0.01, True, seed=83),
    with_shape(CONFIGS["c3"], batch=1, seq=1024, name="ev_c3_1024"),
    with_shape(CONFIGS["c4"], batch=1, seq=2048, name="ev_c4_2048"),
]


def _run(cfg, inp, blocks):
    with mp.plan_options(path=0, epi_blocks=blocks):
        ex = mp.MhcPre(cfg.batch, cfg.seq, cfg.n, cfg.D, inp["x"].dtype, cfg.gamma)
        ex.prepare(inp["phi"], inp["gamma"])
        out = ex(inp["x"], inp["alpha"], inp["bias"])
    torch.cuda.synchronize()
    assert mp.device_status() == 0
    return [t.clone() for t in out]


@pytest.mark.parametrize("cfg", CASES, ids=lambda c: c.name)
def test_epilogue_variants_give_the_same_bits(cfg):
    inp = make_inputs(cfg)
    twelve, sixteen, default = _run(cfg, inp, 12), _run(cfg, inp, 16), _run(cfg, inp, 0)
    for a, b, c in zip(twelve, sixteen, default):
        assert torch.equal(a, b) and torch.equal(a, c)
    M, n, D = cfg.M, cfg.n, cfg.D
    hIn, hPost, hRes = default
    gamma = np32(inp["gamma"])
    compare((bits(hIn.reshape(M, D)), hPost.reshape(M, n).cpu().numpy(), hRes.reshape(M, n, n).cpu().numpy()),
            bits(inp["x"].reshape(M, n * D)), np32(inp["phi"]), np32(inp["alpha"]), np32(inp["bias"]),
            None if gamma is None else gamma.reshape(-1), n, D, cfg.dtype, cfg.name)
