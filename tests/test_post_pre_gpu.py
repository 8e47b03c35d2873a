"""The post step fused with the next layer's MhcPre (mhcPostPreRun): xNext must equal
the post step's C oracle bit for bit, and the next layer's hIn, hPost and hRes must
match the MhcPre oracle on that xNext within the parity tolerances; the fused call
must agree with the two separate calls (mhcPostRun, then mhcPreRunPrepared), in
place and out of place; and where the fused kernel does not apply (n != 4, headDim
not a multiple of 64, few rows) the call is the two separate calls exactly."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import mhcpre_review_b200 as mp
from mhcpre_review_b200.configs import CONFIGS, Config, make_inputs, with_shape
from oracle import ref
from tests.test_parity_gpu import RTOL, compare

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _layer_inputs(cfg, seed):
    """The next layer's MhcPre inputs (weights, alpha, bias) from the config, and the
    ending layer's x, y, hPost, hRes."""
    inp = make_inputs(cfg)
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    x = inp["x"]
    y = torch.randn((cfg.batch, cfg.seq, cfg.D), generator=g, device="cuda", dtype=x.dtype)
    hPost = (2.0 * torch.sigmoid(torch.randn((cfg.batch, cfg.seq, cfg.n), generator=g, device="cuda"))).contiguous()
    hRes = (0.5 * torch.randn((cfg.batch, cfg.seq, cfg.n, cfg.n), generator=g, device="cuda")).contiguous()
    return inp, y, hPost, hRes


def _executor(cfg, inp):
    ex = mp.MhcPre(cfg.batch, cfg.seq, cfg.n, cfg.D, inp["x"].dtype, cfg.gamma)
    ex.prepare(inp["phi"], inp["gamma"])
    return ex


CASES = [
    (with_shape(CONFIGS["c4"], batch=1, seq=2048, name="pp_c4_2048"), True),
    (Config("pp_fp16_ragged", 1, 1000, 4, 1024, "fp16", 0.01, True, seed=91), True),
    (with_shape(CONFIGS["c2"], name="pp_c2"), True),
    (Config("pp_n8_fallback", 1, 600, 8, 512, "bf16", 0.01, True, seed=92), False),   # n = 8: two calls
    (Config("pp_d1040_fallback", 1, 700, 4, 1040, "bf16", 0.01, False, seed=93), False),  # D % 64 != 0
    (Config("pp_small_fallback", 1, 100, 4, 512, "bf16", 0.02, True, seed=94), False),  # single-launch range
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: c[0].name)
def test_post_pre_matches_oracles(case):
    cfg, fused = case
    inp, y, hPost, hRes = _layer_inputs(cfg, seed=7)
    x = inp["x"]
    ex = _executor(cfg, inp)
    x_next, (hIn, hPostN, hResN) = ex.post_and_run(x, y, hPost, hRes, inp["alpha"], inp["bias"])
    torch.cuda.synchronize()
    assert mp.device_status() == 0
    M, n, D = cfg.M, cfg.n, cfg.D
    want = ref.mhc_post_ref(_bits(x), _bits(y), hPost.cpu().numpy(), hRes.cpu().numpy(), n, D, cfg.dtype)
    got_next = _bits(x_next).reshape(want.shape)
    assert np.array_equal(got_next, want), "xNext differs from the post step's oracle"
    gamma = None if inp["gamma"] is None else inp["gamma"].reshape(-1).cpu().numpy()
    compare((_bits(hIn.reshape(M, D)), hPostN.reshape(M, n).cpu().numpy(), hResN.reshape(M, n, n).cpu().numpy()),
            want.reshape(M, n * D), inp["phi"].cpu().numpy(), inp["alpha"].cpu().numpy(), inp["bias"].cpu().numpy(),
            gamma, n, D, cfg.dtype, cfg.name)


@pytest.mark.parametrize("case", CASES, ids=lambda c: c[0].name)
def test_post_pre_agrees_with_the_two_calls(case):
    cfg, fused = case
    inp, y, hPost, hRes = _layer_inputs(cfg, seed=8)
    x = inp["x"]
    ex = _executor(cfg, inp)
    a_next, a = ex.post_and_run(x, y, hPost, hRes, inp["alpha"], inp["bias"])
    b_next = mp.mhc_post(x, y, hPost, hRes)
    b = ex(b_next, inp["alpha"], inp["bias"])
    torch.cuda.synchronize()
    assert torch.equal(a_next, b_next)
    if fused:
        # the fused pass splits K by d-chunks of every stream: last bits may differ
        for u, v in zip(a[1:], b[1:]):
            err = (u.double() - v.double()).abs() / v.double().abs().clamp_min(1.0)
            assert float(err.max()) <= 2 * RTOL
        same = (a[0].view(torch.int16) == b[0].view(torch.int16)).float().mean()
        assert float(same) > 0.99
    else:
        for u, v in zip(a, b):
            assert torch.equal(u, v)
    assert mp.device_status() == 0


def test_post_pre_in_place_and_deterministic():
    cfg = with_shape(CONFIGS["c4"], batch=1, seq=1024, name="pp_in_place")
    inp, y, hPost, hRes = _layer_inputs(cfg, seed=9)
    ex = _executor(cfg, inp)
    out_of_place = ex.post_and_run(inp["x"], y, hPost, hRes, inp["alpha"], inp["bias"])
    again = ex.post_and_run(inp["x"], y, hPost, hRes, inp["alpha"], inp["bias"])
    xi = inp["x"].clone()
    in_place = ex.post_and_run(xi, y, hPost, hRes, inp["alpha"], inp["bias"], x_next=xi)
    torch.cuda.synchronize()
    assert torch.equal(out_of_place[0], in_place[0]) and torch.equal(out_of_place[0], again[0])
    for u, v, w in zip(out_of_place[1], in_place[1], again[1]):
        assert torch.equal(u, v) and torch.equal(u, w)
    assert mp.device_status() == 0
