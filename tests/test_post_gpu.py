"""The mHC post step on the GPU (mhcPostRun through the C ABI): bit-exact parity with
the C oracle, which states the same operation order (parity unpinned: the reference
has no code for the step after the layer), in place and out of place, chained after
MhcPre, and the pointer checks."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import mhcpre_review_b200 as mp
from mhcpre_review_b200.configs import CONFIGS, make_inputs
from oracle import ref

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _inputs(B, S, n, D, dtype, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    dt = torch.bfloat16 if dtype == "bf16" else torch.float16
    x = torch.randn((B, S, n, D), generator=g, device="cuda", dtype=dt)
    y = torch.randn((B, S, D), generator=g, device="cuda", dtype=dt)
    hPost = 2.0 * torch.sigmoid(torch.randn((B, S, n), generator=g, device="cuda"))
    hRes = 0.5 * torch.randn((B, S, n, n), generator=g, device="cuda")
    return x, y, hPost.float().contiguous(), hRes.float().contiguous()


def _oracle(x, y, hPost, hRes, dtype):
    B, S, n, D = x.shape
    return ref.mhc_post_ref(_bits(x), _bits(y), hPost.cpu().numpy(), hRes.cpu().numpy(), n, D, dtype)


SHAPES = [
    (1, 64, 4, 7168, "bf16"),   # config 4's row width
    (2, 150, 4, 2560, "fp16"),  # config 2's row width
    (1, 33, 6, 1040, "bf16"),   # D % 64 == 16
    (1, 5, 8, 16, "fp16"),      # one vector per stream
    (1, 300, 8, 4096, "bf16"),  # config 3's row width
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"B{s[0]}S{s[1]}n{s[2]}D{s[3]}{s[4]}")
def test_post_matches_oracle_bit_for_bit(shape):
    B, S, n, D, dtype = shape
    x, y, hPost, hRes = _inputs(B, S, n, D, dtype, seed=sum(shape[:4]))
    out = mp.mhc_post(x, y, hPost, hRes)
    torch.cuda.synchronize()
    want = _oracle(x, y, hPost, hRes, dtype)
    assert np.array_equal(_bits(out).reshape(want.shape), want)


def test_post_in_place_equals_out_of_place():
    x, y, hPost, hRes = _inputs(2, 77, 4, 7168, "bf16", seed=5)
    out = mp.mhc_post(x, y, hPost, hRes)
    xin = x.clone()
    res = mp.mhc_post(xin, y, hPost, hRes, out=xin)
    torch.cuda.synchronize()
    assert res.data_ptr() == xin.data_ptr()
    assert torch.equal(out.view(torch.int16), xin.view(torch.int16))


def test_post_after_mhc_pre_with_an_identity_layer():
    """One layer's residual update: MhcPre, then a layer that returns its input
    (y = hIn), then the post step; the oracle applies the post step to the same
    hIn, hPost and hRes."""
    cfg = CONFIGS["c5_m128_g"]
    inp = make_inputs(cfg)
    hIn, hPost, hRes = mp.mhc_pre(inp["x"], inp["phi"], inp["alpha"], inp["bias"], inp["gamma"])
    xNext = mp.mhc_post(inp["x"], hIn, hPost, hRes)
    torch.cuda.synchronize()
    assert mp.device_status() == 0
    want = _oracle(inp["x"], hIn, hPost, hRes, cfg.dtype)
    assert np.array_equal(_bits(xNext).reshape(want.shape), want)


def test_post_pointer_checks():
    x, y, hPost, hRes = _inputs(1, 8, 4, 256, "bf16", seed=7)
    out = torch.empty_like(x)
    desc = mp.make_desc(1, 8, 4, 256, mp.BF16, False)
    L = mp.lib()
    p = mp._ptr
    s = mp._stream_ptr(None)
    assert L.mhcPostRun(ctypes.byref(desc), p(x), None, p(hPost), p(hRes), p(out), s) == -1
    ybad = ctypes.c_void_p(y.data_ptr() + 2)  # 2-byte offset: not 16-byte aligned
    assert L.mhcPostRun(ctypes.byref(desc), p(x), ybad, p(hPost), p(hRes), p(out), s) == -7
    assert L.mhcPostRun(ctypes.byref(desc), p(x), p(y), p(hPost), p(hRes), p(out), s) == 0
    torch.cuda.synchronize()
