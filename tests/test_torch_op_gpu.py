"""torch.ops.mhc.pre and torch.ops.mhc.post: the custom-operator registrations over
the C ABI give the same outputs as the direct bindings, and pass
torch.library.opcheck (schema, fake implementation, dispatch) on the GPU."""
from __future__ import annotations

import pytest
import torch

import mhcpre_review_b200 as mp
import mhcpre_review_b200.torch_ops  # noqa: F401  (registers torch.ops.mhc.pre)
from mhcpre_review_b200.configs import CONFIGS, make_inputs, with_shape

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["c1", "c5_m8_g"])
def test_torch_op_matches_binding(name):
    cfg = CONFIGS[name]
    inp = make_inputs(cfg)
    a = torch.ops.mhc.pre(inp["x"], inp["phi"], inp["alpha"], inp["bias"], inp["gamma"], cfg.norm_eps, cfg.hc_eps)
    b = mp.mhc_pre(inp["x"], inp["phi"], inp["alpha"], inp["bias"], inp["gamma"], cfg.norm_eps, cfg.hc_eps)
    for u, v in zip(a, b):
        assert torch.equal(u, v)


def test_torch_op_opcheck():
    cfg = with_shape(CONFIGS["c2"], seq=64)
    inp = make_inputs(cfg)
    torch.library.opcheck(torch.ops.mhc.pre.default,
                          (inp["x"], inp["phi"], inp["alpha"], inp["bias"], inp["gamma"], 1e-6, 1e-6),
                          test_utils=("test_schema", "test_faketensor"))


def test_torch_post_op_matches_binding_and_opcheck():
    cfg = with_shape(CONFIGS["c2"], seq=64)
    inp = make_inputs(cfg)
    hIn, hPost, hRes = mp.mhc_pre(inp["x"], inp["phi"], inp["alpha"], inp["bias"], inp["gamma"])
    a = torch.ops.mhc.post(inp["x"], hIn, hPost, hRes)
    b = mp.mhc_post(inp["x"], hIn, hPost, hRes)
    assert torch.equal(a, b)
    torch.library.opcheck(torch.ops.mhc.post.default, (inp["x"], hIn, hPost, hRes),
                          test_utils=("test_schema", "test_faketensor"))


@pytest.mark.parametrize("seq", [64, 1024], ids=["two_calls", "fused_kernel"])
def test_torch_post_pre_op_matches_binding_and_opcheck(seq):
    """torch.ops.mhc.post_pre equals the one-shot binding (bit for bit: the same
    path), its xNext equals the post step's, and it passes opcheck."""
    cfg = with_shape(CONFIGS["c2"], seq=seq)
    inp = make_inputs(cfg)
    hIn, hPost, hRes = mp.mhc_pre(inp["x"], inp["phi"], inp["alpha"], inp["bias"], inp["gamma"])
    args = (inp["x"], hIn, hPost, hRes, inp["phi"], inp["alpha"], inp["bias"], inp["gamma"], 1e-6, 1e-6)
    a = torch.ops.mhc.post_pre(*args)
    b_next, b = mp.mhc_post_pre(*args)
    for u, v in zip(a, (b_next, *b)):
        assert torch.equal(u, v)
    assert torch.equal(a[0], mp.mhc_post(inp["x"], hIn, hPost, hRes))
    torch.library.opcheck(torch.ops.mhc.post_pre.default, args, test_utils=("test_schema", "test_faketensor"))
