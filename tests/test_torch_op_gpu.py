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
