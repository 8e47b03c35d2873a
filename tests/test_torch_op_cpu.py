"""The custom-operator registration loads without a GPU and its fake implementation
gives the reference's output shapes and dtypes (no kernel runs)."""
from __future__ import annotations

import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import mhcpre_review_b200.torch_ops  # noqa: F401


def test_fake_shapes():
    with FakeTensorMode():
        x = torch.empty(2, 3, 4, 64, dtype=torch.bfloat16)
        phi = torch.empty(24, 256)
        hIn, hPost, hRes = torch.ops.mhc.pre(x, phi, torch.empty(3), torch.empty(24), None, 1e-6, 1e-6)
    assert tuple(hIn.shape) == (2, 3, 64) and hIn.dtype == torch.bfloat16
    assert tuple(hPost.shape) == (2, 3, 4) and hPost.dtype == torch.float32
    assert tuple(hRes.shape) == (2, 3, 4, 4) and hRes.dtype == torch.float32


def test_post_fake_shapes():
    with FakeTensorMode():
        x = torch.empty(2, 3, 4, 64, dtype=torch.float16)
        xNext = torch.ops.mhc.post(x, torch.empty(2, 3, 64, dtype=torch.float16), torch.empty(2, 3, 4),
                                   torch.empty(2, 3, 4, 4))
    assert tuple(xNext.shape) == (2, 3, 4, 64) and xNext.dtype == torch.float16


def test_post_pre_fake_shapes():
    with FakeTensorMode():
        x = torch.empty(2, 3, 4, 64, dtype=torch.bfloat16)
        outs = torch.ops.mhc.post_pre(x, torch.empty(2, 3, 64, dtype=torch.bfloat16), torch.empty(2, 3, 4),
                                      torch.empty(2, 3, 4, 4), torch.empty(24, 256), torch.empty(3),
                                      torch.empty(24), None, 1e-6, 1e-6)
    xNext, hIn, hPost, hRes = outs
    assert tuple(xNext.shape) == (2, 3, 4, 64) and xNext.dtype == torch.bfloat16
    assert tuple(hIn.shape) == (2, 3, 64) and hIn.dtype == torch.bfloat16
    assert tuple(hPost.shape) == (2, 3, 4) and hPost.dtype == torch.float32
    assert tuple(hRes.shape) == (2, 3, 4, 4) and hRes.dtype == torch.float32
