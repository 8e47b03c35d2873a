"""MhcPre and the mHC post step as PyTorch custom operators: ``torch.ops.mhc.pre``,
``torch.ops.mhc.post`` and the two fused, ``torch.ops.mhc.post_pre``.

Thin registrations over the C ABI (through :func:`mhcpre_review_b200.mhc_pre`,
:func:`mhcpre_review_b200.mhc_post` and :func:`mhcpre_review_b200.mhc_post_pre`), so that the operators can sit inside torch
code that expects ops: each has a fake (meta) implementation giving the output
shapes and dtypes, and no autograd (the reference operator is forward-only).
Importing this module registers all three.

    import mhcpre_review_b200.torch_ops  # noqa: F401
    hIn, hPost, hRes = torch.ops.mhc.pre(x, phi, alpha, bias, gamma, 1e-6, 1e-6)
    xNext = torch.ops.mhc.post(x, layer_output, hPost, hRes)
    xNext, hIn2, hPost2, hRes2 = torch.ops.mhc.post_pre(x, layer_output, hPost, hRes,
                                                        phi2, alpha2, bias2, gamma2, 1e-6, 1e-6)
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor

from . import mhc_post, mhc_post_pre, mhc_pre


@torch.library.custom_op("mhc::pre", mutates_args=())
def pre(x: Tensor, phi: Tensor, alpha: Tensor, bias: Tensor, gamma: Optional[Tensor] = None,
        norm_eps: float = 1e-6, hc_eps: float = 1e-6) -> tuple[Tensor, Tensor, Tensor]:
    """x [B, S, n, D] fp16/bf16; phi fp32 [mix, n*D]; alpha fp32 [3]; bias fp32 [mix];
    gamma fp32 [n, D] or None.  Returns (hIn [B, S, D], hPost [B, S, n], hRes [B, S, n, n])."""
    return mhc_pre(x, phi, alpha, bias, gamma, norm_eps, hc_eps)


@pre.register_fake
def _pre_fake(x, phi, alpha, bias, gamma=None, norm_eps=1e-6, hc_eps=1e-6):
    B, S, n, D = x.shape
    return (x.new_empty((B, S, D)), x.new_empty((B, S, n), dtype=torch.float32),
            x.new_empty((B, S, n, n), dtype=torch.float32))


@torch.library.custom_op("mhc::post", mutates_args=())
def post(x: Tensor, y: Tensor, hPost: Tensor, hRes: Tensor) -> Tensor:
    """x [B, S, n, D] fp16/bf16 (the streams); y [B, S, D] in x's dtype (the layer
    output); hPost [B, S, n] and hRes [B, S, n, n] fp32.  Returns xNext [B, S, n, D]."""
    return mhc_post(x, y, hPost, hRes)


@post.register_fake
def _post_fake(x, y, hPost, hRes):
    return x.new_empty(x.shape)


@torch.library.custom_op("mhc::post_pre", mutates_args=())
def post_pre(x: Tensor, y: Tensor, hPost: Tensor, hRes: Tensor, phi: Tensor, alpha: Tensor, bias: Tensor,
             gamma: Optional[Tensor] = None, norm_eps: float = 1e-6,
             hc_eps: float = 1e-6) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """The post step of the layer that ends (x, y, hPost, hRes as in mhc::post) fused
    with the next layer's MhcPre (phi, alpha, bias, gamma as in mhc::pre).  Returns
    (xNext [B, S, n, D], hIn [B, S, D], hPost [B, S, n], hRes [B, S, n, n]) of the next layer."""
    x_next, (hIn, hPostN, hResN) = mhc_post_pre(x, y, hPost, hRes, phi, alpha, bias, gamma, norm_eps, hc_eps)
    return x_next, hIn, hPostN, hResN


@post_pre.register_fake
def _post_pre_fake(x, y, hPost, hRes, phi, alpha, bias, gamma=None, norm_eps=1e-6, hc_eps=1e-6):
    B, S, n, D = x.shape
    return (x.new_empty(x.shape), x.new_empty((B, S, D)), x.new_empty((B, S, n), dtype=torch.float32),
            x.new_empty((B, S, n, n), dtype=torch.float32))
