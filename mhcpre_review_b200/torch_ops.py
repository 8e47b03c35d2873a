"""MhcPre as a PyTorch custom operator: ``torch.ops.mhc.pre``.

A thin registration over the C ABI (through :func:`mhcpre_review_b200.mhc_pre`), so
that the operator can sit inside torch code that expects an op: it has a fake
(meta) implementation giving the output shapes and dtypes, and no autograd (the
reference operator is forward-only).  Importing this module registers the op.

    import mhcpre_review_b200.torch_ops  # noqa: F401
    hIn, hPost, hRes = torch.ops.mhc.pre(x, phi, alpha, bias, gamma, 1e-6, 1e-6)
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor

from . import mhc_pre


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
