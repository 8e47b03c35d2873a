"""Calls on a GPU other than the current one: the binding makes the tensors' device
current for the call (the C ABI plans and launches on the current device), uses that
device's current stream, and restores the previous device afterwards.  Results on
cuda:1 equal those on cuda:0 bit for bit."""
from __future__ import annotations

import pytest
import torch

import mhcpre_review_b200 as mp
from mhcpre_review_b200.configs import CONFIGS, make_inputs, with_shape

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")]


def _to(inp, dev):
    return {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}


@pytest.mark.parametrize("seq", [8, 256, 1024], ids=["decode", "small_batch", "split_k"])
def test_calls_on_another_device(seq):
    torch.cuda.set_device(0)
    cfg = with_shape(CONFIGS["c2"], seq=seq)
    inp0 = make_inputs(cfg)
    inp1 = _to(inp0, "cuda:1")
    outs = {}
    for dev, inp in (("cuda:0", inp0), ("cuda:1", inp1)):
        ex = mp.MhcPre(cfg.batch, cfg.seq, cfg.n, cfg.D, inp["x"].dtype, cfg.gamma, device=dev)
        ex.prepare(inp["phi"], inp["gamma"])
        run = ex(inp["x"], inp["alpha"], inp["bias"])
        one_shot = mp.mhc_pre(inp["x"], inp["phi"], inp["alpha"], inp["bias"], inp["gamma"])
        post = mp.mhc_post(inp["x"], run[0], run[1], run[2])
        assert torch.cuda.current_device() == 0, "the previous device was not restored"
        outs[dev] = [t.cpu() for t in (*run, *one_shot, post)]
    assert mp.device_status() == 0
    for u, v in zip(outs["cuda:0"], outs["cuda:1"]):
        assert torch.equal(u, v)
