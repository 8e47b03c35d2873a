"""Guard bands around every buffer the operator writes: 4 KiB of a known pattern
before and after hIn, hPost, hRes and the workspace, checked after each path runs
on the boundary and ragged shapes.  A kernel that wrote one element past its
output (or before it) changes a guard byte.  This stands in for a memory checker,
which is not available on this pool."""
from __future__ import annotations

import pytest
import torch

import mhcpre_review_b200 as mp
from mhcpre_review_b200.configs import Config, make_inputs

pytestmark = pytest.mark.gpu

GUARD = 4096  # bytes on each side
PATTERN = 0xA5


class Guarded:
    """Buffers laid out [guard][buf][guard]... in one allocation."""

    def __init__(self, sizes):
        self.sizes = sizes
        offs, o = [], GUARD
        for n in sizes:
            offs.append(o)
            o += (n + 255) // 256 * 256 + GUARD
        self.offs = offs
        self.raw = torch.full((o,), PATTERN, dtype=torch.uint8, device="cuda")

    def view(self, i, dtype, shape):
        n = self.sizes[i]
        return self.raw[self.offs[i]:self.offs[i] + n].view(dtype).view(shape)

    def intact(self):
        mask = torch.ones_like(self.raw, dtype=torch.bool)
        for o, n in zip(self.offs, self.sizes):
            mask[o:o + n] = False
        guards = self.raw[mask]
        return bool((guards == PATTERN).all()), int((guards != PATTERN).sum())


SHAPES = [  # (B, S, n, D, gamma, dtype, path)
    (1, 1, 4, 16, True, "bf16", None),      # decode path
    (1, 7, 6, 16, False, "fp16", None),     # decode path, K not a multiple of 64
    (1, 129, 4, 48, True, "fp16", None),    # small-batch path, one row past a tile
    (3, 100, 8, 32, True, "bf16", None),    # small-batch path, n = 8
    (1, 1000, 6, 80, True, "bf16", None),   # split-K path, ragged tile
    (2, 700, 8, 1040, False, "fp16", None), # split-K path, n = 8
    (1, 1000, 4, 1040, True, "bf16", 5),    # one-pass path, ragged tile and item
    (1, 300, 4, 512, True, "bf16", 1),      # fused team path
    (1, 300, 4, 512, True, "fp16", 3),      # cluster team path
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"B{s[0]}S{s[1]}n{s[2]}D{s[3]}{s[5]}p{s[6]}")
def test_outputs_and_workspace_keep_their_guard_bands(shape, monkeypatch):
    B, S, n, D, g, dt, path = shape
    if path is not None:
        monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=path))
    cfg = Config("canary", B, S, n, D, dt, 0.02, g, seed=61)
    inp = make_inputs(cfg)
    x = inp["x"]
    desc = mp.make_desc(B, S, n, D, mp.BF16 if dt == "bf16" else mp.F16, g)
    if path is not None:
        assert mp.query_plan(desc)["path"] == path
    ws_bytes = mp.workspace_size(desc)
    M = B * S
    gb = Guarded([M * D * 2, M * n * 4, M * n * n * 4, ws_bytes])
    out = (gb.view(0, x.dtype, (B, S, D)), gb.view(1, torch.float32, (B, S, n)),
           gb.view(2, torch.float32, (B, S, n, n)))
    ws = gb.view(3, torch.uint8, (ws_bytes,))
    ex = mp.MhcPre(B, S, n, D, x.dtype, g, workspace=ws)
    ex.prepare(inp["phi"], inp["gamma"])
    for _ in range(2):
        ex(x, inp["alpha"], inp["bias"], out=out)
    torch.cuda.synchronize()
    assert mp.device_status() == 0
    ok, bad = gb.intact()
    assert ok, f"{bad} guard bytes changed"
    # the outputs were written (not left at the guard pattern)
    assert torch.isfinite(out[1]).all() and torch.isfinite(out[2]).all()


POST_PRE_SHAPES = [  # (B, S, n, D, gamma, dtype): the fused kernel (n = 4, D % 64 == 0, > 384 rows) and a fallback
    (1, 1000, 4, 1024, True, "bf16"),   # ragged last tile
    (1, 700, 4, 512, False, "fp16"),
    (1, 600, 6, 512, True, "bf16"),     # n = 6: the two calls
]


@pytest.mark.parametrize("shape", POST_PRE_SHAPES, ids=lambda s: f"B{s[0]}S{s[1]}n{s[2]}D{s[3]}{s[5]}")
def test_post_pre_keeps_the_guard_bands(shape):
    """mhcPostPreRun writes xNext (its TMA stores), the next layer's outputs and the
    records; guard bands around each of them stay intact."""
    B, S, n, D, g, dt = shape
    cfg = Config("canary_pp", B, S, n, D, dt, 0.02, g, seed=62)
    inp = make_inputs(cfg)
    x = inp["x"]
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5)
    y = torch.randn((B, S, D), generator=gen, device="cuda", dtype=x.dtype)
    hPost = torch.rand((B, S, n), generator=gen, device="cuda")
    hRes = (0.5 * torch.randn((B, S, n, n), generator=gen, device="cuda")).contiguous()
    desc = mp.make_desc(B, S, n, D, mp.BF16 if dt == "bf16" else mp.F16, g)
    ws_bytes = mp.workspace_size(desc)
    M = B * S
    gb = Guarded([M * n * D * 2, M * D * 2, M * n * 4, M * n * n * 4, ws_bytes])
    x_next = gb.view(0, x.dtype, (B, S, n, D))
    out = (gb.view(1, x.dtype, (B, S, D)), gb.view(2, torch.float32, (B, S, n)),
           gb.view(3, torch.float32, (B, S, n, n)))
    ws = gb.view(4, torch.uint8, (ws_bytes,))
    ex = mp.MhcPre(B, S, n, D, x.dtype, g, workspace=ws)
    ex.prepare(inp["phi"], inp["gamma"])
    for _ in range(2):
        ex.post_and_run(x, y, hPost, hRes, inp["alpha"], inp["bias"], x_next=x_next, out=out)
    torch.cuda.synchronize()
    assert mp.device_status() == 0
    ok, bad = gb.intact()
    assert ok, f"{bad} guard bytes changed"
    assert torch.isfinite(out[1]).all() and torch.isfinite(out[2]).all()
    assert torch.equal(x_next, mp.mhc_post(x, y, hPost, hRes))
