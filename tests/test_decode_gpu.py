"""The single-launch decode kernel (path 2, M <= 32 rows): plan selection, parity
with the CPU oracle over stream counts, dtypes, ragged K-slices and fewer chunks
than SMs, agreement with the split-K path, determinism, repeated launches on one
workspace (the grid barrier's arrival counter carries over between launches), and
CUDA-graph capture and replay."""
from __future__ import annotations

import pytest
import torch

import mhcpre_review_b200 as mp
from mhcpre_review_b200.configs import CONFIGS, Config, make_inputs, with_shape
from tests.test_parity_gpu import RTOL, check_config, run_op

pytestmark = pytest.mark.gpu


def _desc(cfg):
    return mp.make_desc(cfg.batch, cfg.seq, cfg.n, cfg.D, mp.BF16 if cfg.dtype == "bf16" else mp.F16, cfg.gamma)


@pytest.mark.parametrize("m", [1, 8, 16])
def test_decode_plan(m):
    cfg = with_shape(CONFIGS["c5_m8_g"], seq=m)
    plan = mp.query_plan(_desc(cfg))
    assert plan["path"] == 2 and plan["kernels_per_run"] == 1
    assert plan["grid_ctas"] == plan["splits"] == min(torch.cuda.get_device_properties(0).multi_processor_count,
                                                       (cfg.n * cfg.D + 63) // 64)


def test_decode_plan_boundary(monkeypatch):
    base = CONFIGS["c5_m32_g"]
    assert mp.query_plan(_desc(with_shape(base, seq=17)))["path"] == 4  # the small-batch kernel by default
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=2))  # the decode kernel on request, up to 32 rows
    assert mp.query_plan(_desc(base))["path"] == 2
    assert mp.query_plan(_desc(with_shape(base, seq=33)))["path"] == 0


CASES = [
    Config("dec_n4_m3_bf16", 1, 3, 4, 7168, "bf16", 0.005, True, seed=11),
    Config("dec_n6_m17_fp16", 1, 17, 6, 1024, "fp16", 0.01, False, seed=12),
    Config("dec_n8_m32_bf16", 2, 16, 8, 4096, "bf16", 0.005, True, seed=13),
    Config("dec_n8_m5_fp16_outl", 1, 5, 8, 2048, "fp16", 0.01, True, outlier_frac=0.01, outlier_scale=20.0,
           seed=14),
    Config("dec_n4_m7_d7184", 1, 7, 4, 7184, "fp16", 0.005, True, seed=15),      # D % 512 == 16: short last slice
    Config("dec_n6_m9_k_ragged", 1, 9, 6, 1040, "bf16", 0.01, True, seed=17),     # K % 64 == 32: short last chunk
    Config("dec_n4_m2_few_chunks", 1, 2, 4, 256, "bf16", 0.02, False, seed=16),  # 16 chunks < SMs
]


@pytest.mark.parametrize("cfg", CASES, ids=lambda c: c.name)
def test_decode_parity(cfg, monkeypatch):
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=2))  # also above the default range (M <= 16)
    assert mp.query_plan(_desc(cfg))["path"] == 2
    check_config(cfg)


def test_decode_matches_split_k_path(monkeypatch):
    cfg = CONFIGS["c5_m8_g"]
    inp = make_inputs(cfg)
    dec = run_op(inp, use_executor=True)
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=0))
    assert mp.query_plan(_desc(cfg))["path"] == 0
    spl = run_op(inp, use_executor=True)
    for a, b in zip(dec[1:], spl[1:]):
        err = (a.double() - b.double()).abs() / b.double().abs().clamp_min(1.0)
        assert float(err.max()) <= RTOL
    # hIn: both paths round the same fp32 formula once; they differ only where their
    # hPre (last bits) straddle a rounding boundary, or where the stream sum cancels
    # (both are checked against the oracle's budget by the parity tests)
    same = (dec[0].view(torch.int16) == spl[0].view(torch.int16)).float().mean()
    assert float(same) > 0.99


def test_decode_deterministic_and_repeated_launches(monkeypatch):
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=2))
    cfg = CONFIGS["c5_m32_ng"]
    inp = make_inputs(cfg)
    x = inp["x"]
    ex = mp.MhcPre(cfg.batch, cfg.seq, cfg.n, cfg.D, x.dtype, cfg.gamma)
    ex.prepare(inp["phi"], inp["gamma"])
    first = [t.clone() for t in ex(x, inp["alpha"], inp["bias"])]
    out = ex.outputs(x.dtype)
    for _ in range(50):  # every launch adds its grid size to the barrier counter
        ex(x, inp["alpha"], inp["bias"], out=out)
    torch.cuda.synchronize()
    assert mp.device_status() == 0
    for a, b in zip(first, out):
        assert torch.equal(a.view(torch.int16) if a.dtype != torch.float32 else a,
                           b.view(torch.int16) if b.dtype != torch.float32 else b)


def test_decode_cuda_graph_replay():
    cfg = CONFIGS["c5_m1_g"]
    inp = make_inputs(cfg)
    x = inp["x"]
    ex = mp.MhcPre(cfg.batch, cfg.seq, cfg.n, cfg.D, x.dtype, cfg.gamma)
    ex.prepare(inp["phi"], inp["gamma"])
    ref_out = [t.clone() for t in ex(x, inp["alpha"], inp["bias"])]
    out = ex.outputs(x.dtype)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ex(x, inp["alpha"], inp["bias"], out=out)
    for _ in range(5):
        for t in out:
            t.zero_()
        g.replay()
    torch.cuda.synchronize()
    assert mp.device_status() == 0
    for a, b in zip(ref_out, out):
        assert torch.equal(a, b)
