"""The single-launch small-batch kernel (path 4: by default 16 < M <= 384 rows, on
request up to 512): plan selection,
parity with the CPU oracle over stream counts, dtypes, ragged last tiles, ragged
K-slices and fewer chunks than SMs, agreement with the split-K path, determinism,
repeated launches on one workspace (one grid barrier per launch on the header's
arrival counter, which also the decode kernel uses), and CUDA-graph capture and
replay."""
from __future__ import annotations

import pytest
import torch

import mhcpre_review_b200 as mp
from mhcpre_review_b200.configs import CONFIGS, Config, make_inputs, with_shape
from tests.test_parity_gpu import RTOL, check_config, run_op

pytestmark = pytest.mark.gpu


def _desc(cfg):
    return mp.make_desc(cfg.batch, cfg.seq, cfg.n, cfg.D, mp.BF16 if cfg.dtype == "bf16" else mp.F16, cfg.gamma)


def _sms():
    return torch.cuda.get_device_properties(0).multi_processor_count


@pytest.mark.parametrize("m", [32, 128])
def test_small_plan(m):
    cfg = CONFIGS[f"c5_m{m}_g"]
    plan = mp.query_plan(_desc(cfg))
    assert plan["path"] == 4 and plan["kernels_per_run"] == 1
    assert plan["grid_ctas"] == plan["splits"] == min(_sms(), (cfg.n * cfg.D + 63) // 64)


def test_small_plan_boundaries(monkeypatch):
    base = CONFIGS["c5_m32_g"]
    assert mp.query_plan(_desc(with_shape(base, seq=16)))["path"] == 2
    assert mp.query_plan(_desc(with_shape(base, seq=17)))["path"] == 4
    assert mp.query_plan(_desc(with_shape(base, seq=384)))["path"] == 4
    assert mp.query_plan(_desc(with_shape(base, seq=385)))["path"] == 0
    # n=8 (N=160): T tiles need T*160 TMEM columns, at most 512: up to 3 tiles
    n8 = Config("n8", 1, 384, 8, 1024, "bf16", 0.01, True)
    assert mp.query_plan(_desc(n8))["path"] == 4
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=4))  # on request up to 512 rows (4 tiles)
    assert mp.query_plan(_desc(with_shape(base, seq=1)))["path"] == 4
    assert mp.query_plan(_desc(with_shape(base, seq=512)))["path"] == 4
    assert mp.query_plan(_desc(with_shape(base, seq=513)))["path"] == 0
    assert mp.query_plan(_desc(with_shape(n8, seq=385)))["path"] == 0


CASES = [
    Config("sm_n4_m33_fp16", 1, 33, 4, 7168, "fp16", 0.005, True, seed=21),          # one ragged tile
    Config("sm_n4_m200_bf16", 2, 100, 4, 2560, "bf16", 0.01, False, seed=22),        # 2 tiles, ragged
    Config("sm_n4_m512_bf16_outl", 1, 512, 4, 4096, "bf16", 0.005, True, outlier_frac=0.01, outlier_scale=20.0,
           seed=23),
    Config("sm_n6_m256_fp16", 1, 256, 6, 1024, "fp16", 0.01, True, seed=24),
    Config("sm_n8_m300_bf16", 3, 100, 8, 1024, "bf16", 0.01, False, seed=25),        # 3 tiles of N=160
    Config("sm_n4_m64_d7184", 1, 64, 4, 7184, "fp16", 0.005, True, seed=26),         # D % 64 == 16
    Config("sm_n6_m40_k_ragged", 1, 40, 6, 1040, "bf16", 0.01, True, seed=27),       # K % 64 == 32
    Config("sm_n4_m96_few_chunks", 1, 96, 4, 256, "bf16", 0.02, False, seed=28),     # 16 chunks < SMs
    Config("sm_n4_m100_long_k", 1, 100, 4, 32768, "bf16", 0.005, True, seed=29),     # 14 chunks per CTA: 4 segments
    Config("sm_n4_m40_one_chunk", 1, 40, 4, 16, "fp16", 0.05, True, seed=30),        # K=64: G=1, empty quarters
    Config("sm_n8_m130_two_chunks", 1, 130, 8, 16, "bf16", 0.05, False, seed=31),    # K=128: G=2, 2 tiles
]


@pytest.mark.parametrize("cfg", CASES, ids=lambda c: c.name)
def test_small_parity(cfg, monkeypatch):
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=4))  # also the 512-row case, above the default range
    assert mp.query_plan(_desc(cfg))["path"] == 4
    check_config(cfg)


def test_small_forced_for_decode_sizes(monkeypatch):
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=4))
    cfg = CONFIGS["c5_m8_g"]
    assert mp.query_plan(_desc(cfg))["path"] == 4
    check_config(cfg)


@pytest.mark.parametrize("name", ["c5_m128_g", "c5_m512_ng"])
def test_small_matches_split_k_path(name, monkeypatch):
    cfg = CONFIGS[name]
    inp = make_inputs(cfg)
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=4))
    assert mp.query_plan(_desc(cfg))["path"] == 4
    small = run_op(inp, use_executor=True)
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=0))
    assert mp.query_plan(_desc(cfg))["path"] == 0
    spl = run_op(inp, use_executor=True)
    for a, b in zip(small[1:], spl[1:]):
        err = (a.double() - b.double()).abs() / b.double().abs().clamp_min(1.0)
        assert float(err.max()) <= RTOL
    # hIn: both paths round the same fp32 formula once; they differ only where their
    # hPre (last bits) straddle a rounding boundary
    same = (small[0].view(torch.int16) == spl[0].view(torch.int16)).float().mean()
    assert float(same) > 0.99


def test_small_deterministic_and_repeated_launches():
    cfg = CONFIGS["c5_m128_ng"]
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


def test_small_and_decode_share_the_barrier_counter(monkeypatch):
    """Decode and small-batch launches interleaved on one workspace: the same
    description has the same grid in both, so the arrival counter stays a multiple
    of it."""
    cfg = CONFIGS["c5_m32_g"]
    inp = make_inputs(cfg)
    x = inp["x"]
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=4))  # the small-batch plan needs the larger workspace
    ex = mp.MhcPre(cfg.batch, cfg.seq, cfg.n, cfg.D, x.dtype, cfg.gamma)
    assert ex.plan["path"] == 4
    ex.prepare(inp["phi"], inp["gamma"])
    ref4 = [t.clone() for t in ex(x, inp["alpha"], inp["bias"])]
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=2))
    assert ex.plan["path"] == 2
    ref2 = [t.clone() for t in ex(x, inp["alpha"], inp["bias"])]
    for _ in range(5):
        monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=2))
        a = [t.clone() for t in ex(x, inp["alpha"], inp["bias"])]
        monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=4))
        b = [t.clone() for t in ex(x, inp["alpha"], inp["bias"])]
        for r, t in zip(ref2, a):
            assert torch.equal(r, t)
        for r, t in zip(ref4, b):
            assert torch.equal(r, t)
    torch.cuda.synchronize()
    assert mp.device_status() == 0
    for r, t in zip(ref2[1:], ref4[1:]):
        err = (r.double() - t.double()).abs() / r.double().abs().clamp_min(1.0)
        assert float(err.max()) <= RTOL


def test_unprepared_workspace_does_not_disturb_the_barrier_counter():
    """A launch whose workspace holds weights prepared for another description
    returns before the grid barrier (status NOT_PREPARED); launches of the prepared
    description on that workspace afterwards still give the same results."""
    cfg = CONFIGS["c5_m128_g"]
    inp = make_inputs(cfg)
    x = inp["x"]
    ex = mp.MhcPre(cfg.batch, cfg.seq, cfg.n, cfg.D, x.dtype, cfg.gamma)
    ex.prepare(inp["phi"], inp["gamma"])
    ref = [t.clone() for t in ex(x, inp["alpha"], inp["bias"])]
    # the same workspace under a description with fewer chunks (a different grid)
    other = with_shape(cfg, seq=100, D=1024)
    oin = make_inputs(other)
    desc = _desc(other)
    assert mp.query_plan(desc)["path"] == 4 and mp.query_plan(desc)["grid_ctas"] == 64
    hIn = torch.empty(other.M, other.D, dtype=x.dtype, device="cuda")
    hPost = torch.empty(other.M, other.n, dtype=torch.float32, device="cuda")
    hRes = torch.empty(other.M, other.n, other.n, dtype=torch.float32, device="cuda")
    rc = mp.lib().mhcPreRunPrepared(mp.ctypes.byref(desc), mp._ptr(oin["x"]), mp._ptr(oin["alpha"]),
                                    mp._ptr(oin["bias"]), mp._ptr(hIn), mp._ptr(hPost), mp._ptr(hRes),
                                    mp._ptr(ex.workspace), mp.ctypes.c_size_t(ex.workspace.numel()), None)
    assert rc == 0
    torch.cuda.synchronize()
    not_prepared = {v: k for k, v in mp.STATUS_NAMES.items()}["NOT_PREPARED"]
    assert mp.device_status() == not_prepared
    out = [t.clone() for t in ex(x, inp["alpha"], inp["bias"])]
    torch.cuda.synchronize()
    assert mp.device_status() == 0
    for r, t in zip(ref, out):
        assert torch.equal(r, t)


def test_small_cuda_graph_replay(monkeypatch):
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=4))
    cfg = CONFIGS["c5_m512_g"]
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
