"""Parity of the CUDA path with the CPU oracle (and with the reference's own
outputs), called through the C ABI.

Tolerances (stated by the operator's contract):
  hPost, hRes  |got - ref| <= 1e-4 * max(1, |ref|)   (reference's max(1, .) convention,
               cloud_runner/runner.cpp:287)
  hIn          within 1 ulp of the x dtype; an element may differ by more only where
               the stream sum cancels, i.e. |got - ref| <= 1 ulp + 1e-5 * sum_s |hPre_s x_s|
               (hPre carries the GEMM's ~1e-6 relative error into hIn), or where the
               GPU is at least as close as the oracle to the float64 value (within 1
               ulp more; the oracle's sequential fp32 sum is then the less accurate
               side); the exact-match rate must exceed 99%.  Beyond K = 32768 the budget grows with K, because
               fp32 sums over K (the oracle's sequential one included) lose accuracy in
               proportion; there, instead of the exact-match rate against the oracle,
               the GPU must be at least as close to a float64 restatement as the oracle
               is (test_large_head_dims).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import mhcpre_review_b200 as mp
from mhcpre_review_b200.configs import CONFIGS, Config, make_inputs, with_shape
from oracle import ref
from tests._audit_inputs import audit_inputs, load_golden

pytestmark = pytest.mark.gpu

RTOL = ref.RTOL
PARITY_STATS = []  # per-case statistics of compare(), written out by tests/conftest.py


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def np32(t):
    return None if t is None else t.detach().float().cpu().numpy()


def compare(got, x_bits, phi, alpha, bias, gamma, n, D, dtype, label="", norm_eps=1e-6, hc_eps=1e-6):
    """got = (hIn bits [R,D], hPost [R,n], hRes [R,n,n]) for the rows in x_bits; the
    rule is oracle.ref.parity_check (tolerances in this module's docstring).  The
    statistics are kept for the parity report (tests/conftest.py)."""
    stats = ref.parity_check(got, x_bits, phi, alpha, bias, gamma, n, D, dtype, label, norm_eps, hc_eps)
    PARITY_STATS.append(stats)
    return stats


def run_op(inp, use_executor=False):
    x = inp["x"]
    if use_executor:
        B, S, n, D = x.shape
        ex = mp.MhcPre(B, S, n, D, x.dtype, inp["gamma"] is not None)
        ex.prepare(inp["phi"], inp["gamma"])
        out = ex(x, inp["alpha"], inp["bias"])
    else:
        out = mp.mhc_pre(x, inp["phi"], inp["alpha"], inp["bias"], inp["gamma"])
    torch.cuda.synchronize()
    return out


def check_config(cfg: Config, sample_rows: int | None = None, seed: int = 0):
    inp = make_inputs(cfg)
    hIn, hPost, hRes = run_op(inp)
    M, n, D = cfg.M, cfg.n, cfg.D
    if sample_rows is None or sample_rows >= M:
        rows = np.arange(M)
    else:
        rng = np.random.default_rng(seed)
        rows = np.unique(np.concatenate([np.arange(64), np.arange(M - 64, M),
                                         rng.choice(M, sample_rows, replace=False)]))
    if len(rows) == M:
        x_rows = bits(inp["x"].reshape(M, n * D))
        got = (bits(hIn.reshape(M, D)), hPost.reshape(M, n).cpu().numpy(), hRes.reshape(M, n, n).cpu().numpy())
    else:
        idx = torch.as_tensor(rows, device="cuda")
        x_rows = bits(inp["x"].reshape(M, n * D).index_select(0, idx))
        got = (bits(hIn.reshape(M, D).index_select(0, idx)), hPost.reshape(M, n).index_select(0, idx).cpu().numpy(),
               hRes.reshape(M, n, n).index_select(0, idx).cpu().numpy())
    gamma = np32(inp["gamma"])
    stats = compare(got, x_rows, np32(inp["phi"]), np32(inp["alpha"]), np32(inp["bias"]),
                    None if gamma is None else gamma.reshape(-1), n, D, cfg.dtype, cfg.name)
    assert mp.device_status() == 0
    return stats


@pytest.mark.parametrize("name", ["c1", "c2"])
def test_small_configs_all_rows(name):
    check_config(CONFIGS[name])


@pytest.mark.parametrize("name", ["c3", "c4"])
def test_large_configs_all_rows(name):
    """Every row of BASELINE configs 3 and 4 against the oracle (a tile-, split- or
    wave-dependent fault anywhere in the grid shows up)."""
    check_config(CONFIGS[name])


@pytest.mark.parametrize("name", [k for k in CONFIGS if k.startswith("c5_")])
def test_decode_configs(name):
    check_config(CONFIGS[name])


# The reference's E3 shape matrix (cloud_runner/runner.cpp:320-327) with its own
# srand(42) inputs (:368-382): (B, S, n, D, gamma, bf16)
E3 = [(1, 2048, 4, 2560, True, False), (1, 2048, 6, 1024, True, False), (1, 1024, 8, 1024, True, False),
      (1, 2048, 4, 2560, False, False), (1, 2048, 6, 1024, True, True), (1, 1024, 8, 1024, False, True)]


@pytest.mark.parametrize("case", E3, ids=lambda c: f"S{c[1]}n{c[2]}D{c[3]}g{int(c[4])}{'bf16' if c[5] else 'fp16'}")
def test_reference_e3_matrix(case):
    B, S, n, D, has_gamma, is_bf16 = case
    dtype = "bf16" if is_bf16 else "fp16"
    M = B * S
    x32, phi, bias, gamma, alpha = ref.runner_inputs(M, n, D, seed=42)
    xb = ref.from_float(x32, dtype)
    tdt = torch.bfloat16 if is_bf16 else torch.float16
    x = torch.from_numpy(xb.view(np.int16)).view(tdt).reshape(B, S, n, D).cuda()
    g = torch.from_numpy(gamma).cuda() if has_gamma else None
    out = mp.mhc_pre(x, torch.from_numpy(phi).cuda(), torch.from_numpy(alpha).cuda(), torch.from_numpy(bias).cuda(), g)
    torch.cuda.synchronize()
    got = (bits(out[0].reshape(M, D)), out[1].reshape(M, n).cpu().numpy(), out[2].reshape(M, n, n).cpu().numpy())
    compare(got, xb, phi, alpha, bias, gamma if has_gamma else None, n, D, dtype, f"E3{case}")


GOLDEN = load_golden()


@pytest.mark.parametrize("case", GOLDEN, ids=lambda c: f"{c[0]['source']}{c[0]['idx']}")
def test_matches_reference_golden_outputs(case):
    """GPU vs the outputs the reference's own formula code produced."""
    m, gold = case
    n, d, dtype, rows = m["n"], m["d"], m["dtype"], m["rows"]
    xb, phi, gamma, alpha, bias = audit_inputs(n, d, m["gamma"], dtype, rows, m["seed"])
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
    x = torch.from_numpy(xb.view(np.int16)).view(tdt).reshape(1, rows, n, d).cuda()
    out = mp.mhc_pre(x, torch.from_numpy(phi).cuda(), torch.from_numpy(alpha).cuda(), torch.from_numpy(bias).cuda(),
                     None if gamma is None else torch.from_numpy(gamma).cuda())
    torch.cuda.synchronize()
    g_post = out[1].reshape(rows, n).cpu().numpy().astype(np.float64)
    g_res = out[2].reshape(rows, n, n).cpu().numpy().astype(np.float64)
    assert np.max(np.abs(g_post - gold["hPost"]) / np.maximum(1, np.abs(gold["hPost"]))) <= RTOL
    assert np.max(np.abs(g_res - gold["hRes"]) / np.maximum(1, np.abs(gold["hRes"]))) <= RTOL
    d_ulp = ref.ulp_distance(bits(out[0].reshape(rows, d)), gold["hIn"])
    assert (d_ulp <= 1).mean() >= 0.999
    # and against the oracle with the full hIn rule
    compare((bits(out[0].reshape(rows, d)), g_post.astype(np.float32), g_res.astype(np.float32)), xb, phi, alpha,
            bias, gamma, n, d, dtype, f"golden{m['idx']}")


BOUNDARY = [
    (1, 1, 4, 16, True, "bf16"),     # M=1, smallest D
    (1, 7, 6, 16, False, "fp16"),    # n=6: K=96 is not a multiple of the 64-wide K chunk
    (1, 129, 4, 48, True, "fp16"),   # one row past a 128-row tile
    (3, 100, 8, 32, True, "bf16"),   # M=300: ragged last tile, n=8
    (1, 300, 6, 80, True, "bf16"),
    (2, 64, 8, 16, False, "fp16"),
]


@pytest.mark.parametrize("shape", BOUNDARY, ids=lambda s: f"B{s[0]}S{s[1]}n{s[2]}D{s[3]}g{int(s[4])}{s[5]}")
def test_boundary_shapes(shape):
    B, S, n, D, g, dt = shape
    cfg = Config("boundary", B, S, n, D, dt, 0.05, g, seed=11)
    check_config(cfg)


@pytest.mark.parametrize("shape", [s for s in BOUNDARY if s[0] * s[1] <= 32],
                         ids=lambda s: f"B{s[0]}S{s[1]}n{s[2]}D{s[3]}g{int(s[4])}{s[5]}")
def test_boundary_shapes_split_k_path(shape, monkeypatch):
    """The smallest shapes run a single-launch kernel by default; the split-K path
    must handle them too (one 64-wide chunk or a partial one, one ragged row tile)."""
    monkeypatch.setattr(mp, "_OPTIONS", mp.make_plan_options(path=0))
    B, S, n, D, g, dt = shape
    cfg = Config("boundary_splitk", B, S, n, D, dt, 0.05, g, seed=12)
    assert mp.query_plan(mp.make_desc(B, S, n, D, mp.BF16 if dt == "bf16" else mp.F16, g))["path"] == 0
    check_config(cfg)


LARGE_D = [
    Config("large_d_decode", 1, 3, 4, 32768, "bf16", 0.005, True, seed=21),     # K = 131072 on the decode path
    Config("large_d_splitk", 1, 200, 8, 16384, "fp16", 0.002, False, seed=22),  # K = 131072, mix 80, split-K
    Config("large_d_n6", 1, 150, 6, 16400, "bf16", 0.002, True, seed=23),       # D % 64 == 16
]


@pytest.mark.parametrize("cfg", LARGE_D, ids=lambda c: c.name)
def test_large_head_dims(cfg):
    check_config(cfg)
    # accuracy against a float64 restatement: no worse than the oracle's own
    inp = make_inputs(cfg)
    hIn, hPost, _ = run_op(inp)
    M, n, D = cfg.M, cfg.n, cfg.D
    xb = bits(inp["x"].reshape(M, n * D))
    gamma = np32(inp["gamma"])
    g = None if gamma is None else gamma.reshape(-1)
    h64, post64, _, _ = ref.mhc_pre_numpy(xb, np32(inp["phi"]), np32(inp["alpha"]), np32(inp["bias"]), g, n, D,
                                          cfg.dtype)
    o_in, o_post, _ = ref.mhc_pre_ref(xb, np32(inp["phi"]), np32(inp["alpha"]), np32(inp["bias"]), g, n, D,
                                      cfg.dtype)
    r64 = ref.from_float(h64.astype(np.float32), cfg.dtype)
    d_gpu = ref.ulp_distance(bits(hIn.reshape(M, D)), r64)
    d_oracle = ref.ulp_distance(o_in, r64)
    assert d_gpu.max() <= max(d_oracle.max(), 1) + 1, (d_gpu.max(), d_oracle.max())
    assert (d_gpu == 0).mean() >= (d_oracle == 0).mean() - 0.002, ((d_gpu == 0).mean(), (d_oracle == 0).mean())
    gpu_post = np.abs(hPost.reshape(M, n).cpu().numpy() - post64).max()
    oracle_post = np.abs(o_post - post64).max()
    assert gpu_post <= 2 * oracle_post + 1e-6, (gpu_post, oracle_post)


def test_relaunch_is_idempotent_and_matches_one_shot():
    """E2 analogue (cloud_runner/probe_e1e2.cpp:312-326): relaunching a prepared
    executor gives bit-identical outputs, equal to the one-shot call."""
    cfg = with_shape(CONFIGS["c2"], seq=512)
    inp = make_inputs(cfg)
    B, S, n, D = inp["x"].shape
    ex = mp.MhcPre(B, S, n, D, inp["x"].dtype, True)
    ex.prepare(inp["phi"], inp["gamma"])
    a = ex(inp["x"], inp["alpha"], inp["bias"])
    b = ex(inp["x"], inp["alpha"], inp["bias"])
    c = mp.mhc_pre(inp["x"], inp["phi"], inp["alpha"], inp["bias"], inp["gamma"])
    torch.cuda.synchronize()
    for u, v, w in zip(a, b, c):
        assert torch.equal(u, v) and torch.equal(u, w)
    assert mp.device_status() == 0


def test_row_shards_are_bitwise_consistent():
    """Rows are independent and, from 8192 rows up, the launch plan depends on K
    only: two halves run separately reproduce the full run bit for bit (what token
    sharding across GPUs relies on)."""
    cfg = with_shape(CONFIGS["c4"], batch=2, seq=8192)
    inp = make_inputs(cfg)
    full = run_op(inp)
    x = inp["x"]
    halves = [run_op(dict(inp, x=x[i:i + 1].contiguous())) for i in range(2)]
    for k in range(3):
        assert torch.equal(full[k], torch.cat([h[k] for h in halves], dim=0))


def test_gamma_folding_equivalence():
    """gamma is folded into phi in fp32; passing gamma*phi with no gamma is bitwise
    identical (the fold is a single fp32 multiply either way)."""
    cfg = with_shape(CONFIGS["c2"], seq=256)
    inp = make_inputs(cfg)
    a = run_op(inp)
    phi_g = (inp["phi"] * inp["gamma"].reshape(1, -1)).contiguous()
    b = run_op(dict(inp, phi=phi_g, gamma=None))
    for u, v in zip(a, b):
        assert torch.equal(u, v)


def test_error_paths_on_device():
    cfg = with_shape(CONFIGS["c1"], seq=16)
    inp = make_inputs(cfg)
    B, S, n, D = inp["x"].shape
    desc = mp.make_desc(B, S, n, D, mp.F16, False)
    need = mp.workspace_size(desc)
    small = torch.empty(need - 256, dtype=torch.uint8, device="cuda")
    with pytest.raises(mp.MhcPreError) as ei:
        mp.mhc_pre(inp["x"], inp["phi"], inp["alpha"], inp["bias"], None, workspace=small)
    assert ei.value.status == -8
    # x misaligned by one element
    buf = torch.empty(inp["x"].numel() + 8, dtype=inp["x"].dtype, device="cuda")
    xm = buf[1:1 + inp["x"].numel()].view(inp["x"].shape)
    with pytest.raises(mp.MhcPreError) as ei:
        mp.mhc_pre(xm, inp["phi"], inp["alpha"], inp["bias"], None)
    assert ei.value.status == -7
    assert mp.device_status() == 0


@pytest.mark.parametrize("seq", [4, 64, 1024], ids=["decode_path", "small_batch_path", "split_k_path"])
def test_weights_prepared_for_another_shape_are_refused(seq):
    """A workspace holds weights prepared for one (n, D, dtype, gamma); running a
    different description on it must not compute silently with them: the kernels
    compare the prepared signature and report MHC_STATUS_NOT_PREPARED."""
    cfg_a = Config("sig_a", 1, seq, 4, 256, "bf16", 0.02, True, seed=31)
    cfg_b = Config("sig_b", 1, seq, 4, 512, "bf16", 0.02, True, seed=32)
    ia, ib = make_inputs(cfg_a), make_inputs(cfg_b)
    da = mp.make_desc(1, seq, 4, 256, mp.BF16, True)
    db = mp.make_desc(1, seq, 4, 512, mp.BF16, True)
    ws = torch.zeros(max(mp.workspace_size(da), mp.workspace_size(db)), dtype=torch.uint8, device="cuda")
    ex_a = mp.MhcPre(1, seq, 4, 256, torch.bfloat16, True, workspace=ws)
    ex_a.prepare(ia["phi"], ia["gamma"])
    ex_b = mp.MhcPre(1, seq, 4, 512, torch.bfloat16, True, workspace=ws)
    ex_b(ib["x"], ib["alpha"], ib["bias"])  # never prepared for D=512
    assert mp.device_status() == -12  # MHC_STATUS_NOT_PREPARED
    ex_b.prepare(ib["phi"], ib["gamma"])
    ex_b(ib["x"], ib["alpha"], ib["bias"])
    assert mp.device_status() == 0


def test_full_size_c4_output_properties():
    """Size-independent properties at the full BASELINE config 4 size."""
    cfg = CONFIGS["c4"]
    inp = make_inputs(cfg)
    hIn, hPost, hRes = run_op(inp)
    assert torch.isfinite(hIn.float()).all()
    assert ((hPost > 0) & (hPost < 2)).all()
    assert torch.isfinite(hRes).all()
    # hRes - bias is linear in alpha[2]: doubling alpha[2] doubles it (to fp32 rounding)
    a2 = inp["alpha"].clone()
    a2[2] *= 2
    _, _, hRes2 = run_op(dict(inp, alpha=a2))
    b = inp["bias"][2 * cfg.n:].reshape(cfg.n, cfg.n)
    lhs = (hRes2 - b).double()
    rhs = 2 * (hRes - b).double()
    assert torch.allclose(lhs, rhs, rtol=1e-5, atol=1e-6)
