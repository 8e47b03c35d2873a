"""MhcPre benchmark on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c4]

A step is one MhcPre call over one batch of the workload (default: BASELINE
config 4, M = 65536 tokens (B=16, S=4096), n=4, D=7168, bf16, gamma on) with the
weights prepared once beforehand (they are model parameters).  With N GPUs the
batch's tokens are sharded: rank r takes the contiguous rows shard_range(M, N, r)
(phi replicated, no collective on the data path), so the total work is fixed and
scaling is strong; value = M / the slowest rank's device time.  Config 4's inputs
(3.76 GB of x on one GPU, 0.47 GB per GPU at N=8) are larger than the 126 MB L2, so
no flush is needed between steps.  Smaller shards (x under 2x L2, e.g. --config c2)
get a 256 MB L2 flush before every step, outside that step's CUDA events, and the
step time is the sum of the steps' own events.

The JSON line also carries:
  roofline      the main kernel's algorithmic bytes per launch / its average launch
                time (CUDA events recorded around that kernel in a second loop of the
                same steps right after the timed one, inside the same clock-sampled
                region: events between kernels would stop the programmatic dependent
                launches the timed loop uses), against the measured HBM copy
                bandwidth in MEASURED_PEAKS.json; traffic = DRAM bytes per launch from
                the committed ncu summary.
  cpu_baseline  the CPU oracle (a port of the reference's formula) timed on this
                box's host cores on a bounded sample (rank 0, N=1).
  e2e           the same metric through the public API with host buffers: per step,
                pinned host x is copied in, the operator runs, hIn/hPost/hRes are
                copied out (chunked over three streams so copies overlap compute).
  clocks        nvidia-smi samples taken during the timed region.
  configs_2_3_5 (default one-GPU config-4 run only; --no-extra skips it) the other
                BASELINE configs measured in the same run, with their own clock
                samples: configs 2 and 3 (device ms per step, tokens/s, the
                operator's algorithmic GB/s against the measured copy bandwidth and
                8 TB/s, the main kernel's fraction), config 5's p50 latencies (as
                --decode-sweep) and the graph-replay floor of a one-element kernel.
--impl reference times the reference's own CPU formula (the oracle port; the
reference itself is AscendC for Ascend 910B and cannot run here) on all host cores.

    python bench.py --decode-sweep [--steps K]

prints instead one JSON line with BASELINE config 5: the p50 latency of one MhcPre
call for M in {1, 8, 32, 128, 512}, n=4, D=7168, fp16, gamma on and off, with L2
flushed before every call (a 256 MB write) and without the flush.  "graph" is the
call captured once in a CUDA graph and replayed (CUDA events around each replay:
device time only); "eager" is the call itself between the events, so it includes
the host's launch work whenever that is slower than the kernels; "host_us" is the
host time of one eager call.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MhcPre tokens/s & HBM GB/s (% of 8 TB/s), n=4 D=7168 bf16, at 1/2/4/8 B200"
UNIT = "tokens/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c4")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--batch", type=int, default=0, help="override the config's batch (profiling cases)")
    ap.add_argument("--decode-sweep", action="store_true", help="config 5 latency sweep (its own JSON line)")
    ap.add_argument("--post-pre", action="store_true",
                    help="post step + next MhcPre, fused (mhcPostPreRun) against two calls (its own JSON line)")
    ap.add_argument("--post", action="store_true",
                    help="the mHC post step (mhcPostRun) at the config's shape (its own JSON line, one GPU)")
    ap.add_argument("--path", type=int, default=-1, help="plan option: force a path (default: the library's)")
    ap.add_argument("--splits", type=int, default=0, help="plan option: K splits")
    ap.add_argument("--ctas", type=int, default=0, help="plan option: GEMM CTAs per SM")
    ap.add_argument("--stages", type=int, default=0, help="plan option: TMA ring depth")
    ap.add_argument("--ring", type=int, default=0, help="plan option: one-pass record ring slots")
    ap.add_argument("--paired", type=int, default=0,
                    help="plan option: n = 8 GEMM layout (1 one CTA, 2 CTA pairs)")
    ap.add_argument("--epi-blocks", type=int, default=0,
                    help="plan option: split-K epilogue rows resident per SM (12 or 16)")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the configs 2, 3 and 5 measurements the default one-GPU run adds to its line")
    ap.add_argument("--no-flush", action="store_true",
                    help="time small shards with a warm L2 (no flush between steps; not a headline number)")
    return ap.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def committed_traffic(kernel: str, workload: str):
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        return d.get(kernel, {}).get(workload)
    except Exception:
        return None


def scaled_traffic(traffic, rows, total):
    """DRAM bytes per launch from the committed ncu summary (captured on the full
    one-GPU workload), scaled to a shard's rows: the GEMM's traffic is x plus the
    prepared weights, in proportion to the rows."""
    if traffic is None:
        return None
    return int(traffic * rows / total)


class ClockSampler:
    """Samples nvidia-smi every 20 ms during the timed region (the first sample is
    taken before the region starts)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.out = None

    def __enter__(self):
        try:
            self.out = open(f"/tmp/mhc_clocks_{os.getpid()}.csv", "w+")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "20"], stdout=self.out,
                                         stderr=subprocess.DEVNULL)
            # wait (bounded) for the first sample so the timed region is covered
            t0 = time.time()
            while time.time() - t0 < 5.0 and os.path.getsize(self.out.name) == 0 and self.proc.poll() is None:
                time.sleep(0.01)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.out is None:
            return None
        self.out.flush()
        self.out.seek(0)
        rows = [[c.strip() for c in r.split(",")] for r in self.out.read().strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return None

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def time_oracle(cfg, x_bits, phi, alpha, bias, gamma, rows, threads):
    from oracle import ref
    t0 = time.perf_counter()
    ref.mhc_pre_ref(x_bits[:rows], phi, alpha, bias, gamma, cfg.n, cfg.D, cfg.dtype, threads=threads)
    return time.perf_counter() - t0


def host_inputs(cfg):
    """Inputs of the workload on the host (for the CPU runs), generated exactly like
    the GPU run's (same seeds) when a GPU is present, else with numpy."""
    import numpy as np
    try:
        import torch
        if torch.cuda.is_available():
            from mhcpre_review_b200.configs import make_inputs
            inp = make_inputs(cfg)
            xb = inp["x"].reshape(cfg.M, cfg.K).view(torch.int16).cpu().numpy().view(np.uint16)
            g = None if inp["gamma"] is None else inp["gamma"].reshape(-1).cpu().numpy()
            out = (xb, inp["phi"].cpu().numpy(), inp["alpha"].cpu().numpy(), inp["bias"].cpu().numpy(), g)
            del inp
            torch.cuda.empty_cache()
            return out
    except Exception:
        pass
    from oracle import ref
    rng = np.random.default_rng(cfg.seed)
    rows = min(cfg.M, 16384)
    x = ref.from_float(rng.standard_normal((rows, cfg.K), dtype=np.float32), cfg.dtype)
    phi = (rng.standard_normal((cfg.mix, cfg.K)) * cfg.phi_std).astype(np.float32)
    g = (1 + 0.05 * rng.standard_normal(cfg.K)).astype(np.float32) if cfg.gamma else None
    alpha = (0.5 + rng.random(3)).astype(np.float32)
    bias = (0.1 * rng.standard_normal(cfg.mix)).astype(np.float32)
    return x, phi, alpha, bias, g


def cpu_sample_rows(cfg, x, phi, alpha, bias, gamma, threads, target_s=10.0):
    """Rows for a bounded CPU sample of about target_s seconds."""
    probe = min(len(x), 512)
    t = time_oracle(cfg, x, phi, alpha, bias, gamma, probe, threads)
    per_row = max(t / probe, 1e-7)
    return int(max(probe, min(len(x), target_s / per_row)))


# Below this many bytes of x per GPU (2x the 126 MB L2) the timed steps are separated
# by an L2 flush (a 256 MB write, outside the step's CUDA events).
FLUSH_BELOW_BYTES = 252 << 20
FLUSH_BYTES = 256 << 20


def needs_flush(cfg, rows):
    return rows * cfg.K * 2 < FLUSH_BELOW_BYTES


def workload_config(cfg, n_gpus, flushed=None):
    from mhcpre_review_b200.shard import shard_range
    rows = shard_range(cfg.M, n_gpus, 0)[1]
    xgb = rows * cfg.K * 2 / 1e9
    if flushed is None:
        flushed = needs_flush(cfg, rows)
    if flushed:
        l2 = "L2 flushed before every step (a 256 MB write, outside the step's CUDA events; x = %.3f GB per GPU)" % xgb
    elif needs_flush(cfg, rows):
        l2 = "warm L2, no flush (--no-flush; x = %.3f GB per GPU fits in L2): not a headline number" % xgb
    else:
        l2 = "inputs larger than L2 (x = %.2f GB per GPU), no flush" % xgb
    return {"workload": f"{cfg.name}: M={cfg.M} (B={cfg.batch},S={cfg.seq}) in total, n={cfg.n}, D={cfg.D}, "
                        f"{cfg.dtype}, gamma {'on' if cfg.gamma else 'off'}",
            "tokens_per_gpu": rows, "global_tokens": cfg.M, "streams": cfg.n, "head_dim": cfg.D,
            "parallelism": f"token-sharded x{n_gpus} (contiguous rows), phi replicated, no collective",
            "l2": l2}


def run_reference(args, cfg, world, rank):
    """CPU reference arm: the reference formula (oracle port) on all host cores."""
    if rank != 0:
        return
    x, phi, alpha, bias, gamma = host_inputs(cfg)
    threads = cpu_cores()
    rows = cpu_sample_rows(cfg, x, phi, alpha, bias, gamma, threads, target_s=8.0)
    for _ in range(args.warmup):
        time_oracle(cfg, x, phi, alpha, bias, gamma, min(rows, 256), threads)
    times = [time_oracle(cfg, x, phi, alpha, bias, gamma, rows, threads) for _ in range(args.steps)]
    per_step = sum(times) / len(times)
    value = rows / per_step
    sample = f"{rows} of the {cfg.M} rows of {cfg.name} per step (the same rows every step)"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3 * cfg.M / rows,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": cfg.dtype,
        "data": "synthetic (seeded, BASELINE config shapes and distributions)",
        "config": workload_config(cfg, args.gpus),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference operator is AscendC for Ascend 910B; its own CPU formula "
                "(cloud_runner/runner.cpp:122-192, audit_group_vec.py:279-324) is timed via the oracle port",
    }
    print(json.dumps(line), flush=True)


def measure_e2e(mp, inp, cfg, steps, pg, dist, world, total_tokens):
    """Public API with pinned host buffers: H2D x, run, D2H outputs, per step,
    chunked over rows on three streams so the copies overlap the kernels."""
    import torch
    x = inp["x"]
    # chunks of at least 2048 rows, so the H2D copy of one chunk, the operator on the
    # previous one and the D2H copy of the one before overlap (at 1 to 8 GPUs: 8 chunks
    # of 8192 / 4096 / 2048 rows, 4 of 2048 at 8 GPUs)
    chunks = 1
    for c in (8, 4, 2):
        if cfg.M % c == 0 and cfg.M // c >= 2048:
            chunks = c
            break
    rows = cfg.M // chunks
    xh = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    xh.copy_(x)
    hin_h = torch.empty((cfg.batch, cfg.seq, cfg.D), dtype=x.dtype, pin_memory=True)
    post_h = torch.empty((cfg.batch, cfg.seq, cfg.n), dtype=torch.float32, pin_memory=True)
    res_h = torch.empty((cfg.batch, cfg.seq, cfg.n, cfg.n), dtype=torch.float32, pin_memory=True)
    cex = mp.MhcPre(1, rows, cfg.n, cfg.D, x.dtype, cfg.gamma, cfg.norm_eps, cfg.hc_eps)
    cex.prepare(inp["phi"], inp["gamma"])
    xd = torch.empty((2, rows, cfg.n, cfg.D), dtype=x.dtype, device="cuda")
    od = [cex.outputs(x.dtype) for _ in range(2)]
    s_in, s_run, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    xh_r = xh.reshape(cfg.M, cfg.n, cfg.D)
    hin_r, post_r, res_r = hin_h.reshape(cfg.M, cfg.D), post_h.reshape(cfg.M, cfg.n), res_h.reshape(cfg.M, cfg.n, cfg.n)
    h2d = cfg.M * cfg.K * 2
    d2h = cfg.M * cfg.D * 2 + cfg.M * cfg.n * 4 + cfg.M * cfg.n * cfg.n * 4

    def one_step():
        done_out = [None, None]
        for c in range(chunks):
            b = c % 2
            with torch.cuda.stream(s_in):
                if done_out[b] is not None:
                    s_in.wait_event(done_out[b])
                xd[b].copy_(xh_r[c * rows:(c + 1) * rows], non_blocking=True)
                ev_in = torch.cuda.Event()
                ev_in.record(s_in)
            with torch.cuda.stream(s_run):
                s_run.wait_event(ev_in)
                cex(xd[b].reshape(1, rows, cfg.n, cfg.D), inp["alpha"], inp["bias"], out=od[b], stream=s_run)
                ev_run = torch.cuda.Event()
                ev_run.record(s_run)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_run)
                hin_r[c * rows:(c + 1) * rows].copy_(od[b][0].reshape(rows, cfg.D), non_blocking=True)
                post_r[c * rows:(c + 1) * rows].copy_(od[b][1].reshape(rows, cfg.n), non_blocking=True)
                res_r[c * rows:(c + 1) * rows].copy_(od[b][2].reshape(rows, cfg.n, cfg.n), non_blocking=True)
                ev_o = torch.cuda.Event()
                ev_o.record(s_out)
                done_out[b] = ev_o
        torch.cuda.current_stream().wait_stream(s_out)

    one_step()
    torch.cuda.synchronize()
    if pg:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0.record()
    for _ in range(steps):
        one_step()
    t1.record()
    torch.cuda.synchronize()
    t = torch.tensor([t0.elapsed_time(t1) / steps], device="cuda", dtype=torch.float64)
    if pg:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    return {"value": total_tokens / (ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": ms, "chunks": chunks, "pinned_host": True}


def post_step(args):
    """The mHC post step after the layer (mhcPostRun) at the config's shape on one GPU:
    xNext = hRes-mix of x + hPost * y.  Inputs (x, y: 4.7 GB at config 4) are larger
    than L2, so no flush; CUDA events around the K timed calls."""
    import torch
    import mhcpre_review_b200 as mp
    from mhcpre_review_b200.configs import CONFIGS, with_shape
    torch.cuda.set_device(0)
    cfg = CONFIGS[args.config]
    if args.batch > 0:
        cfg = with_shape(cfg, batch=args.batch, name=f"{cfg.name}_b{args.batch}")
    dt = torch.bfloat16 if cfg.dtype == "bf16" else torch.float16
    g = torch.Generator(device="cuda")
    g.manual_seed(cfg.seed * 1000003 + 11)
    x = torch.randn((cfg.batch, cfg.seq, cfg.n, cfg.D), generator=g, device="cuda", dtype=dt)
    y = torch.randn((cfg.batch, cfg.seq, cfg.D), generator=g, device="cuda", dtype=dt)
    hPost = 2.0 * torch.sigmoid(torch.randn((cfg.batch, cfg.seq, cfg.n), generator=g, device="cuda"))
    hRes = 0.5 * torch.randn((cfg.batch, cfg.seq, cfg.n, cfg.n), generator=g, device="cuda")
    out = torch.empty_like(x)
    for _ in range(max(args.warmup, 3)):
        mp.mhc_post(x, y, hPost, hRes, out=out)
    torch.cuda.synchronize()
    b, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        torch.cuda.synchronize()
        b.record()
        for _ in range(args.steps):
            mp.mhc_post(x, y, hPost, hRes, out=out)
        e.record()
        torch.cuda.synchronize()
    if mp.device_status() != 0:
        raise RuntimeError("device status")
    ms = b.elapsed_time(e) / args.steps
    M, n, D = cfg.M, cfg.n, cfg.D
    nbytes = M * n * D * 2 * 2 + M * D * 2 + 4 * M * (n + n * n)
    peak, kind = measured_peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    print(json.dumps({
        "metric": "mHC post step (mhcPostRun) tokens/s and HBM GB/s", "value": M / (ms * 1e-3), "unit": "tokens/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "dtype": cfg.dtype, "data": "synthetic (seeded)",
        "config": {"workload": f"{cfg.name} shape: M={M}, n={n}, D={D}, {cfg.dtype}",
                   "l2": "inputs larger than L2 (x + y = %.2f GB), no flush" % ((M * n * D + M * D) * 2 / 1e9)},
        "gpu_launches": args.steps,
        "roofline": {"bound": "hbm", "kernel": "mhc_post", "achieved": gbs, "peak": peak, "unit": "GB/s",
                     "frac": gbs / peak, "peak_kind": f"{kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "algorithmic_bytes_per_launch": nbytes},
        "clocks": clocks.summary()}), flush=True)


def post_pre_step(args):
    """One layer boundary at the config's shape on one GPU: the post step of the layer
    that ends followed by the next layer's MhcPre, fused (mhcPostPreRun) and as two
    calls (mhcPostRun, then mhcPreRunPrepared), back to back, CUDA events around K
    steps of each.  Reports both times and the bytes each moves: the fused path writes
    xNext once and reads it once; the two calls write it once and read it twice."""
    import torch
    import mhcpre_review_b200 as mp
    from mhcpre_review_b200.configs import CONFIGS, make_inputs, with_shape
    torch.cuda.set_device(0)
    cfg = CONFIGS[args.config]
    if args.batch > 0:
        cfg = with_shape(cfg, batch=args.batch, name=f"{cfg.name}_b{args.batch}")
    inp = make_inputs(cfg)
    x = inp["x"]
    g = torch.Generator(device="cuda")
    g.manual_seed(cfg.seed * 1000003 + 13)
    y = torch.randn((cfg.batch, cfg.seq, cfg.D), generator=g, device="cuda", dtype=x.dtype)
    hPost = (2.0 * torch.sigmoid(torch.randn((cfg.batch, cfg.seq, cfg.n), generator=g, device="cuda"))).contiguous()
    hRes = (0.5 * torch.randn((cfg.batch, cfg.seq, cfg.n, cfg.n), generator=g, device="cuda")).contiguous()
    ex = mp.MhcPre(cfg.batch, cfg.seq, cfg.n, cfg.D, x.dtype, cfg.gamma, cfg.norm_eps, cfg.hc_eps)
    ex.prepare(inp["phi"], inp["gamma"])
    out = ex.outputs(x.dtype)
    xn = torch.empty_like(x)

    def fused():
        ex.post_and_run(x, y, hPost, hRes, inp["alpha"], inp["bias"], x_next=xn, out=out)

    def separate():
        mp.mhc_post(x, y, hPost, hRes, out=xn)
        ex(xn, inp["alpha"], inp["bias"], out=out)

    res = {}
    with ClockSampler(0) as clocks:
        for name, fn in (("separate", separate), ("fused", fused)):
            for _ in range(max(args.warmup, 3)):
                fn()
            torch.cuda.synchronize()
            b, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            b.record()
            for _ in range(args.steps):
                fn()
            e.record()
            torch.cuda.synchronize()
            res[name] = b.elapsed_time(e) / args.steps
    if mp.device_status() != 0:
        raise RuntimeError("device status")
    M, n, D = cfg.M, cfg.n, cfg.D
    xb, yb, hb = M * n * D * 2, M * D * 2, M * D * 2
    coef = M * (n + n * n) * 4
    fused_bytes = (xb + yb + coef + xb) + (xb + hb + coef)       # post in and out; the hIn pass; outputs
    separate_bytes = fused_bytes + xb                             # plus the first MhcPre pass reading xNext
    peak, kind = measured_peaks()
    print(json.dumps({
        "metric": "mHC layer boundary: post step + next MhcPre, fused vs two calls", "unit": "ms per step",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
        "dtype": cfg.dtype, "data": "synthetic (seeded)",
        "config": {"workload": f"{cfg.name} shape: M={M}, n={n}, D={D}, {cfg.dtype}",
                   "l2": "inputs larger than L2, no flush"},
        "fused_ms": res["fused"], "separate_ms": res["separate"], "speedup": res["separate"] / res["fused"],
        "fused_bytes": fused_bytes, "separate_bytes": separate_bytes,
        "fused_GBps_of_its_bytes": fused_bytes / (res["fused"] * 1e-3) / 1e9,
        "separate_GBps_of_its_bytes": separate_bytes / (res["separate"] * 1e-3) / 1e9,
        "peak_GBps": peak, "peak_kind": kind, "clocks": clocks.summary()}), flush=True)


def decode_sweep(args):
    """p50 latency per M, flushed and unflushed L2 (own JSON line)."""
    import torch
    torch.cuda.set_device(0)
    steps = max(args.steps, 20)
    results = decode_latencies(args, steps)
    print(json.dumps({"metric": "MhcPre decode latency (BASELINE config 5)", "unit": "us", "stat": "p50",
                      "steps": steps, "results": results, "graph_replay_floor": graph_replay_floor()}),
          flush=True)


def graph_replay_floor(reps=200):
    """p50 time between CUDA events around the replay of a CUDA graph holding one
    trivial kernel (a one-element add), and around the kernel launched eagerly: the
    launch floor under the config-5 latencies on this box."""
    import torch
    t = torch.zeros(1, device="cuda")
    for _ in range(10):
        t.add_(1)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        t.add_(1)
    out = {}
    for mode, call in (("graph", graph.replay), ("eager", lambda: t.add_(1))):
        for _ in range(10):
            call()
        ts = []
        for _ in range(reps):
            b = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            b.record()
            call()
            e.record()
            torch.cuda.synchronize()
            ts.append(b.elapsed_time(e) * 1e3)
        ts.sort()
        out[f"p50_us_{mode}"] = ts[len(ts) // 2]
    del graph
    return out


def decode_latencies(args, steps):
    """Config 5's p50 latencies: M in {1, 8, 32, 128, 512}, gamma on and off; graph
    replay and eager call, with L2 flushed before every call and warm."""
    import torch
    import mhcpre_review_b200 as mp
    from mhcpre_review_b200.configs import CONFIGS, make_inputs
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    results = []
    for m in (1, 8, 32, 128, 512):
        for g in (True, False):
            cfg = CONFIGS[f"c5_m{m}_{'g' if g else 'ng'}"]
            inp = make_inputs(cfg)
            ex = mp.MhcPre(cfg.batch, cfg.seq, cfg.n, cfg.D, inp["x"].dtype, cfg.gamma, cfg.norm_eps, cfg.hc_eps)
            ex.prepare(inp["phi"], inp["gamma"])
            out = ex.outputs(inp["x"].dtype)
            row = {"M": m, "gamma": g, "plan": ex.plan}
            for _ in range(max(args.warmup, 3)):
                ex(inp["x"], inp["alpha"], inp["bias"], out=out)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(200):
                ex(inp["x"], inp["alpha"], inp["bias"], out=out)
            row["host_us"] = (time.perf_counter() - t0) / 200 * 1e6
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                ex(inp["x"], inp["alpha"], inp["bias"], out=out)
            for mode in ("eager", "graph"):
                call = graph.replay if mode == "graph" else (lambda: ex(inp["x"], inp["alpha"], inp["bias"], out=out))
                for flushed in (True, False):
                    for _ in range(max(args.warmup, 3)):
                        call()
                    ts = []
                    for _ in range(steps):
                        if flushed:
                            flush.fill_(1)
                        b = torch.cuda.Event(enable_timing=True)
                        e = torch.cuda.Event(enable_timing=True)
                        b.record()
                        call()
                        e.record()
                        torch.cuda.synchronize()
                        ts.append(b.elapsed_time(e) * 1e3)
                    ts.sort()
                    row[f"p50_us_{mode}_{'flushed' if flushed else 'warm'}"] = ts[len(ts) // 2]
            del graph
            row["algorithmic_bytes"] = cfg.algorithmic_bytes()
            results.append(row)
            if mp.device_status() != 0:
                raise RuntimeError("device status")
    del flush
    torch.cuda.empty_cache()
    return results


def main_kernel(cfg, plan):
    """The operator's main kernel for a plan and its algorithmic bytes per launch."""
    if plan["path"] == 1:
        return "mhc_pre_fused", cfg.algorithmic_bytes()
    if plan["path"] == 2:
        return "mhc_pre_decode", cfg.algorithmic_bytes()
    if plan["path"] == 3:
        return "mhc_pre_cluster", cfg.algorithmic_bytes()
    if plan["path"] == 4:
        return "mhc_pre_small", cfg.algorithmic_bytes()
    if plan["path"] == 5:
        return "mhc_pre_onepass", cfg.algorithmic_bytes()
    return "gemm_sumsq", cfg.M * cfg.K * 2 + 4 * cfg.K * cfg.mix + (4 * cfg.K if cfg.gamma else 0)


def other_configs(args, peak):
    """BASELINE configs 2 and 3 on this GPU, in the same run as the headline line:
    device time per step from CUDA events (config 2's x fits in L2, so L2 is flushed
    with a 256 MB write before each of its steps, outside the step's events; config
    3's 1.07 GB of x is not), the operator's algorithmic GB/s as a fraction of the
    measured copy bandwidth and of 8 TB/s, and the main kernel's own fraction."""
    import torch
    import mhcpre_review_b200 as mp
    from mhcpre_review_b200.configs import CONFIGS, make_inputs
    res = {}
    steps = max(args.steps, 10)
    for name in ("c2", "c3"):
        cfg = CONFIGS[name]
        inp = make_inputs(cfg)
        x = inp["x"]
        ex = mp.MhcPre(cfg.batch, cfg.seq, cfg.n, cfg.D, x.dtype, cfg.gamma, cfg.norm_eps, cfg.hc_eps)
        ex.prepare(inp["phi"], inp["gamma"])
        out = ex.outputs(x.dtype)
        flush = needs_flush(cfg, cfg.M)
        flush_buf = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda") if flush else None
        for _ in range(max(args.warmup, 3)):
            ex(x, inp["alpha"], inp["bias"], out=out)
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(steps)] for _ in range(4)]
        for e in ev[2] + ev[3]:
            e.record()
        torch.cuda.synchronize()
        if flush:
            # each step alone between events, after its flush
            for i in range(steps):
                flush_buf.fill_(i & 0xFF)
                ev[0][i].record()
                ex(x, inp["alpha"], inp["bias"], out=out)
                ev[1][i].record()
            torch.cuda.synchronize()
            ms = sum(b.elapsed_time(e) for b, e in zip(ev[0], ev[1])) / steps
            # and unflushed: back to back, x warm in L2 (reported beside the number)
            ev[0][0].record()
            for i in range(steps):
                ex(x, inp["alpha"], inp["bias"], out=out)
            ev[1][0].record()
            torch.cuda.synchronize()
            ms_warm = ev[0][0].elapsed_time(ev[1][0]) / steps
        else:
            # back to back, as the headline loop
            ev[0][0].record()
            for i in range(steps):
                ex(x, inp["alpha"], inp["bias"], out=out)
            ev[1][0].record()
            torch.cuda.synchronize()
            ms = ev[0][0].elapsed_time(ev[1][0]) / steps
            ms_warm = None
        # the main kernel's launch times (a loop of its own: see main())
        for i in range(steps):
            if flush:
                flush_buf.fill_(i & 0xFF)
            ex.run_profiled(x, inp["alpha"], inp["bias"], out, ev[2][i], ev[3][i])
        torch.cuda.synchronize()
        if mp.device_status() != 0:
            raise RuntimeError(f"device status after {name}")
        kms = sum(b.elapsed_time(e) for b, e in zip(ev[2], ev[3])) / steps
        plan = ex.plan
        kernel, kbytes = main_kernel(cfg, plan)
        op_gbs = cfg.algorithmic_bytes() / (ms * 1e-3) / 1e9
        k_gbs = kbytes / (kms * 1e-3) / 1e9
        res[name] = {
            "workload": f"M={cfg.M} (B={cfg.batch},S={cfg.seq}), n={cfg.n}, D={cfg.D}, {cfg.dtype}, "
                        f"gamma {'on' if cfg.gamma else 'off'}",
            "ms_per_step": ms, "tokens_per_s": cfg.M / (ms * 1e-3), "steps": steps, "plan": plan,
            "l2": "flushed before every step" if flush else "inputs larger than L2, no flush",
            "ms_per_step_unflushed": ms_warm,
            "algorithmic_bytes": cfg.algorithmic_bytes(), "op_GBps": op_gbs, "op_frac_of_measured": op_gbs / peak,
            "op_frac_of_8TBps": op_gbs / 8000.0,
            "main_kernel": {"kernel": kernel, "launch_ms": kms, "achieved_GBps": k_gbs, "frac": k_gbs / peak,
                            "algorithmic_bytes_per_launch": kbytes}}
        del inp, x, ex, out, flush_buf
        torch.cuda.empty_cache()
    return res


def main():
    args = parse()
    if args.decode_sweep:
        decode_sweep(args)
        return
    if args.post:
        post_step(args)
        return
    if args.post_pre:
        post_pre_step(args)
        return
    world, rank, local = dist_env()
    from mhcpre_review_b200.configs import CONFIGS, with_shape as _ws
    cfg = CONFIGS[args.config]
    if args.batch > 0:
        cfg = _ws(cfg, batch=args.batch, name=f"{cfg.name}_b{args.batch}")
    if world > 1:
        args.gpus = world

    if args.impl == "reference":
        run_reference(args, cfg, world, rank)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    pg = False
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
        pg = True

    import mhcpre_review_b200 as mp
    from mhcpre_review_b200.configs import make_inputs, with_shape
    if args.path >= 0 or args.splits or args.ctas or args.stages or args.ring or args.epi_blocks or args.paired:
        mp._OPTIONS = mp.make_plan_options(path=args.path, splits=args.splits, gemm_ctas_per_sm=args.ctas,
                                           gemm_stages=args.stages, ring_tiles=args.ring, epi_blocks=args.epi_blocks,
                                           paired_gemm=args.paired)

    # every rank generates the same batch (same seeds) and keeps its contiguous rows;
    # the weights are replicated
    from mhcpre_review_b200.shard import shard_range
    total = cfg.M
    start, rows = shard_range(total, world, rank)
    inp = make_inputs(cfg)
    inp["x"] = inp["x"].reshape(total, cfg.n, cfg.D)[start:start + rows].reshape(1, rows, cfg.n, cfg.D).clone()
    torch.cuda.empty_cache()
    full_cfg = cfg
    cfg = with_shape(cfg, batch=1, seq=rows)  # this rank's shard
    x = inp["x"]
    ex = mp.MhcPre(cfg.batch, cfg.seq, cfg.n, cfg.D, x.dtype, cfg.gamma, cfg.norm_eps, cfg.hc_eps)
    ex.prepare(inp["phi"], inp["gamma"])
    out = ex.outputs(x.dtype)
    plan = ex.plan

    for _ in range(max(args.warmup, 3)):
        ex(x, inp["alpha"], inp["bias"], out=out)
    torch.cuda.synchronize()
    if pg:
        dist.barrier()

    # Small shards (x under 2x L2): flush L2 between steps and time each step alone.
    # Every rank decides from the same shard sizes, so all take the same branch.
    flush = needs_flush(cfg, rows) and not args.no_flush
    flush_buf = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda") if flush else None
    ev_b = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ev_e = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    op_b = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    op_e = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for e in ev_b + ev_e:
        e.record()  # materialise the CUDA events before handing them to the library
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        if pg:
            dist.barrier()
        torch.cuda.synchronize()
        t_start.record()
        for i in range(args.steps):
            if flush:
                flush_buf.fill_(i & 0xFF)
                op_b[i].record()
            ex(x, inp["alpha"], inp["bias"], out=out)
            if flush:
                op_e[i].record()
        t_end.record()
        torch.cuda.synchronize()
        # The main kernel's launch times, for the roofline: the same steps again with
        # CUDA events recorded on the launching stream around that kernel.  This is a
        # loop of its own because an event between two kernels stops the second from
        # launching early as a programmatic dependent of the first: the headline loop
        # above has no events between its kernels (at 8192 rows per GPU, events
        # around every launch cost about 9 us per step).
        for i in range(args.steps):
            if flush:
                flush_buf.fill_(i & 0xFF)
            ex.run_profiled(x, inp["alpha"], inp["bias"], out, ev_b[i], ev_e[i])
        torch.cuda.synchronize()
        if pg:
            dist.barrier()
    ms_total = t_start.elapsed_time(t_end)
    if flush:
        # the steps' own device time, without the flushes between them
        ms_total = sum(b.elapsed_time(e) for b, e in zip(op_b, op_e))
    main_ms = [b.elapsed_time(e) for b, e in zip(ev_b, ev_e)]
    status = mp.device_status()
    if status != 0:
        raise RuntimeError(f"device status {status}")

    t = torch.tensor([ms_total], device="cuda", dtype=torch.float64)
    if pg:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = float(t.item()) / args.steps
    value = total / (ms_step * 1e-3)

    # roofline of the main kernel
    peak, peak_kind = measured_peaks()
    main_avg_ms = sum(main_ms) / len(main_ms)
    kernel, kbytes = main_kernel(cfg, plan)
    achieved = kbytes / (main_avg_ms * 1e-3) / 1e9
    op_gbs = cfg.algorithmic_bytes() / (ms_step * 1e-3) / 1e9
    roofline = {"bound": "hbm", "kernel": kernel, "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                "traffic": scaled_traffic(committed_traffic(kernel, cfg.name), rows, total),
                "algorithmic_bytes_per_launch": kbytes,
                "launch_ms": main_avg_ms, "op_GBps": op_gbs, "op_frac_of_8TBps": op_gbs / 8000.0}

    e2e = None
    if not args.no_e2e:
        del out
        torch.cuda.empty_cache()
        e2e = measure_e2e(mp, inp, cfg, args.e2e_steps, pg, dist, world, total)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        xb, phi, alpha, bias, gamma = host_inputs(cfg)
        threads = cpu_cores()
        rows = cpu_sample_rows(cfg, xb, phi, alpha, bias, gamma, threads, target_s=10.0)
        # repeat the sample until about 10 s of CPU work (the whole workload can be
        # faster than that on many cores)
        secs, passes = 0.0, 0
        while passes < 1 or (secs < 10.0 and passes < 50):
            secs += time_oracle(cfg, xb, phi, alpha, bias, gamma, rows, threads)
            passes += 1
        cpu = {"value": rows * passes / secs, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"first {rows} of the {cfg.M} rows of {cfg.name} (same inputs), {passes} pass(es), "
                         f"{secs:.1f} s"}

    # BASELINE configs 2, 3 and 5 in the same run (one GPU): their own numbers with
    # clocks, kept out of the headline value
    extra = None
    if world == 1 and not args.no_extra and args.config == "c4" and args.batch == 0:
        del x, inp
        torch.cuda.empty_cache()
        with ClockSampler(local) as xclocks:
            extra = {"other_configs": other_configs(args, peak),
                     "c5_decode_latency": {"stat": "p50", "unit": "us",
                                           "results": decode_latencies(args, max(args.steps, 20)),
                                           "graph_replay_floor": graph_replay_floor()}}
        extra["clocks"] = xclocks.summary()

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": cfg.dtype,
            "data": "synthetic (seeded, BASELINE config shapes and distributions)",
            "config": workload_config(full_cfg, world, flushed=flush), "plan": plan,
            "gpu_launches": args.steps * plan["kernels_per_run"],
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks.summary(),
        }
        if extra is not None:
            line["configs_2_3_5"] = extra
        print(json.dumps(line), flush=True)
    if pg:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
