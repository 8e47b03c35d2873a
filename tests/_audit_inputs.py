"""Restatement of the reference audit's input generator, for the golden fixtures.

audit_group_vec.py:259-277 draws every input from a Lehmer generator
(state <- state*48271 mod 2^31-1, value = (state mod 2e6)/1e6 - 1) in this order:
x [rows][n*d] (scaled by 0.5 and rounded to the x dtype), phi [mix][n*d] (x0.1),
gamma [n*d] (1 + 0.1*r, only when present), alpha [3] (x0.2), bias [mix] (x0.2).
"""
from __future__ import annotations

import hashlib
import io
import json
from pathlib import Path

import numpy as np

from oracle.ref import from_float

GOLDEN = Path(__file__).resolve().parent / "golden" / "audit_cases.npz"


def lehmer_values(seed: int, count: int) -> np.ndarray:
    out = np.empty(count, dtype=np.float64)
    state = seed
    for i in range(count):
        state = (state * 48271) % 2147483647
        out[i] = (state % 2000000) / 1000000.0 - 1.0
    return out


def audit_inputs(n: int, d: int, has_gamma: bool, dtype: str, rows: int, seed: int):
    flat = n * d
    mix = n * n + 2 * n
    count = rows * flat + mix * flat + (flat if has_gamma else 0) + 3 + mix
    v = lehmer_values(seed, count)
    pos = 0
    x32 = (v[pos:pos + rows * flat] * 0.5).astype(np.float32); pos += rows * flat
    x_bits = from_float(x32, dtype, audit_carry=True).reshape(rows, flat)
    phi = (v[pos:pos + mix * flat] * 0.1).astype(np.float32).reshape(mix, flat); pos += mix * flat
    gamma = None
    if has_gamma:
        gamma = (1.0 + v[pos:pos + flat] * 0.1).astype(np.float32); pos += flat
    alpha = (v[pos:pos + 3] * 0.2).astype(np.float32); pos += 3
    bias = (v[pos:pos + mix] * 0.2).astype(np.float32); pos += mix
    return x_bits, phi, gamma, alpha, bias


def digest(arr) -> str:
    return hashlib.sha256(np.ascontiguousarray(arr).tobytes()).hexdigest()


def load_golden():
    data = np.load(GOLDEN)
    meta = json.loads(bytes(data["meta_json"]).decode())
    cases = []
    for m in meta:
        i = m["idx"]
        outs = {k: data[f"c{i}_{k}"] for k in ("hIn", "hPost", "hRes", "hPre", "invRms")}
        cases.append((m, outs))
    return cases
