"""Generate golden MhcPre fixtures from the reference's own Python formula.

The reference's offline audit (audit_group_vec.py) recomputes the whole operator
bit-accurately in fp32 (run_formula_case, audit_group_vec.py:259-333) but returns
nothing.  This script runs that function UNMODIFIED on its own seeded inputs and
captures its local variables at its final ``check`` call (the audit looks ``check``
up as a module global, so wrapping it lets us read the caller's frame).  The
captured outputs (hIn, hPost, hRes, plus hPre and invRms) are saved to
``audit_cases.npz`` with SHA-256 digests of the captured inputs, so the tests can
regenerate the inputs with their own restatement of the audit's Lehmer generator
and prove they are the same bytes.

Run from the repository root, where the reference checkout is available:
    python tests/golden/make_golden.py /path/to/reference
The reference is not needed afterwards: tests read only the .npz.
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# The audit's own case list (audit_group_vec.py:336-345) plus extra shapes run
# through the same function.  (n, d, has_gamma, dtype, rows, seed)
AUDIT_CASES = []
_seed = 20260905
for _n in (4, 6, 8):
    for _dt in ("fp16", "bf16"):
        AUDIT_CASES.append((_n, 16, True, _dt, 36, _seed)); _seed += 1
        AUDIT_CASES.append((_n, 32, False, _dt, 36, _seed)); _seed += 1
AUDIT_CASES.append((8, 1024, True, "fp16", 8, _seed))
EXTRA_CASES = [
    (4, 64, True, "bf16", 20, 777),
    (4, 256, False, "fp16", 12, 4242),
    (6, 48, True, "fp16", 10, 31337),
    (8, 64, False, "bf16", 9, 99),
]


def _load_audit(ref_root: Path):
    spec = importlib.util.spec_from_file_location("audit_group_vec", ref_root / "audit_group_vec.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _bits16(values, dtype):
    a = np.asarray(values, dtype=np.float32)
    if dtype == "bf16":
        u = a.view(np.uint32)
        assert np.all((u & 0xFFFF) == 0), "bf16 value not exactly representable"
        return (u >> 16).astype(np.uint16)
    h = a.astype(np.float16)
    assert np.array_equal(h.astype(np.float32), a), "fp16 value not exactly representable"
    return h.view(np.uint16)


def _digest(arr: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(arr).tobytes()).hexdigest()


def run_case(audit, case):
    n, d, has_gamma, dtype, rows, seed = case
    captured = {}
    orig_check = audit.check

    def capturing_check(cond, msg):
        if msg == "section sizes wrong":
            captured.update(sys._getframe(1).f_locals)
        return orig_check(cond, msg)

    audit.check = capturing_check
    try:
        audit.run_formula_case(n, d, has_gamma, dtype, rows, seed)
    finally:
        audit.check = orig_check
    loc = captured
    x = _bits16(loc["x"], dtype)                                   # [rows, n*d]
    phi = np.asarray(loc["phi"], dtype=np.float32)                 # [mix, n*d]
    gamma = None if loc["gamma"] is None else np.asarray(loc["gamma"], dtype=np.float32)
    alpha = np.asarray(loc["alpha"], dtype=np.float32)
    bias = np.asarray(loc["bias"], dtype=np.float32)
    out = {
        "hIn": _bits16(loc["h_in"], dtype),
        "hPost": np.asarray(loc["h_post"], dtype=np.float32),
        "hRes": np.asarray(loc["h_res"], dtype=np.float32).reshape(rows, n, n),
        "hPre": np.asarray(loc["h_pre"], dtype=np.float32),
        "invRms": np.asarray(loc["inv_rms"], dtype=np.float32),
    }
    digests = {"x": _digest(x), "phi": _digest(phi), "alpha": _digest(alpha), "bias": _digest(bias),
               "gamma": None if gamma is None else _digest(gamma)}
    return out, digests


def main(argv):
    if len(argv) < 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <reference checkout>")
    ref_root = Path(argv[1])
    audit = _load_audit(ref_root)
    # the reference's own known-answer test for its rounding helpers must pass first
    audit._self_test_arith()
    arrays = {}
    meta = []
    for idx, case in enumerate(AUDIT_CASES + EXTRA_CASES):
        out, dig = run_case(audit, case)
        n, d, has_gamma, dtype, rows, seed = case
        for k, v in out.items():
            arrays[f"c{idx}_{k}"] = v
        meta.append({"idx": idx, "n": n, "d": d, "gamma": has_gamma, "dtype": dtype, "rows": rows,
                     "seed": seed, "source": "audit" if idx < len(AUDIT_CASES) else "extra",
                     "digests": dig})
        print(f"case {idx}: n={n} d={d} gamma={has_gamma} {dtype} rows={rows} seed={seed}")
    arrays["meta_json"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(HERE / "audit_cases.npz", **arrays)
    print("wrote", HERE / "audit_cases.npz")


if __name__ == "__main__":
    main(sys.argv)
