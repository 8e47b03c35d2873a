"""Python front end of the CPU oracle for MhcPre -- TEST INFRASTRUCTURE ONLY.

``mhc_pre_ref`` calls the C restatement in ``mhc_pre_oracle.c`` (see its header for
the formula and the reference lines it follows).  ``mhc_pre_numpy`` is an
independent float64 restatement used to cross-check the C oracle: it follows
cloud_runner/runner.cpp:122-192 (double square-sum) with float64 everywhere
else, so it is "truth" up to the final fp32/16-bit rounding of the outputs.

x and hIn are 16-bit patterns (np.uint16) of the x dtype ("fp16" or "bf16").
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "libmhc_oracle.so"
_lib = None

ORDER_KERNEL = 0
ORDER_AUDIT = 1
DTYPE_CODE = {"fp16": 0, "bf16": 1}


def build(force: bool = False) -> Path:
    """Compile the C oracle in place (gcc + OpenMP)."""
    srcs = [_HERE / "mhc_pre_oracle.c", _HERE / "mhc_post_oracle.c", _HERE / "mhc_pre_oracle.h"]
    if force or not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < max(s.stat().st_mtime for s in srcs):
        subprocess.check_call(["make", "-s", "-C", str(_HERE), "libmhc_oracle.so"])
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        lib = ctypes.CDLL(str(_LIB_PATH))
        u16p = ctypes.POINTER(ctypes.c_uint16)
        f32p = ctypes.POINTER(ctypes.c_float)
        lib.mhc_pre_oracle.restype = ctypes.c_int
        lib.mhc_pre_oracle.argtypes = [
            ctypes.c_int64, ctypes.c_int, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
            u16p, f32p, f32p, f32p, f32p, ctypes.c_float, ctypes.c_float,
            u16p, f32p, f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int]
        lib.mhc_oracle_f32_to_f16.restype = ctypes.c_uint16
        lib.mhc_oracle_f32_to_f16.argtypes = [ctypes.c_float]
        lib.mhc_oracle_f32_to_f16_audit.restype = ctypes.c_uint16
        lib.mhc_oracle_f32_to_f16_audit.argtypes = [ctypes.c_float]
        lib.mhc_oracle_f32_to_bf16.restype = ctypes.c_uint16
        lib.mhc_oracle_f32_to_bf16.argtypes = [ctypes.c_float]
        lib.mhc_oracle_f16_to_f32.restype = ctypes.c_float
        lib.mhc_oracle_f16_to_f32.argtypes = [ctypes.c_uint16]
        lib.mhc_oracle_bf16_to_f32.restype = ctypes.c_float
        lib.mhc_oracle_bf16_to_f32.argtypes = [ctypes.c_uint16]
        lib.mhc_oracle_max_threads.restype = ctypes.c_int
        lib.mhc_post_oracle.restype = ctypes.c_int
        lib.mhc_post_oracle.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_int64, ctypes.c_int, u16p, u16p,
                                        f32p, f32p, u16p, ctypes.c_int]
        lib.mhc_oracle_runner_inputs.restype = None
        lib.mhc_oracle_runner_inputs.argtypes = [ctypes.c_uint, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                                 ctypes.c_int64, f32p, f32p, f32p, f32p]
        _lib = lib
    return _lib


def _ptr(a: np.ndarray, ctype):
    return a.ctypes.data_as(ctypes.POINTER(ctype))


def runner_inputs(M: int, n: int, D: int, seed: int = 42):
    """The reference E3 runner's inputs (cloud_runner/runner.cpp:368-382) as fp32
    arrays: x [M, n*D], phi [mix, n*D], bias [mix], gamma [n*D], alpha [3]."""
    lib = _load()
    K = n * D
    mix = n * n + 2 * n
    x = np.empty(M * K, np.float32)
    phi = np.empty(mix * K, np.float32)
    bias = np.empty(mix, np.float32)
    gamma = np.empty(K, np.float32)
    f = ctypes.c_float
    lib.mhc_oracle_runner_inputs(seed, x.size, phi.size, bias.size, gamma.size, _ptr(x, f), _ptr(phi, f),
                                 _ptr(bias, f), _ptr(gamma, f))
    alpha = np.array([0.5, 0.3, 0.2], np.float32)
    return x.reshape(M, K), phi.reshape(mix, K), bias, gamma, alpha


def max_threads() -> int:
    return int(_load().mhc_oracle_max_threads())


def f32_to_f16_bits(v: float) -> int:
    return int(_load().mhc_oracle_f32_to_f16(ctypes.c_float(v)))


def f32_to_bf16_bits(v: float) -> int:
    return int(_load().mhc_oracle_f32_to_bf16(ctypes.c_float(v)))


def f16_bits_to_f32(b: int) -> float:
    return float(_load().mhc_oracle_f16_to_f32(b))


def bf16_bits_to_f32(b: int) -> float:
    return float(_load().mhc_oracle_bf16_to_f32(b))


def to_float(bits: np.ndarray, dtype: str) -> np.ndarray:
    """Decode 16-bit patterns to float32 (vectorised, exact)."""
    bits = np.asarray(bits, dtype=np.uint16)
    if dtype == "bf16":
        return (bits.astype(np.uint32) << 16).view(np.float32)
    return bits.view(np.float16).astype(np.float32)


def from_float(values: np.ndarray, dtype: str, audit_carry: bool = False) -> np.ndarray:
    """Round float32 values to 16-bit patterns, IEEE nearest even (vectorised).

    audit_carry=True reproduces the reference helper's fp16 quirk
    (audit_group_vec.py:181): a subnormal that rounds up to the smallest normal
    (2^-14) becomes zero."""
    v = np.ascontiguousarray(values, dtype=np.float32)
    if dtype == "bf16":
        u = v.view(np.uint32).astype(np.uint64)
        lsb = (u >> 16) & 1
        return (((u + 0x7FFF + lsb) & 0xFFFF0000) >> 16).astype(np.uint16)
    b = v.astype(np.float16).view(np.uint16)
    if audit_carry:
        carried = ((b & 0x7FFF) == 0x0400) & (np.abs(v) < np.float32(2.0 ** -14))
        b = np.where(carried, b & 0x8000, b).astype(np.uint16)
    return b


def mhc_pre_ref(x_bits, phi, alpha, bias, gamma, n: int, D: int, dtype: str,
                norm_eps: float = 1e-6, hc_eps: float = 1e-6, order: int = ORDER_KERNEL,
                rows: tuple[int, int] | None = None, threads: int = 0):
    """Run the C oracle.  x_bits: uint16 [M, n, D] (or [M, n*D]); phi: float32 [mix, n*D].

    Returns (hIn_bits uint16 [R, D], hPost float32 [R, n], hRes float32 [R, n, n]) for
    rows [r0, r1) (all rows by default)."""
    lib = _load()
    K = n * D
    mix = n * n + 2 * n
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16).reshape(-1, K)
    M = x_bits.shape[0]
    phi = np.ascontiguousarray(phi, dtype=np.float32).reshape(mix, K)
    alpha = np.ascontiguousarray(alpha, dtype=np.float32).reshape(3)
    bias = np.ascontiguousarray(bias, dtype=np.float32).reshape(mix)
    g = None if gamma is None else np.ascontiguousarray(gamma, dtype=np.float32).reshape(K)
    r0, r1 = (0, M) if rows is None else rows
    hIn = np.zeros((M, D), dtype=np.uint16)
    hPost = np.zeros((M, n), dtype=np.float32)
    hRes = np.zeros((M, n, n), dtype=np.float32)
    f32p = ctypes.c_float
    rc = lib.mhc_pre_oracle(
        M, n, D, DTYPE_CODE[dtype], order,
        _ptr(x_bits, ctypes.c_uint16), _ptr(phi, f32p), _ptr(alpha, f32p), _ptr(bias, f32p),
        None if g is None else _ptr(g, f32p), norm_eps, hc_eps,
        _ptr(hIn, ctypes.c_uint16), _ptr(hPost, f32p), _ptr(hRes, f32p), r0, r1, threads)
    if rc != 0:
        raise RuntimeError(f"mhc_pre_oracle failed with code {rc}")
    return hIn[r0:r1], hPost[r0:r1], hRes[r0:r1]


def mhc_post_ref(x_bits, y_bits, hPost, hRes, n: int, D: int, dtype: str, threads: int = 0):
    """The mHC post step in the library's operation order (C oracle; parity
    unpinned: the reference has no such step).  x_bits: uint16 [M, n, D] (or
    [M, n*D]); y_bits: uint16 [M, D]; hPost float32 [M, n]; hRes float32 [M, n, n].
    Returns xNext bits uint16 [M, n, D]."""
    lib = _load()
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16).reshape(-1, n, D)
    M = x_bits.shape[0]
    y_bits = np.ascontiguousarray(y_bits, dtype=np.uint16).reshape(M, D)
    hPost = np.ascontiguousarray(hPost, dtype=np.float32).reshape(M, n)
    hRes = np.ascontiguousarray(hRes, dtype=np.float32).reshape(M, n, n)
    out = np.zeros((M, n, D), dtype=np.uint16)
    rc = lib.mhc_post_oracle(M, n, D, DTYPE_CODE[dtype], _ptr(x_bits, ctypes.c_uint16), _ptr(y_bits, ctypes.c_uint16),
                             _ptr(hPost, ctypes.c_float), _ptr(hRes, ctypes.c_float), _ptr(out, ctypes.c_uint16),
                             threads)
    if rc != 0:
        raise RuntimeError(f"mhc_post_oracle failed with code {rc}")
    return out


def mhc_post_numpy(x_bits, y_bits, hPost, hRes, n: int, D: int, dtype: str):
    """Float64 restatement of the post step (independent of the C oracle's operation
    order), returned unrounded: float64 [M, n, D]."""
    x = to_float(np.asarray(x_bits, dtype=np.uint16), dtype).astype(np.float64).reshape(-1, n, D)
    y = to_float(np.asarray(y_bits, dtype=np.uint16), dtype).astype(np.float64).reshape(x.shape[0], D)
    hPost = np.asarray(hPost, dtype=np.float64).reshape(-1, n)
    hRes = np.asarray(hRes, dtype=np.float64).reshape(-1, n, n)
    return np.einsum("mst,mtd->msd", hRes, x) + hPost[:, :, None] * y[:, None, :]


def mhc_pre_numpy(x_bits, phi, alpha, bias, gamma, n: int, D: int, dtype: str,
                  norm_eps: float = 1e-6, hc_eps: float = 1e-6):
    """float64 restatement (vectorised over rows); returns float64 hIn (before the
    16-bit rounding), hPost, hRes and hPre."""
    K = n * D
    mix = n * n + 2 * n
    xf = to_float(np.asarray(x_bits).reshape(-1, K), dtype).astype(np.float64)
    sumsq = (xf * xf).sum(axis=1)
    inv_rms = 1.0 / np.sqrt(sumsq / K + norm_eps)
    xg = xf * (np.asarray(gamma, np.float64).reshape(1, K) if gamma is not None else 1.0)
    mixv = xg @ np.asarray(phi, np.float64).reshape(mix, K).T
    scaled = mixv * inv_rms[:, None]
    a = np.asarray(alpha, np.float64)
    b = np.asarray(bias, np.float64)
    h_pre = 1.0 / (1.0 + np.exp(-(scaled[:, :n] * a[0] + b[:n]))) + hc_eps
    h_post = 2.0 / (1.0 + np.exp(-(scaled[:, n:2 * n] * a[1] + b[n:2 * n])))
    h_res = (scaled[:, 2 * n:] * a[2] + b[2 * n:]).reshape(-1, n, n)
    xs = xf.reshape(-1, n, D)
    h_in = np.einsum("rs,rsd->rd", h_pre, xs)
    return h_in, h_post, h_res, h_pre


def ulp_size(bits: np.ndarray, dtype: str) -> np.ndarray:
    """Spacing between the magnitude of each 16-bit value and the next larger one."""
    mag = np.asarray(bits, dtype=np.uint16) & 0x7FFF
    top = 0x7BFF if dtype == "fp16" else 0x7F7F
    lo = np.minimum(mag, top - 1).astype(np.uint16)
    hi = (lo + 1).astype(np.uint16)
    return (to_float(hi, dtype).astype(np.float64) - to_float(lo, dtype).astype(np.float64))


def ulp_distance(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """Distance in units of the last place between two arrays of 16-bit float
    patterns (fp16 or bf16: both are sign-magnitude with the exponent above the
    mantissa, so ordering the magnitudes works for either)."""
    def ordered(bits):
        b = np.asarray(bits, dtype=np.uint16).astype(np.int32)
        mag = b & 0x7FFF
        return np.where(b & 0x8000, -mag, mag)
    return np.abs(ordered(a_bits) - ordered(b_bits))


# Tolerances of the operator's contract, shared by the GPU parity tests and the
# driver's smoke check.
RTOL = 1e-4          # hPost, hRes: |got - ref| <= RTOL * max(1, |ref|)
HIN_BUDGET = 1e-5    # hIn beyond 1 ulp: <= 1 ulp + HIN_BUDGET * sum_s |hPre_s x_s|
HIN_EXACT_MIN = 0.99  # hIn exact-match rate against the oracle (K <= 32768)


def parity_check(got, x_bits, phi, alpha, bias, gamma, n: int, D: int, dtype: str, label: str = "",
                 norm_eps: float = 1e-6, hc_eps: float = 1e-6) -> dict:
    """Checks a result against the oracle with the contract's tolerances and returns
    the statistics.  got = (hIn bits [R, D], hPost [R, n], hRes [R, n, n]) for the
    rows in x_bits [R, n*D].

    hPost, hRes: |got - ref| <= 1e-4 * max(1, |ref|) (the reference's max(1, .)
    convention, cloud_runner/runner.cpp:287).  hIn: within 1 ulp of the x dtype; an
    element may differ by more only where the stream sum cancels, i.e. |got - ref| <=
    1 ulp + 1e-5 * sum_s |hPre_s x_s| (hPre carries the GEMM's ~1e-6 relative error
    into hIn), or where got is at least as close as the oracle to the float64 value
    sum_s hPre64_s x_s (within 1 ulp more): both are fp32 approximations, and where the
    oracle's own sequential fp32 sum over K is the less accurate one, the difference
    is the oracle's.  More than 99% of elements must match exactly.  Beyond K = 32768
    the budget grows with K, because fp32 sums over K (the oracle's sequential one
    included) lose accuracy in proportion, and the exact-match floor is not applied
    (both sides are then fp32 approximations of the same float64 value)."""
    budget = HIN_BUDGET * max(1.0, n * D / 32768)
    g_in, g_post, g_res = got
    x_bits = np.asarray(x_bits, dtype=np.uint16).reshape(-1, n * D)
    r_in, r_post, r_res = mhc_pre_ref(x_bits, phi, alpha, bias, gamma, n, D, dtype, norm_eps, hc_eps)
    stats = {"label": label, "rows": int(x_bits.shape[0])}
    for name, g, r in (("hPost", g_post, r_post), ("hRes", g_res, r_res)):
        g = np.asarray(g).reshape(r.shape)
        assert np.all(np.isfinite(g)), f"{label} {name} not finite"
        err = np.abs(g.astype(np.float64) - r) / np.maximum(1.0, np.abs(r))
        stats[name + "_max_err"] = float(err.max())
        assert err.max() <= RTOL, f"{label} {name} max rel err {err.max():.3e}"
    g_in = np.asarray(g_in, dtype=np.uint16).reshape(r_in.shape)
    d = ulp_distance(g_in, r_in)
    stats["hIn_exact"] = float((d == 0).mean())
    stats["hIn_max_ulp"] = int(d.max())
    stats["hIn_over_1ulp"] = int((d > 1).sum())
    stats["hIn_closer_than_oracle"] = 0
    if (d > 1).any():
        bad_rows = np.nonzero((d > 1).any(axis=1))[0]
        xs = x_bits[bad_rows]
        _, _, _, pre64 = mhc_pre_numpy(xs, phi, alpha, bias, gamma, n, D, dtype, norm_eps, hc_eps)
        xf = to_float(xs, dtype).astype(np.float64).reshape(-1, n, D)
        mag = np.einsum("rs,rsd->rd", np.abs(pre64), np.abs(xf))
        gf = to_float(g_in[bad_rows], dtype).astype(np.float64)
        rf = to_float(r_in[bad_rows], dtype).astype(np.float64)
        ulp = ulp_size(r_in[bad_rows], dtype)
        ok = np.abs(gf - rf) <= ulp + budget * mag
        h64 = np.einsum("rs,rsd->rd", pre64, xf)
        closer = np.abs(gf - h64) <= np.abs(rf - h64) + ulp
        over = d[bad_rows] > 1
        stats["hIn_closer_than_oracle"] = int((over & ~ok & closer).sum())
        assert (ok | closer)[over].all(), f"{label} hIn differs beyond 1 ulp without cancellation"
    if n * D <= 32768:
        assert stats["hIn_exact"] > HIN_EXACT_MIN, f"{label} hIn exact-match rate {stats['hIn_exact']}"
    return stats


if __name__ == "__main__":  # pragma: no cover
    print(build(force=True), max_threads(), os.cpu_count())
