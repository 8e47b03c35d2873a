"""Pins the CPU oracle to the reference before anything is checked against it.

1. The reference's own known-answer tests for its rounding helpers
   (audit_group_vec.py:225-235) against the oracle's C helpers.
2. Golden fixtures captured from the reference's unmodified formula code
   (tests/golden/make_golden.py): the inputs are regenerated here by our own
   restatement of the audit's generator and must hash to the captured inputs, and
   the oracle in audit order must reproduce the captured outputs bit for bit.
3. The oracle in kernel order (the order the Ascend kernel uses) stays within the
   operator's tolerances of the same fixtures, and a float64 restatement agrees.
"""
import numpy as np
import pytest

from oracle import ref
from tests._audit_inputs import audit_inputs, digest, load_golden

CASES = load_golden()


@pytest.mark.parametrize("value,bits", [
    (1.0, 0x3C00), (0.5, 0x3800), (-2.0, 0xC000), (65504.0, 0x7BFF), (1e-30, 0x0000),
    (0.1, 0x2E66), (1.5, 0x3E00), (3.5, 0x4300), (2.5, 0x4100)])
def test_reference_fp16_known_answers(value, bits):
    assert ref.f32_to_f16_bits(value) == bits
    assert ref.from_float(np.array([value], np.float32), "fp16")[0] == bits


def test_reference_bf16_known_answer():
    b = ref.f32_to_bf16_bits(0.1)
    assert ref.bf16_bits_to_f32(b) == 0.10009765625
    assert ref.from_float(np.array([0.1], np.float32), "bf16")[0] == b


def test_fp16_subnormal_carry_quirk_of_reference_helper():
    """The reference's fp16 helper (audit_group_vec.py:181, runner.cpp:85) drops the
    carry when a subnormal rounds up to the smallest normal 2^-14; the device cast
    (CAST_RINT, and CUDA's __float2half_rn) rounds correctly.  The oracle keeps the
    quirk only in audit order."""
    import ctypes
    L = ref._load()
    rng = np.random.default_rng(1)
    vals = np.concatenate([rng.uniform(-1e-4, 1e-4, 50000), rng.uniform(-2, 2, 50000),
                           np.float32(2.0 ** -14) * (1 - rng.uniform(0, 1e-3, 2000))]).astype(np.float32)
    ieee = ref.from_float(vals, "fp16")
    quirk = ref.from_float(vals, "fp16", audit_carry=True)
    c_ieee = np.array([L.mhc_oracle_f32_to_f16(ctypes.c_float(v)) for v in vals], np.uint16)
    c_quirk = np.array([L.mhc_oracle_f32_to_f16_audit(ctypes.c_float(v)) for v in vals], np.uint16)
    assert np.array_equal(c_ieee, ieee)
    assert np.array_equal(c_quirk, quirk)
    assert np.array_equal(ieee, vals.astype(np.float16).view(np.uint16))
    differs = ieee != quirk
    assert differs.sum() > 0 and np.all((ieee[differs] & 0x7FFF) == 0x0400) and np.all((quirk[differs] & 0x7FFF) == 0)


def test_half_conversions_roundtrip_exhaustive():
    bits = np.arange(0, 1 << 16, dtype=np.uint32).astype(np.uint16)
    f16 = ref.to_float(bits, "fp16")
    finite = np.isfinite(f16)
    assert np.array_equal(ref.from_float(f16[finite], "fp16"), bits[finite])
    bf = ref.to_float(bits, "bf16")
    finite = np.isfinite(bf)
    assert np.array_equal(ref.from_float(bf[finite], "bf16"), bits[finite])
    # C helpers agree with the vectorised ones on a sample, including subnormals
    for b in (0x0001, 0x03FF, 0x0400, 0x3C01, 0x7BFF, 0x8001, 0xFBFF):
        assert ref.f16_bits_to_f32(b) == float(f16[b])


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]['source']}{c[0]['idx']}_n{c[0]['n']}d{c[0]['d']}{c[0]['dtype']}g{int(c[0]['gamma'])}")
def test_oracle_reproduces_reference_outputs(case):
    m, gold = case
    n, d, dtype = m["n"], m["d"], m["dtype"]
    x, phi, gamma, alpha, bias = audit_inputs(n, d, m["gamma"], dtype, m["rows"], m["seed"])
    dig = m["digests"]
    assert digest(x) == dig["x"] and digest(phi) == dig["phi"]
    assert digest(alpha) == dig["alpha"] and digest(bias) == dig["bias"]
    assert (gamma is None) == (dig["gamma"] is None)
    if gamma is not None:
        assert digest(gamma) == dig["gamma"]

    hin, hpost, hres = ref.mhc_pre_ref(x, phi, alpha, bias, gamma, n, d, dtype, order=ref.ORDER_AUDIT)
    assert np.array_equal(hin, gold["hIn"])
    assert np.array_equal(hpost.view(np.uint32), gold["hPost"].view(np.uint32))
    assert np.array_equal(hres.view(np.uint32), gold["hRes"].view(np.uint32))

    # kernel order: same math, Ascend kernel rounding order
    hin_k, hpost_k, hres_k = ref.mhc_pre_ref(x, phi, alpha, bias, gamma, n, d, dtype,
                                             order=ref.ORDER_KERNEL)
    for got, want in ((hpost_k, gold["hPost"]), (hres_k, gold["hRes"])):
        err = np.abs(got.astype(np.float64) - want) / np.maximum(1.0, np.abs(want))
        assert err.max() <= 1e-5  # rounding-order difference only; operator tolerance is 1e-4
    assert ref.ulp_distance(hin_k, gold["hIn"]).max() <= 1

    # float64 restatement (runner.cpp-style double square-sum)
    h_in64, h_post64, h_res64, h_pre64 = ref.mhc_pre_numpy(x, phi, alpha, bias, gamma, n, d, dtype)
    assert np.max(np.abs(h_post64 - gold["hPost"]) / np.maximum(1, np.abs(gold["hPost"]))) <= 1e-5
    assert np.max(np.abs(h_res64 - gold["hRes"]) / np.maximum(1, np.abs(gold["hRes"]))) <= 1e-5
    assert np.max(np.abs(h_pre64 - gold["hPre"])) <= 1e-5


def test_oracle_semantic_red_lines():
    """The two semantic rules the reference audit enforces (audit_group_vec.py:499-511):
    the square-sum uses the raw x (before gamma), and hRes is linear (no sigmoid)."""
    n, d = 4, 16
    rng = np.random.default_rng(0)
    x = ref.from_float(rng.standard_normal((3, n * d)).astype(np.float32), "bf16")
    phi = (rng.standard_normal((24, n * d)) * 0.05).astype(np.float32)
    alpha = np.array([0.7, 1.1, 1.3], np.float32)
    bias = (rng.standard_normal(24) * 0.1).astype(np.float32)
    gamma = np.full(n * d, 2.0, np.float32)
    _, _, res_g = ref.mhc_pre_ref(x, phi, alpha, bias, gamma, n, d, "bf16")
    _, _, res_1 = ref.mhc_pre_ref(x, phi, alpha, bias, None, n, d, "bf16")
    # gamma=2 doubles mix but not invRms, so (hRes - bias) doubles exactly
    assert np.allclose((res_g - bias[8:].reshape(n, n)), 2 * (res_1 - bias[8:].reshape(n, n)), rtol=1e-6)
    # linear in alpha[2]
    a2 = alpha.copy(); a2[2] *= 2
    _, _, res_a = ref.mhc_pre_ref(x, phi, a2, bias, None, n, d, "bf16")
    assert np.allclose(res_a - bias[8:].reshape(n, n), 2 * (res_1 - bias[8:].reshape(n, n)), rtol=1e-6)
