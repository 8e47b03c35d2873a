"""The CPU oracle of the mHC post step (test infrastructure; parity unpinned: the
reference has no code for the step after the layer).  Its known answers follow from
the formula xNext[s] = sum_t hRes[s,t] * x[t] + hPost[s] * y, and a float64
restatement bounds its rounding."""
import numpy as np
import pytest

from oracle import ref


def _inputs(M, n, D, dtype, seed):
    rng = np.random.default_rng(seed)
    x = ref.from_float(rng.standard_normal((M, n, D), dtype=np.float32), dtype)
    y = ref.from_float(rng.standard_normal((M, D), dtype=np.float32), dtype)
    hPost = (2.0 / (1.0 + np.exp(-rng.standard_normal((M, n))))).astype(np.float32)
    hRes = (0.5 * rng.standard_normal((M, n, n))).astype(np.float32)
    return x, y, hPost, hRes


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_identity_mix_and_no_layer_output_returns_x(dtype):
    x, y, _, _ = _inputs(5, 4, 48, dtype, 1)
    hRes = np.broadcast_to(np.eye(4, dtype=np.float32), (5, 4, 4)).copy()
    out = ref.mhc_post_ref(x, y, np.zeros((5, 4), np.float32), hRes, 4, 48, dtype)
    assert np.array_equal(out, x)


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_zero_mix_scatters_the_layer_output(dtype):
    x, y, _, _ = _inputs(3, 6, 32, dtype, 2)
    hPost = np.ones((3, 6), np.float32)
    out = ref.mhc_post_ref(x, y, hPost, np.zeros((3, 6, 6), np.float32), 6, 32, dtype)
    assert np.array_equal(out, np.repeat(y[:, None, :], 6, axis=1))


def test_hand_computed_element():
    # x streams 1, 2, 3, 4; y = 0.5; row s=1 of hRes = (0.25, 0.5, 0.75, 1); hPost[1] = 2
    n, D = 4, 16
    x = np.stack([ref.from_float(np.full((1, D), v, np.float32), "bf16") for v in (1, 2, 3, 4)], axis=1)
    y = ref.from_float(np.full((1, D), 0.5, np.float32), "bf16")
    hRes = np.zeros((1, n, n), np.float32)
    hRes[0, 1] = (0.25, 0.5, 0.75, 1.0)
    hPost = np.zeros((1, n), np.float32)
    hPost[0, 1] = 2.0
    out = ref.to_float(ref.mhc_post_ref(x, y, hPost, hRes, n, D, "bf16"), "bf16")
    assert np.all(out[0, 1] == 0.25 + 1.0 + 2.25 + 4.0 + 1.0)
    assert np.all(out[0, 0] == 0.0)


@pytest.mark.parametrize("n,D,dtype", [(4, 256, "bf16"), (6, 144, "fp16"), (8, 64, "bf16")])
def test_within_one_ulp_of_float64(n, D, dtype):
    x, y, hPost, hRes = _inputs(64, n, D, dtype, 3)
    out = ref.mhc_post_ref(x, y, hPost, hRes, n, D, dtype)
    exact = ref.mhc_post_numpy(x, y, hPost, hRes, n, D, dtype)
    ulp = ref.ulp_distance(out, ref.from_float(exact.astype(np.float32), dtype))
    # fp32 accumulation of n+1 terms, then one rounding to 16 bits: within one unit
    # except where the terms cancel to a small result
    big = np.abs(exact) > 1e-2
    assert (ulp[big] <= 1).all()
    assert (ulp == 0).mean() > 0.97


def test_rejects_bad_arguments():
    lib = ref._load()
    assert lib.mhc_post_oracle(1, 4, 16, 0, None, None, None, None, None, 0) == -1
