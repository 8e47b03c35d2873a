"""The Python binding rejects tensors the kernels would misread, before any pointer
crosses the C ABI: strided views, tensors on another device, wrong dtypes and
short buffers.  The checks run on CPU tensors here (the device rule compares
against whichever device the executor is pinned to); the GPU-side calls are
covered in test_parity_gpu.py."""
import pytest
import torch

import mhcpre_review_b200 as mp

CPU = torch.device("cpu")


def desc(n=4, D=64, B=1, S=8, bf16=True, gamma=True):
    return mp.make_desc(B, S, n, D, mp.BF16 if bf16 else mp.F16, gamma)


def good(n=4, D=64, B=1, S=8, bf16=True):
    mix = n * n + 2 * n
    dt = torch.bfloat16 if bf16 else torch.float16
    return dict(x=torch.zeros(B, S, n, D, dtype=dt), phi=torch.zeros(mix, n * D), gamma=torch.ones(n, D),
                alpha=torch.ones(3), bias=torch.zeros(mix))


def test_well_formed_arguments_pass():
    a = good()
    mp._check_weights(desc(), CPU, a["phi"], a["gamma"])
    mp._check_run(desc(), CPU, a["x"], a["alpha"], a["bias"])


def test_non_contiguous_x_is_rejected():
    a = good()
    xt = torch.zeros(1, 8, 64, 4, dtype=torch.bfloat16).transpose(2, 3)  # [1, 8, 4, 64], strided
    assert not xt.is_contiguous()
    with pytest.raises(mp.MhcPreError, match="contiguous"):
        mp._check_run(desc(), CPU, xt, a["alpha"], a["bias"])


@pytest.mark.parametrize("field,bad,msg", [
    ("phi", torch.zeros(24, 256, dtype=torch.bfloat16), "dtype"),
    ("phi", torch.zeros(24, 255), "elements"),
    ("gamma", torch.ones(4, 32), "elements"),
    ("gamma", torch.ones(4, 64, dtype=torch.float64), "dtype"),
])
def test_mistyped_or_short_weights_are_rejected(field, bad, msg):
    a = good()
    a[field] = bad
    with pytest.raises(mp.MhcPreError, match=msg):
        mp._check_weights(desc(), CPU, a["phi"], a["gamma"])


@pytest.mark.parametrize("field,bad,msg", [
    ("x", torch.zeros(1, 8, 4, 64, dtype=torch.float16), "dtype"),
    ("x", torch.zeros(1, 8, 4, 48, dtype=torch.bfloat16), "elements"),
    ("alpha", torch.ones(2), "elements"),
    ("bias", torch.zeros(23), "elements"),
    ("bias", torch.zeros(24, dtype=torch.float64), "dtype"),
])
def test_mistyped_or_short_run_arguments_are_rejected(field, bad, msg):
    a = good()
    a[field] = bad
    with pytest.raises(mp.MhcPreError, match=msg):
        mp._check_run(desc(), CPU, a["x"], a["alpha"], a["bias"])


def test_gamma_presence_must_match_description():
    a = good()
    with pytest.raises(mp.MhcPreError, match="gamma"):
        mp._check_weights(desc(gamma=False), CPU, a["phi"], a["gamma"])
    with pytest.raises(mp.MhcPreError, match="gamma"):
        mp._check_weights(desc(gamma=True), CPU, a["phi"], None)


def test_tensor_on_another_device_is_rejected():
    a = good()
    with pytest.raises(mp.MhcPreError, match="expected"):
        mp._check_run(desc(), torch.device("cuda", 1), a["x"], a["alpha"], a["bias"])


def test_cpu_x_has_no_cpu_path():
    a = good()
    with pytest.raises(mp.MhcPreError, match="CUDA tensor"):
        mp.mhc_pre(a["x"], a["phi"], a["alpha"], a["bias"], a["gamma"])


def test_wrong_outputs_are_rejected():
    a = good()
    out = (torch.empty(1, 8, 64, dtype=torch.bfloat16), torch.empty(1, 8, 4), torch.empty(1, 8, 4, 3))
    with pytest.raises(mp.MhcPreError, match="hRes"):
        mp._check_run(desc(), CPU, a["x"], a["alpha"], a["bias"], out)
