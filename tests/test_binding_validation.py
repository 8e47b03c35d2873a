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


def _cpu_executor(d):
    """An executor object pinned to the CPU device, without a workspace: enough for
    the argument checks, which all run before any call into the library."""
    ex = object.__new__(mp.MhcPre)
    ex.desc = d
    ex.device = CPU
    return ex


def _post_pre_args():
    a = good()
    return dict(x=a["x"], y=torch.zeros(1, 8, 64, dtype=torch.bfloat16), hPost=torch.zeros(1, 8, 4),
                hRes=torch.zeros(1, 8, 4, 4), alpha=a["alpha"], bias=a["bias"])


@pytest.mark.parametrize("field,bad,msg", [
    ("y", torch.zeros(1, 8, 64, dtype=torch.float16), "dtype"),
    ("y", torch.zeros(1, 8, 48, dtype=torch.bfloat16), "elements"),
    ("y", torch.zeros(1, 64, 8, dtype=torch.bfloat16).transpose(1, 2), "contiguous"),
    ("hPost", torch.zeros(1, 8, 4, dtype=torch.float64), "dtype"),
    ("hRes", torch.zeros(1, 8, 4, 3), "elements"),
    ("x", torch.zeros(1, 8, 4, 32, dtype=torch.bfloat16), "elements"),
    ("alpha", torch.ones(2), "elements"),
])
def test_post_and_run_rejects_bad_arguments(field, bad, msg):
    """MhcPre.post_and_run (mhcPostPreRun) checks the ending layer's y, hPost and
    hRes as well as the next layer's run arguments."""
    args = _post_pre_args()
    args[field] = bad
    with pytest.raises(mp.MhcPreError, match=msg):
        _cpu_executor(desc()).post_and_run(**args)


def test_post_and_run_rejects_a_wrong_x_next():
    args = _post_pre_args()
    with pytest.raises(mp.MhcPreError, match="elements"):
        _cpu_executor(desc()).post_and_run(**args, x_next=torch.zeros(1, 8, 4, 32, dtype=torch.bfloat16))


def test_fast_argument_check_agrees_with_the_full_one():
    """The executor's hot-call check (_args_ok) accepts exactly what the full checks
    accept; anything else goes through the full checks, which raise."""
    a = good()
    d = desc()
    specs = ((torch.bfloat16, 1 * 8 * 4 * 64), (torch.float32, 3), (torch.float32, 24))
    cpu = -1  # get_device() of a CPU tensor
    assert mp._args_ok((a["x"], a["alpha"], a["bias"]), specs, cpu)
    mp._check_run(d, CPU, a["x"], a["alpha"], a["bias"])
    strided = torch.zeros(1, 8, 64, 4, dtype=torch.bfloat16).transpose(2, 3)
    for bad in ((a["x"].half(), a["alpha"], a["bias"]), (a["x"], a["alpha"][:2], a["bias"]),
                (strided, a["alpha"], a["bias"]), (a["x"], [1.0, 1.0, 1.0], a["bias"])):
        assert not mp._args_ok(bad, specs, cpu)
        with pytest.raises(mp.MhcPreError):
            mp._check_run(d, CPU, *bad)
    assert not mp._args_ok((a["x"], a["alpha"], a["bias"]), specs, 0)  # another device
