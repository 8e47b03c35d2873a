"""C-ABI checks that need no GPU: the library loads, exports every entry point
include/mhc_pre.h declares, and rejects the same descriptions the reference's
TilingFunc rejects (code/op_host/mhc_pre.cpp:57-79, :126-129) before touching
the device."""
import ctypes
import re
from pathlib import Path

import pytest

import mhcpre_review_b200 as mp

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "mhc_pre.h").read_text()
    return sorted(set(re.findall(r"MHC_API\s+[\w\s\*]+?\b(mhc(?:Pre|Post)\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    syms = declared_symbols()
    assert len(syms) >= 9
    L = mp.lib()
    for s in syms:
        assert hasattr(L, s), s
    assert set(syms) == set(mp.EXPORTED_SYMBOLS)
    assert L.mhcPreAbiVersion() == 1


def test_desc_struct_layout_matches_header():
    assert ctypes.sizeof(mp.MhcPreDesc) == 48
    assert ctypes.sizeof(mp.MhcPrePlan) == 32


@pytest.mark.parametrize("kw,status", [
    (dict(batch=0), -2), (dict(seq=-1), -2), (dict(head_dim=0), -2),
    (dict(streams=5), -3), (dict(streams=2), -3), (dict(streams=10), -3),
    (dict(head_dim=24), -4), (dict(head_dim=8), -4),
    (dict(dtype=7), -6),
])
def test_rejects_like_reference_tiling(kw, status):
    args = dict(batch=1, seq=64, streams=4, head_dim=256, dtype=mp.F16, has_gamma=False)
    args.update(kw)
    desc = mp.make_desc(args["batch"], args["seq"], args["streams"], args["head_dim"], args["dtype"],
                        args["has_gamma"])
    n = ctypes.c_size_t(0)
    assert mp.lib().mhcPreGetWorkspaceSize(ctypes.byref(desc), ctypes.byref(n)) == status
    with pytest.raises(mp.MhcPreError) as ei:
        mp.workspace_size(desc)
    assert ei.value.status == status


@pytest.mark.parametrize("kw,status", [
    (dict(batch=0), -2), (dict(streams=5), -3), (dict(head_dim=24), -4), (dict(dtype=7), -6),
])
def test_post_step_rejects_bad_descriptions_before_the_device(kw, status):
    args = dict(batch=1, seq=64, streams=4, head_dim=256, dtype=mp.F16)
    args.update(kw)
    desc = mp.make_desc(args["batch"], args["seq"], args["streams"], args["head_dim"], args["dtype"], False)
    assert mp.lib().mhcPostRun(ctypes.byref(desc), None, None, None, None, None, None) == status
    assert mp.lib().mhcPostRun(None, None, None, None, None, None, None) == -1


def test_null_pointers_rejected():
    L = mp.lib()
    assert L.mhcPreGetWorkspaceSize(None, None) == -1
    desc = mp.make_desc(1, 64, 4, 256, mp.F16, False)
    assert L.mhcPreGetWorkspaceSize(ctypes.byref(desc), None) == -1
    assert L.mhcPreQueryPlan(ctypes.byref(desc), None) == -1
    assert L.mhcPreGetDeviceStatus(None) == -1


def test_status_strings():
    L = mp.lib()
    for code in mp.STATUS_NAMES:
        s = L.mhcPreStatusString(code)
        assert isinstance(s, bytes) and len(s) > 3
    assert L.mhcPreStatusString(12345) == b"unknown status"


def test_valid_desc_without_gpu_reports_cuda_error_not_crash():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present: covered by the GPU tests")
    desc = mp.make_desc(1, 64, 4, 256, mp.F16, False)
    n = ctypes.c_size_t(0)
    rc = mp.lib().mhcPreGetWorkspaceSize(ctypes.byref(desc), ctypes.byref(n))
    assert rc in (-9, -10)


def test_algorithmic_bytes_match_baseline_table():
    from mhcpre_review_b200.configs import CONFIGS
    assert CONFIGS["c1"].algorithmic_bytes() == 267_372
    assert CONFIGS["c2"].algorithmic_bytes() == 106_209_388
    assert CONFIGS["c3"].algorithmic_bytes() == 1_223_164_236
    assert CONFIGS["c4"].algorithmic_bytes() == 4_705_730_668
    assert CONFIGS["c5_m1_g"].algorithmic_bytes() == 2_939_068
    assert CONFIGS["c5_m512_g"].algorithmic_bytes() == 39_608_428


def test_plan_options_are_validated_before_the_device():
    desc = mp.make_desc(1, 64, 4, 256, mp.F16, False)
    n = ctypes.c_size_t(0)
    bad = mp.make_plan_options(path=9)
    assert mp.lib().mhcPreGetWorkspaceSizeEx(ctypes.byref(desc), ctypes.byref(bad), ctypes.byref(n)) == -2
    bad = mp.make_plan_options()
    bad.reserved[3] = 1
    assert mp.lib().mhcPreGetWorkspaceSizeEx(ctypes.byref(desc), ctypes.byref(bad), ctypes.byref(n)) == -2
    bad = mp.make_plan_options(epi_blocks=8)  # 12 or 16 only
    assert mp.lib().mhcPreGetWorkspaceSizeEx(ctypes.byref(desc), ctypes.byref(bad), ctypes.byref(n)) == -2


def test_library_reads_no_environment():
    """The default plan depends only on the description and the device: no source of
    the library reads environment variables (tuning goes through plan options)."""
    csrc = ROOT / "mhcpre_review_b200" / "csrc"
    for f in list(csrc.glob("*.cu")) + list(csrc.glob("*.cuh")) + list(csrc.glob("*.cpp")) + list(csrc.glob("*.h")):
        assert "getenv" not in f.read_text(), f.name


def test_trace_build_exports_trace_read():
    """The trace build (-DMHC_TRACE) compiles and adds mhcPreTraceRead, declared in
    include/mhc_pre_trace.h; the default library does not export it."""
    from mhcpre_review_b200 import build

    path = build.build(trace=True)
    L = ctypes.CDLL(str(path))
    text = (ROOT / "include" / "mhc_pre_trace.h").read_text()
    for sym in re.findall(r"MHC_API\s+[\w\s\*]+?\b(mhcPre\w+)\s*\(", text):
        assert hasattr(L, sym), sym
    assert not hasattr(mp.lib(), "mhcPreTraceRead")
    for s in declared_symbols():
        assert hasattr(L, s), s


def test_debug_build_exports_its_entry_points():
    """The debug build (-DMHC_DEBUG) compiles and adds the entry points of
    include/mhc_pre_debug.h; the default library does not export them."""
    from mhcpre_review_b200 import build

    path = build.build(debug=True)
    L = ctypes.CDLL(str(path))
    text = (ROOT / "include" / "mhc_pre_debug.h").read_text()
    syms = re.findall(r"MHC_API\s+[\w\s\*]+?\b(mhcPre\w+)\s*\(", text)
    assert len(syms) == 2
    for sym in syms:
        assert hasattr(L, sym) and not hasattr(mp.lib(), sym), sym
