"""B200-native MhcPre operator: Python front end over the C ABI (include/mhc_pre.h).

This mirrors the reference's operator interface (the aclnn pair generated from the
OpDef in code/op_host/mhc_pre.cpp:261-304 and used at cloud_runner/runner.cpp:440-472):

    executor = MhcPre(batch, seq, streams, head_dim, dtype, has_gamma, norm_eps, hc_eps)
    executor.prepare(phi, gamma)                  # once per weight set
    hIn, hPost, hRes = executor(x, alpha, bias)   # relaunchable, like aclnnMhcPre

    hIn, hPost, hRes = mhc_pre(x, phi, alpha, bias, gamma, norm_eps, hc_eps)  # one shot

Inputs/outputs are torch CUDA tensors (torch is used only for device memory and
streams); every computation runs in libmhcpre_b200.so.  There is no CPU fallback:
if the library is missing or no sm_100 GPU is present, calls raise.
Errors mirror the reference's rejects and raise ``MhcPreError`` with the status code.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libmhcpre_b200.so"
# the same library built with -DMHC_TRACE: stage stamps, mhcPreTraceRead
TRACE_LIB_PATH = _PKG / "libmhcpre_b200_trace.so"
# ... and with -DMHC_DEBUG: bounds checks in the kernels (include/mhc_pre_debug.h)
DEBUG_LIB_PATH = _PKG / "libmhcpre_b200_debug.so"

F16 = 0
BF16 = 1

STATUS_NAMES = {
    0: "SUCCESS", -1: "NULL_POINTER", -2: "BAD_SHAPE", -3: "BAD_STREAM_COUNT", -4: "BAD_HEAD_DIM",
    -5: "MIX_TOO_LARGE", -6: "BAD_DTYPE", -7: "MISALIGNED", -8: "WORKSPACE_TOO_SMALL", -9: "CUDA_ERROR",
    -10: "UNSUPPORTED_DEVICE", -11: "DEVICE_TIMEOUT", -12: "NOT_PREPARED", -13: "TOO_LARGE",
    -14: "INTERNAL_CHECK",
}

EXPORTED_SYMBOLS = (
    "mhcPreGetWorkspaceSize", "mhcPrePrepareWeights", "mhcPreRun", "mhcPreRunPrepared",
    "mhcPreRunPreparedProfiled", "mhcPreQueryPlan", "mhcPreGetDeviceStatus", "mhcPreStatusString",
    "mhcPreAbiVersion", "mhcPreRunNoAlloc", "mhcPreDiagWaitTimeout", "mhcPostRun",
    "mhcPreGetWorkspaceSizeEx", "mhcPreQueryPlanEx", "mhcPrePrepareWeightsEx", "mhcPreRunPreparedEx",
    "mhcPostPreRun",
)

PATH_AUTO = -1


class MhcPreError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        name = STATUS_NAMES.get(status, str(status))
        detail = ""
        try:
            detail = lib().mhcPreStatusString(status).decode()
        except Exception:  # pragma: no cover
            pass
        super().__init__(f"MhcPre {what}: {name} ({status}) {detail}".strip())


class MhcPreDesc(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int64), ("seq", ctypes.c_int64), ("streams", ctypes.c_int64),
                ("headDim", ctypes.c_int64), ("dtype", ctypes.c_int32), ("hasGamma", ctypes.c_int32),
                ("normEps", ctypes.c_float), ("hcEps", ctypes.c_float)]


class MhcPrePlan(ctypes.Structure):
    _fields_ = [("path", ctypes.c_int32), ("kernelsPerRun", ctypes.c_int32), ("gridCtas", ctypes.c_int32),
                ("splits", ctypes.c_int32), ("rowsPerTile", ctypes.c_int32), ("reserved", ctypes.c_int32 * 3)]


class MhcPrePlanOptions(ctypes.Structure):
    """mhcPrePlanOptions_t: an explicit override of the launch plan (tests, benchmarks,
    profiling).  0 keeps the library's choice, except path (PATH_AUTO)."""
    _fields_ = [("path", ctypes.c_int32), ("splits", ctypes.c_int32), ("gemmCtasPerSm", ctypes.c_int32),
                ("gemmStages", ctypes.c_int32), ("tmaBatch", ctypes.c_int32), ("teamSize", ctypes.c_int32),
                ("clusterLead", ctypes.c_int32), ("l2Hint", ctypes.c_int32), ("ringTiles", ctypes.c_int32),
                ("pairedGemm", ctypes.c_int32), ("epiBlocks", ctypes.c_int32), ("reserved", ctypes.c_int32 * 5)]


def make_plan_options(path=PATH_AUTO, splits=0, gemm_ctas_per_sm=0, gemm_stages=0, tma_batch=0, team_size=0,
                      cluster_lead=0, l2_hint=0, ring_tiles=0, paired_gemm=0, epi_blocks=0) -> MhcPrePlanOptions:
    return MhcPrePlanOptions(int(path), int(splits), int(gemm_ctas_per_sm), int(gemm_stages), int(tma_batch),
                             int(team_size), int(cluster_lead), int(l2_hint), int(ring_tiles), int(paired_gemm),
                             int(epi_blocks))


# Plan options every call of this module passes to the library (None: the default
# plan, which depends only on the description and the device).  Tests and the bench
# set it, e.g. ``mp._OPTIONS = mp.make_plan_options(path=0)``, or use plan_options().
_OPTIONS = None


class plan_options:
    """Context manager: ``with plan_options(path=3): ...`` runs the enclosed calls
    under the given plan options."""

    def __init__(self, **kw):
        self.opts = make_plan_options(**kw)

    def __enter__(self):
        global _OPTIONS
        self.prev = _OPTIONS
        _OPTIONS = self.opts
        return self.opts

    def __exit__(self, *exc):
        global _OPTIONS
        _OPTIONS = self.prev
        return False


def _opt():
    return None if _OPTIONS is None else ctypes.byref(_OPTIONS)


_libs = {}
_lib_path = LIB_PATH


def lib():
    """Loads libmhcpre_b200.so, or the library selected with use_library (raises if
    it has not been built)."""
    L = _libs.get(_lib_path)
    if L is None:
        if not _lib_path.exists():
            raise RuntimeError(f"{_lib_path} is missing: run `python -m mhcpre_review_b200.build` "
                               "(the operator has no CPU fallback)")
        L = ctypes.CDLL(str(_lib_path))
        vp, sz = ctypes.c_void_p, ctypes.c_size_t
        dp = ctypes.POINTER(MhcPreDesc)
        L.mhcPreGetWorkspaceSize.argtypes = [dp, ctypes.POINTER(sz)]
        L.mhcPrePrepareWeights.argtypes = [dp, vp, vp, vp, sz, vp]
        L.mhcPreRun.argtypes = [dp, vp, vp, vp, vp, vp, vp, vp, vp, vp, sz, vp]
        L.mhcPreRunPrepared.argtypes = [dp, vp, vp, vp, vp, vp, vp, vp, sz, vp]
        L.mhcPreRunPreparedProfiled.argtypes = [dp, vp, vp, vp, vp, vp, vp, vp, sz, vp, vp, vp]
        L.mhcPreQueryPlan.argtypes = [dp, ctypes.POINTER(MhcPrePlan)]
        L.mhcPreRunNoAlloc.argtypes = [dp, vp, vp, vp, vp, vp, vp, vp, vp, vp]
        L.mhcPostRun.argtypes = [dp, vp, vp, vp, vp, vp, vp]
        L.mhcPostPreRun.argtypes = [dp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, sz, vp]
        L.mhcPreGetDeviceStatus.argtypes = [ctypes.POINTER(ctypes.c_int32)]
        op = ctypes.POINTER(MhcPrePlanOptions)
        L.mhcPreGetWorkspaceSizeEx.argtypes = [dp, op, ctypes.POINTER(sz)]
        L.mhcPreQueryPlanEx.argtypes = [dp, op, ctypes.POINTER(MhcPrePlan)]
        L.mhcPrePrepareWeightsEx.argtypes = [dp, op, vp, vp, vp, sz, vp]
        L.mhcPreRunPreparedEx.argtypes = [dp, op, vp, vp, vp, vp, vp, vp, vp, sz, vp, vp, vp]
        L.mhcPreStatusString.argtypes = [ctypes.c_int]
        L.mhcPreStatusString.restype = ctypes.c_char_p
        L.mhcPreAbiVersion.argtypes = []
        for name in EXPORTED_SYMBOLS:
            if name != "mhcPreStatusString":
                getattr(L, name).restype = ctypes.c_int
        if hasattr(L, "mhcPreTraceRead"):
            L.mhcPreTraceRead.argtypes = [vp, sz, ctypes.POINTER(sz)]
            L.mhcPreTraceRead.restype = ctypes.c_int
        if hasattr(L, "mhcPreDebugSetRecordCap"):
            L.mhcPreDebugSetRecordCap.argtypes = [ctypes.c_int64]
            L.mhcPreDebugSetRecordCap.restype = ctypes.c_int
            L.mhcPreDebugLastCheckLine.argtypes = [ctypes.POINTER(ctypes.c_int32)]
            L.mhcPreDebugLastCheckLine.restype = ctypes.c_int
        _libs[_lib_path] = L
    return L


class use_library:
    """``with use_library(TRACE_LIB_PATH): ...`` sends the enclosed calls of this
    module to another build of the library (each keeps its own device state)."""

    def __init__(self, path):
        self.path = Path(path)

    def __enter__(self):
        global _lib_path
        self.prev = _lib_path
        _lib_path = self.path
        return lib()

    def __exit__(self, *exc):
        global _lib_path
        _lib_path = self.prev
        return False


TRACE_DTYPE = [("t_ns", "<u8"), ("cta", "<u4"), ("warp", "<u2"), ("event", "<u2"), ("a", "<u4"), ("b", "<u4")]


def trace_read(max_records: int = 4 << 20):
    """Reads and clears the stage stamps of the trace build (use inside
    use_library(TRACE_LIB_PATH)); returns (numpy records, how many were recorded)."""
    import numpy as np
    L = lib()
    if not hasattr(L, "mhcPreTraceRead"):
        raise RuntimeError("the loaded library is not the trace build")
    buf = np.zeros(max_records, dtype=TRACE_DTYPE)
    n = ctypes.c_size_t(0)
    _check(L.mhcPreTraceRead(ctypes.c_void_p(buf.ctypes.data), max_records, ctypes.byref(n)), "TraceRead")
    return buf[:min(int(n.value), max_records)], int(n.value)


def _check(rc: int, what: str):
    if rc != 0:
        raise MhcPreError(rc, what)


def make_desc(batch, seq, streams, head_dim, dtype, has_gamma, norm_eps=1e-6, hc_eps=1e-6) -> MhcPreDesc:
    return MhcPreDesc(int(batch), int(seq), int(streams), int(head_dim), int(dtype), int(bool(has_gamma)),
                      float(norm_eps), float(hc_eps))


def workspace_size(desc: MhcPreDesc) -> int:
    n = ctypes.c_size_t(0)
    _check(lib().mhcPreGetWorkspaceSizeEx(ctypes.byref(desc), _opt(), ctypes.byref(n)), "GetWorkspaceSize")
    return int(n.value)


def query_plan(desc: MhcPreDesc) -> dict:
    p = MhcPrePlan()
    _check(lib().mhcPreQueryPlanEx(ctypes.byref(desc), _opt(), ctypes.byref(p)), "QueryPlan")
    return {"path": p.path, "kernels_per_run": p.kernelsPerRun, "grid_ctas": p.gridCtas, "splits": p.splits,
            "rows_per_tile": p.rowsPerTile}


def device_status() -> int:
    """Reads and clears the device error word (synchronizes the device)."""
    s = ctypes.c_int32(0)
    _check(lib().mhcPreGetDeviceStatus(ctypes.byref(s)), "GetDeviceStatus")
    return int(s.value)


def diag_wait_timeout(limit_us: int = 2000, stream=None) -> tuple[bool, bool]:
    """Makes a counter wait and an mbarrier wait run out on the device (nothing ever
    signals them) with the given limit; returns (counter gave up, barrier gave up).
    The device status word is left at MHC_STATUS_DEVICE_TIMEOUT."""
    c, b = ctypes.c_int32(0), ctypes.c_int32(0)
    _check(lib().mhcPreDiagWaitTimeout(ctypes.c_uint32(limit_us), ctypes.byref(c), ctypes.byref(b),
                                       _stream_ptr(stream)), "DiagWaitTimeout")
    return bool(c.value), bool(b.value)


def _torch():
    import torch
    return torch


def _dtype_code(t) -> int:
    torch = _torch()
    if t == torch.bfloat16:
        return BF16
    if t == torch.float16:
        return F16
    raise MhcPreError(-6, f"x dtype {t}")


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _require(t, name, device, dtype=None, shape=None):
    """Checks one tensor argument before its pointer crosses the C ABI: the kernels
    read every tensor as dense row-major memory on the device they launch on, so a
    strided view, a tensor on another GPU, a wrong dtype or a short buffer would be
    read as something else (or past its end)."""
    torch = _torch()
    if not isinstance(t, torch.Tensor):
        raise MhcPreError(-1, f"{name} must be a torch tensor")
    if t.device != device:
        raise MhcPreError(-2, f"{name} is on {t.device}, expected {device}")
    if not t.is_contiguous():
        raise MhcPreError(-2, f"{name} must be contiguous")
    if dtype is not None and t.dtype != dtype:
        raise MhcPreError(-6, f"{name} dtype {t.dtype}, expected {dtype}")
    if shape is not None and t.numel() != _numel(shape):
        raise MhcPreError(-2, f"{name} has {t.numel()} elements, expected {_numel(shape)} ({list(shape)})")


def _numel(shape) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n


def _check_weights(desc, device, phi, gamma):
    torch = _torch()
    K = desc.streams * desc.headDim
    mix = desc.streams * desc.streams + 2 * desc.streams
    _require(phi, "phi", device, torch.float32, (mix, K))
    if bool(desc.hasGamma) != (gamma is not None):
        raise MhcPreError(-1, "gamma must be given exactly when has_gamma is set")
    if gamma is not None:
        _require(gamma, "gamma", device, torch.float32, (desc.streams, desc.headDim))


def _check_run(desc, device, x, alpha, bias, out=None):
    torch = _torch()
    mix = desc.streams * desc.streams + 2 * desc.streams
    x_dtype = torch.bfloat16 if desc.dtype == BF16 else torch.float16
    _require(x, "x", device, x_dtype, (desc.batch, desc.seq, desc.streams, desc.headDim))
    _require(alpha, "alpha", device, torch.float32, (3,))
    _require(bias, "bias", device, torch.float32, (mix,))
    if out is not None:
        hIn, hPost, hRes = out
        _require(hIn, "hIn", device, x_dtype, (desc.batch, desc.seq, desc.headDim))
        _require(hPost, "hPost", device, torch.float32, (desc.batch, desc.seq, desc.streams))
        _require(hRes, "hRes", device, torch.float32, (desc.batch, desc.seq, desc.streams, desc.streams))


def _args_ok(tensors, specs, device_index) -> bool:
    """Fast form of the argument checks for a hot call: every tensor has its expected
    dtype and element count, is dense and sits on the executor's device.  False sends
    the call through the full checks, which raise with the reason."""
    try:
        for t, (dtype, numel) in zip(tensors, specs):
            if t.dtype != dtype or t.numel() != numel or t.get_device() != device_index or not t.is_contiguous():
                return False
        return True
    except AttributeError:  # not a tensor
        return False


def _stream_ptr(stream):
    """The cudaStream_t to launch on: the given torch stream, else torch's current
    stream on the current device (read as a raw handle, without building a Stream
    object, which costs more host time than the launch itself)."""
    if stream is not None:
        return ctypes.c_void_p(stream.cuda_stream)
    C = _torch()._C
    return ctypes.c_void_p(C._cuda_getCurrentRawStream(C._cuda_getDevice()))


class _on_device:
    """``with _on_device(dev): ...`` makes the CUDA device dev current for the enclosed
    calls (the library plans and launches on the current device) and restores the
    previous one afterwards; it switches nothing when dev is already current."""

    __slots__ = ("idx", "prev")

    def __init__(self, device):
        self.idx = device.index

    def __enter__(self):
        C = _torch()._C
        self.prev = C._cuda_getDevice()
        if self.prev != self.idx:
            C._cuda_setDevice(self.idx)
        return self

    def __exit__(self, *exc):
        if self.prev != self.idx:
            _torch()._C._cuda_setDevice(self.prev)
        return False


class MhcPre:
    """Reusable executor: owns the workspace and the prepared weights."""

    def __init__(self, batch, seq, streams, head_dim, dtype, has_gamma, norm_eps=1e-6, hc_eps=1e-6,
                 device=None, workspace=None):
        torch = _torch()
        self.desc = make_desc(batch, seq, streams, head_dim,
                              dtype if isinstance(dtype, int) else _dtype_code(dtype), has_gamma, norm_eps, hc_eps)
        dev = torch.device("cuda") if device is None else torch.device(device)
        if dev.type != "cuda":
            raise MhcPreError(-2, f"device {dev} is not a CUDA device; there is no CPU path")
        # the plan and the launches use the current device: pin the executor to one
        self.device = torch.device("cuda", torch.cuda.current_device() if dev.index is None else dev.index)
        with torch.cuda.device(self.device):
            self.ws_bytes = workspace_size(self.desc)
        if workspace is None:
            workspace = torch.empty(self.ws_bytes, dtype=torch.uint8, device=self.device)
        else:
            _require(workspace, "workspace", self.device)
            if workspace.numel() * workspace.element_size() < self.ws_bytes:
                raise MhcPreError(-8, "workspace")
        self.workspace = workspace
        self.prepared = False
        # expected (dtype, elements) of x, alpha, bias, hIn, hPost, hRes for _args_ok
        d = self.desc
        x_dtype = torch.bfloat16 if d.dtype == BF16 else torch.float16
        mix = d.streams * d.streams + 2 * d.streams
        self._run_specs = ((x_dtype, d.batch * d.seq * d.streams * d.headDim), (torch.float32, 3),
                           (torch.float32, mix), (x_dtype, d.batch * d.seq * d.headDim),
                           (torch.float32, d.batch * d.seq * d.streams),
                           (torch.float32, d.batch * d.seq * d.streams * d.streams))

    @property
    def plan(self) -> dict:
        return query_plan(self.desc)

    def prepare(self, phi, gamma=None, stream=None):
        _check_weights(self.desc, self.device, phi, gamma)
        with _on_device(self.device):
            _check(lib().mhcPrePrepareWeightsEx(ctypes.byref(self.desc), _opt(), _ptr(phi), _ptr(gamma),
                                                _ptr(self.workspace), self.ws_bytes, _stream_ptr(stream)),
                   "PrepareWeights")
        self.prepared = True

    def outputs(self, x_dtype):
        torch = _torch()
        d = self.desc
        hIn = torch.empty((d.batch, d.seq, d.headDim), dtype=x_dtype, device=self.device)
        hPost = torch.empty((d.batch, d.seq, d.streams), dtype=torch.float32, device=self.device)
        hRes = torch.empty((d.batch, d.seq, d.streams, d.streams), dtype=torch.float32, device=self.device)
        return hIn, hPost, hRes

    def run_profiled(self, x, alpha, bias, out, ev_begin, ev_end, stream=None):
        """Like __call__, recording torch.cuda.Event ev_begin/ev_end around the main kernel."""
        _check_run(self.desc, self.device, x, alpha, bias, out)
        hIn, hPost, hRes = out
        with _on_device(self.device):
            _check(lib().mhcPreRunPreparedEx(ctypes.byref(self.desc), _opt(), _ptr(x), _ptr(alpha), _ptr(bias),
                                             _ptr(hIn), _ptr(hPost), _ptr(hRes), _ptr(self.workspace),
                                             self.ws_bytes, _stream_ptr(stream),
                                             ctypes.c_void_p(ev_begin.cuda_event),
                                             ctypes.c_void_p(ev_end.cuda_event)), "RunPreparedProfiled")
        return hIn, hPost, hRes

    def post_and_run(self, x, y, hPost, hRes, alpha, bias, x_next=None, out=None, stream=None):
        """The previous layer's post step fused with this executor's MhcPre
        (mhcPostPreRun): x_next = sum_t hRes[..., s, t] * x[..., t, :] + hPost[..., s] * y,
        then MhcPre on x_next with the prepared weights.  x: [B, S, n, D] (the streams
        the previous layer read), y: [B, S, D] its output, hPost/hRes its fp32
        coefficients.  Returns (x_next, (hIn, hPost, hRes)); x_next may be x."""
        torch = _torch()
        d = self.desc
        x_dtype = torch.bfloat16 if d.dtype == BF16 else torch.float16
        _require(x, "x", self.device, x_dtype, (d.batch, d.seq, d.streams, d.headDim))
        _require(y, "y", self.device, x_dtype, (d.batch, d.seq, d.headDim))
        _require(hPost, "hPost", self.device, torch.float32, (d.batch, d.seq, d.streams))
        _require(hRes, "hRes", self.device, torch.float32, (d.batch, d.seq, d.streams, d.streams))
        if x_next is None:
            x_next = torch.empty_like(x)
        _check_run(d, self.device, x_next, alpha, bias, out)
        hIn, hPostN, hResN = out if out is not None else self.outputs(x_dtype)
        with _on_device(self.device):
            _check(lib().mhcPostPreRun(ctypes.byref(d), _ptr(x), _ptr(y), _ptr(hPost), _ptr(hRes), _ptr(x_next),
                                       _ptr(alpha), _ptr(bias), _ptr(hIn), _ptr(hPostN), _ptr(hResN),
                                       _ptr(self.workspace), self.ws_bytes, _stream_ptr(stream)), "PostPreRun")
        return x_next, (hIn, hPostN, hResN)

    def __call__(self, x, alpha, bias, out=None, stream=None):
        args = (x, alpha, bias) if out is None else (x, alpha, bias, *out)
        if not _args_ok(args, self._run_specs, self.device.index):
            _check_run(self.desc, self.device, x, alpha, bias, out)
        hIn, hPost, hRes = out if out is not None else self.outputs(x.dtype)
        with _on_device(self.device):
            if _OPTIONS is None:
                rc = lib().mhcPreRunPrepared(ctypes.byref(self.desc), _ptr(x), _ptr(alpha), _ptr(bias), _ptr(hIn),
                                             _ptr(hPost), _ptr(hRes), _ptr(self.workspace), self.ws_bytes,
                                             _stream_ptr(stream))
            else:
                rc = lib().mhcPreRunPreparedEx(ctypes.byref(self.desc), _opt(), _ptr(x), _ptr(alpha), _ptr(bias),
                                               _ptr(hIn), _ptr(hPost), _ptr(hRes), _ptr(self.workspace),
                                               self.ws_bytes, _stream_ptr(stream), None, None)
            _check(rc, "RunPrepared")
        return hIn, hPost, hRes


def mhc_pre(x, phi, alpha, bias, gamma=None, norm_eps=1e-6, hc_eps=1e-6, out=None, workspace=None, stream=None):
    """One-shot MhcPre (prepare + run).  x: [B, S, n, D] fp16/bf16 CUDA tensor;
    phi: fp32 [mix, n*D] (the reference's K-contiguous layout); alpha: fp32 [3];
    bias: fp32 [mix]; gamma: fp32 [n, D] or None.  Returns (hIn [B,S,D], hPost [B,S,n],
    hRes [B,S,n,n])."""
    torch = _torch()
    if not isinstance(x, torch.Tensor) or x.dim() != 4:
        raise MhcPreError(-2, "x must be a 4-D tensor [B, S, n, D]")
    if x.device.type != "cuda":
        raise MhcPreError(-2, f"x must be a CUDA tensor (got {x.device}); there is no CPU path")
    B, S, n, D = x.shape
    with _on_device(x.device):
        ex = MhcPre(B, S, n, D, x.dtype, gamma is not None, norm_eps, hc_eps, device=x.device, workspace=workspace)
        _check_weights(ex.desc, ex.device, phi, gamma)
        _check_run(ex.desc, ex.device, x, alpha, bias, out)
        hIn, hPost, hRes = out if out is not None else ex.outputs(x.dtype)
        if _OPTIONS is None:
            _check(lib().mhcPreRun(ctypes.byref(ex.desc), _ptr(x), _ptr(phi), _ptr(alpha), _ptr(bias), _ptr(gamma),
                                   _ptr(hIn), _ptr(hPost), _ptr(hRes), _ptr(ex.workspace), ex.ws_bytes,
                                   _stream_ptr(stream)), "Run")
        else:
            ex.prepare(phi, gamma, stream)
            ex(x, alpha, bias, out=(hIn, hPost, hRes), stream=stream)
    return hIn, hPost, hRes


def mhc_post_pre(x, y, hPost, hRes, phi, alpha, bias, gamma=None, norm_eps=1e-6, hc_eps=1e-6, x_next=None,
                 out=None, workspace=None, stream=None):
    """One-shot layer boundary: the ending layer's post step (x, y, hPost, hRes) fused
    with the next layer's MhcPre (phi, alpha, bias, gamma), i.e. the weights are
    prepared, then mhcPostPreRun.  Returns (x_next, (hIn, hPost, hRes)) of the next
    layer; x_next may be x."""
    torch = _torch()
    if not isinstance(x, torch.Tensor) or x.dim() != 4:
        raise MhcPreError(-2, "x must be a 4-D tensor [B, S, n, D]")
    if x.device.type != "cuda":
        raise MhcPreError(-2, f"x must be a CUDA tensor (got {x.device}); there is no CPU path")
    B, S, n, D = x.shape
    with _on_device(x.device):
        ex = MhcPre(B, S, n, D, x.dtype, gamma is not None, norm_eps, hc_eps, device=x.device, workspace=workspace)
        ex.prepare(phi, gamma, stream)
        return ex.post_and_run(x, y, hPost, hRes, alpha, bias, x_next=x_next, out=out, stream=stream)


def mhc_post(x, y, hPost, hRes, out=None, stream=None):
    """The mHC post step after the layer: xNext[..., s, :] = sum_t hRes[..., s, t] *
    x[..., t, :] + hPost[..., s] * y[..., :].  x: [B, S, n, D] fp16/bf16 CUDA tensor
    (the streams MhcPre read); y: [B, S, D] in x's dtype (the layer output); hPost
    [B, S, n] and hRes [B, S, n, n] fp32 from MhcPre.  Returns xNext [B, S, n, D]
    (out may be x itself: the step runs in place)."""
    if x.dim() != 4:
        raise MhcPreError(-2, "x must be 4-D [B, S, n, D]")
    B, S, n, D = x.shape
    torch = _torch()
    if y.dtype != x.dtype:
        raise MhcPreError(-6, f"y dtype {y.dtype} differs from x dtype {x.dtype}")
    if tuple(y.shape) != (B, S, D) or tuple(hPost.shape) != (B, S, n) or tuple(hRes.shape) != (B, S, n, n):
        raise MhcPreError(-2, "y, hPost, hRes shapes must be [B,S,D], [B,S,n], [B,S,n,n]")
    if hPost.dtype != torch.float32 or hRes.dtype != torch.float32:
        raise MhcPreError(-6, "hPost and hRes must be fp32")
    if x.device.type != "cuda":
        raise MhcPreError(-2, f"x must be a CUDA tensor (got {x.device}); there is no CPU path")
    for name, t in (("x", x), ("y", y), ("hPost", hPost), ("hRes", hRes)):
        _require(t, name, x.device)
    if out is None:
        out = torch.empty_like(x)
    _require(out, "out", x.device, x.dtype, tuple(x.shape))
    desc = make_desc(B, S, n, D, _dtype_code(x.dtype), False)
    with _on_device(x.device):
        _check(lib().mhcPostRun(ctypes.byref(desc), _ptr(x), _ptr(y), _ptr(hPost), _ptr(hRes), _ptr(out),
                                _stream_ptr(stream)), "PostRun")
    return out
