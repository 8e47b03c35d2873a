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

F16 = 0
BF16 = 1

STATUS_NAMES = {
    0: "SUCCESS", -1: "NULL_POINTER", -2: "BAD_SHAPE", -3: "BAD_STREAM_COUNT", -4: "BAD_HEAD_DIM",
    -5: "MIX_TOO_LARGE", -6: "BAD_DTYPE", -7: "MISALIGNED", -8: "WORKSPACE_TOO_SMALL", -9: "CUDA_ERROR",
    -10: "UNSUPPORTED_DEVICE", -11: "DEVICE_TIMEOUT", -12: "NOT_PREPARED", -13: "TOO_LARGE",
}

EXPORTED_SYMBOLS = (
    "mhcPreGetWorkspaceSize", "mhcPrePrepareWeights", "mhcPreRun", "mhcPreRunPrepared",
    "mhcPreRunPreparedProfiled", "mhcPreQueryPlan", "mhcPreGetDeviceStatus", "mhcPreStatusString",
    "mhcPreAbiVersion", "mhcPreRunNoAlloc", "mhcPreDiagWaitTimeout", "mhcPostRun",
)


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


_lib = None


def lib():
    """Loads libmhcpre_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run `python -m mhcpre_review_b200.build` "
                               "(the operator has no CPU fallback)")
        L = ctypes.CDLL(str(LIB_PATH))
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
        L.mhcPreGetDeviceStatus.argtypes = [ctypes.POINTER(ctypes.c_int32)]
        L.mhcPreStatusString.argtypes = [ctypes.c_int]
        L.mhcPreStatusString.restype = ctypes.c_char_p
        L.mhcPreAbiVersion.argtypes = []
        for name in EXPORTED_SYMBOLS:
            if name != "mhcPreStatusString":
                getattr(L, name).restype = ctypes.c_int
        _lib = L
    return _lib


def _check(rc: int, what: str):
    if rc != 0:
        raise MhcPreError(rc, what)


def make_desc(batch, seq, streams, head_dim, dtype, has_gamma, norm_eps=1e-6, hc_eps=1e-6) -> MhcPreDesc:
    return MhcPreDesc(int(batch), int(seq), int(streams), int(head_dim), int(dtype), int(bool(has_gamma)),
                      float(norm_eps), float(hc_eps))


def workspace_size(desc: MhcPreDesc) -> int:
    n = ctypes.c_size_t(0)
    _check(lib().mhcPreGetWorkspaceSize(ctypes.byref(desc), ctypes.byref(n)), "GetWorkspaceSize")
    return int(n.value)


def query_plan(desc: MhcPreDesc) -> dict:
    p = MhcPrePlan()
    _check(lib().mhcPreQueryPlan(ctypes.byref(desc), ctypes.byref(p)), "QueryPlan")
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


def _stream_ptr(stream):
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


class MhcPre:
    """Reusable executor: owns the workspace and the prepared weights."""

    def __init__(self, batch, seq, streams, head_dim, dtype, has_gamma, norm_eps=1e-6, hc_eps=1e-6,
                 device=None, workspace=None):
        torch = _torch()
        self.desc = make_desc(batch, seq, streams, head_dim,
                              dtype if isinstance(dtype, int) else _dtype_code(dtype), has_gamma, norm_eps, hc_eps)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.ws_bytes = workspace_size(self.desc)
        if workspace is None:
            workspace = torch.empty(self.ws_bytes, dtype=torch.uint8, device=self.device)
        elif workspace.numel() * workspace.element_size() < self.ws_bytes:
            raise MhcPreError(-8, "workspace")
        self.workspace = workspace
        self.prepared = False

    @property
    def plan(self) -> dict:
        return query_plan(self.desc)

    def prepare(self, phi, gamma=None, stream=None):
        _check(lib().mhcPrePrepareWeights(ctypes.byref(self.desc), _ptr(phi), _ptr(gamma), _ptr(self.workspace),
                                          self.ws_bytes, _stream_ptr(stream)), "PrepareWeights")
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
        hIn, hPost, hRes = out
        _check(lib().mhcPreRunPreparedProfiled(ctypes.byref(self.desc), _ptr(x), _ptr(alpha), _ptr(bias), _ptr(hIn),
                                               _ptr(hPost), _ptr(hRes), _ptr(self.workspace), self.ws_bytes,
                                               _stream_ptr(stream), ctypes.c_void_p(ev_begin.cuda_event),
                                               ctypes.c_void_p(ev_end.cuda_event)), "RunPreparedProfiled")
        return hIn, hPost, hRes

    def __call__(self, x, alpha, bias, out=None, stream=None):
        hIn, hPost, hRes = out if out is not None else self.outputs(x.dtype)
        _check(lib().mhcPreRunPrepared(ctypes.byref(self.desc), _ptr(x), _ptr(alpha), _ptr(bias), _ptr(hIn),
                                       _ptr(hPost), _ptr(hRes), _ptr(self.workspace), self.ws_bytes,
                                       _stream_ptr(stream)), "RunPrepared")
        return hIn, hPost, hRes


def mhc_pre(x, phi, alpha, bias, gamma=None, norm_eps=1e-6, hc_eps=1e-6, out=None, workspace=None, stream=None):
    """One-shot MhcPre (prepare + run).  x: [B, S, n, D] fp16/bf16 CUDA tensor;
    phi: fp32 [mix, n*D] (the reference's K-contiguous layout); alpha: fp32 [3];
    bias: fp32 [mix]; gamma: fp32 [n, D] or None.  Returns (hIn [B,S,D], hPost [B,S,n],
    hRes [B,S,n,n])."""
    if x.dim() != 4:
        raise MhcPreError(-2, "x must be 4-D [B, S, n, D]")
    B, S, n, D = x.shape
    ex = MhcPre(B, S, n, D, x.dtype, gamma is not None, norm_eps, hc_eps, device=x.device, workspace=workspace)
    hIn, hPost, hRes = out if out is not None else ex.outputs(x.dtype)
    _check(lib().mhcPreRun(ctypes.byref(ex.desc), _ptr(x), _ptr(phi), _ptr(alpha), _ptr(bias), _ptr(gamma),
                           _ptr(hIn), _ptr(hPost), _ptr(hRes), _ptr(ex.workspace), ex.ws_bytes,
                           _stream_ptr(stream)), "Run")
    return hIn, hPost, hRes


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
    for t in (x, y, hPost, hRes):
        if not t.is_contiguous():
            raise MhcPreError(-2, "tensors must be contiguous")
    if out is None:
        out = torch.empty_like(x)
    desc = make_desc(B, S, n, D, _dtype_code(x.dtype), False)
    _check(lib().mhcPostRun(ctypes.byref(desc), _ptr(x), _ptr(y), _ptr(hPost), _ptr(hRes), _ptr(out),
                            _stream_ptr(stream)), "PostRun")
    return out
