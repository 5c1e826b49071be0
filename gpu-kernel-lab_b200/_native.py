"""ctypes binding of ``libkl_b200.so`` -- the C ABI declared in ``include/kl_b200.h``.

This is the only place Python touches the native library.  Every call passes
raw device pointers, sizes and the current CUDA stream; a non-zero status is
turned into an exception carrying ``kl_last_error()``.  There is no fallback:
if the library is missing or the device is not an sm_100 GPU the call raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().with_name("libkl_b200.so")

# ---- constants mirrored from include/kl_b200.h --------------------------------
KL_OK, KL_ERR_INVALID, KL_ERR_UNSUPPORTED, KL_ERR_CUDA, KL_ERR_WORKSPACE, KL_ERR_TIMEOUT = range(6)
KL_DT_BF16, KL_DT_F16, KL_DT_F32 = 0, 1, 2
KL_W8_ROW, KL_W8_GROUP, KL_W4_SYM, KL_W4_ASYM, KL_BF16_DENSE = range(5)
KL_FLAG_FORCE_SIMT, KL_FLAG_FORCE_TC, KL_FLAG_PDL, KL_FLAG_Y_TRANSPOSED, KL_FLAG_PERSISTENT = 1, 2, 4, 8, 16
KL_GROUPED_INT8_MMA = 1

EXPORTED_SYMBOLS = (
    "kl_linear", "kl_linear_workspace_bytes", "kl_project", "kl_int4_gemv",
    "kl_int4_lm_head_topk", "kl_int4_lm_head_topk_workspace_bytes", "kl_quantize_w8_row",
    "kl_quantize_w4", "kl_dequantize", "kl_status_string", "kl_last_error",
    "kl_device_status", "kl_version", "kl_describe_plan",
    "kl_grouped_table_bytes", "kl_grouped_encode", "kl_grouped_workspace_bytes", "kl_linear_grouped",
    "kl_linear_noalloc", "kl_topk_rows_workspace_bytes", "kl_topk_rows", "kl_topk_merge_rows", "kl_rmsnorm",
    "kl_linear_topk", "kl_linear_topk_workspace_bytes", "kl_grouped_digits_bytes", "kl_grouped_encode_ex",
)


class KlProblem(ctypes.Structure):
    """``kl_problem`` of include/kl_b200.h."""
    _fields_ = [("x", ctypes.c_void_p), ("w", ctypes.c_void_p), ("scales", ctypes.c_void_p),
                ("zeros", ctypes.c_void_p), ("y", ctypes.c_void_p), ("m", ctypes.c_int), ("n", ctypes.c_int),
                ("k", ctypes.c_int), ("group", ctypes.c_int)]

_P, _I, _S = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
_SIGNATURES = {
    "kl_linear": (_I, [_P, _I, _I, _I, _P, _I, _I, _I, _P, _P, _P, _I, _P, _P, _S, _I, _P]),
    "kl_linear_workspace_bytes": (_S, [_I, _I, _I, _I, _I, _I]),
    "kl_project": (_I, [_P, _I, _P, _I, _P, _P, _I, _I, _I, _I, _I, _P, _P, _S, _P]),
    "kl_int4_gemv": (_I, [_P, _I, _I, _P, _P, _I, _I, _I, _P, _P]),
    "kl_int4_lm_head_topk": (_I, [_P, _I, _I, _P, _P, _I, _I, _I, _I, _P, _P, _P, _S, _P]),
    "kl_int4_lm_head_topk_workspace_bytes": (_S, [_I, _I, _I]),
    "kl_quantize_w8_row": (_I, [_P, _I, _I, _I, _P, _P, _P]),
    "kl_quantize_w4": (_I, [_P, _I, _I, _I, _I, _I, _P, _P, _P, _P]),
    "kl_dequantize": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _P, _P]),
    "kl_status_string": (ctypes.c_char_p, [_I]),
    "kl_last_error": (ctypes.c_char_p, []),
    "kl_device_status": (_I, [_I, _I]),
    "kl_version": (_I, []),
    "kl_describe_plan": (_I, [_I, _I, _I, _I, _I, _I, _I, ctypes.POINTER(ctypes.c_int)]),
    "kl_grouped_table_bytes": (_S, [_I]),
    "kl_grouped_encode": (_I, [_P, _I, _I, _I, _I, _P, _S]),
    "kl_grouped_workspace_bytes": (_S, [_P]),
    "kl_grouped_digits_bytes": (_S, [_P, _I, _I]),
    "kl_grouped_encode_ex": (_I, [_P, _I, _I, _I, _I, _I, _P, _S, _P, _S]),
    "kl_linear_grouped": (_I, [_P, _P, _P, _S, _I, _P]),
    "kl_linear_noalloc": (_I, [_P, _I, _I, _I, _P, _I, _P, _I, _P, _P]),
    "kl_topk_rows_workspace_bytes": (_S, [_I, _I, _I]),
    "kl_topk_rows": (_I, [_P, _I, _I, _I, ctypes.c_longlong, ctypes.c_longlong, _I, _P, _P, _P, _S, _P]),
    "kl_topk_merge_rows": (_I, [_P, _I, _I, _I, _P, _P, _P]),
    "kl_rmsnorm": (_I, [_P, _P, _P, _I, _I, _I, ctypes.c_float, _I, _P, _P, _P]),
    "kl_linear_topk": (_I, [_P, _I, _I, _I, _P, _I, _I, _I, _P, _P, _I, ctypes.c_longlong, _P, _P, _P, _S, _I, _P]),
    "kl_linear_topk_workspace_bytes": (_S, [_I, _I, _I, _I, _I]),
}

_lib = None
_lock = threading.Lock()


class NativeError(RuntimeError):
    """A non-OK status from libkl_b200 (the reference's TORCH_CHECK -> RuntimeError)."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def lib() -> ctypes.CDLL:
    """Load libkl_b200.so (once) and declare the C signatures."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"{LIB_PATH.name} is not built: run __graft_entry__.build() "
                        "(nvcc for sm_100a) before using the quantized linear ops")
                handle = ctypes.CDLL(str(LIB_PATH))
                for name, (res, args) in _SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = handle
    return _lib


def check(status: int, exc=NativeError) -> None:
    if status != KL_OK:
        l = lib()
        msg = f"{l.kl_status_string(status).decode()}: {l.kl_last_error().decode()}"
        if exc is NativeError:
            raise NativeError(status, msg)
        raise exc(msg)


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_handle(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def act_dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return KL_DT_BF16
    if dtype == torch.float16:
        return KL_DT_F16
    if dtype == torch.float32:
        return KL_DT_F32
    raise ValueError(f"unsupported dtype {dtype}")


# ---- workspaces ---------------------------------------------------------------
# The persistent tcgen05 kernel's split-K fixup needs scratch (arrival counters
# that must start at zero, plus f32 partial tiles).  A zero-initialised buffer
# is kept per device for the default stream and for CUDA-graph capture, and
# one per (device, stream) for every other stream, so that calls on different
# streams never share scratch; each grows on demand and the kernels leave the
# counters at zero.  (Captured graphs replayed concurrently on different
# streams should pass their own ``workspace``.)
_workspaces: dict = {}
_retired_workspaces: list = []


def workspace(device: torch.device, nbytes: int, stream=None) -> torch.Tensor | None:
    if nbytes == 0:
        return None
    idx = device.index if device.index is not None else torch.cuda.current_device()
    capturing = torch.cuda.is_current_stream_capturing()
    key = idx
    if stream is not None and not capturing and stream != torch.cuda.default_stream(idx):
        key = (idx, stream.cuda_stream)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        if capturing:
            raise RuntimeError("the first quantized-linear call on a device must happen before CUDA-graph "
                               "capture (it allocates the device workspace); run one warm-up call first")
        buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=torch.device("cuda", idx))
        if key in _workspaces:
            # CUDA graphs captured earlier may still point at the old buffer: keep it alive
            _retired_workspaces.append(_workspaces[key])
        _workspaces[key] = buf
    return buf


def describe_plan(m: int, n: int, k: int, w_format: int, swiglu: bool = False, flags: int = 0,
                  sm_count: int = 148) -> dict:
    """Host-only launch plan + partition self-check (no GPU needed)."""
    out = (ctypes.c_int * 8)()
    check(lib().kl_describe_plan(m, n, k, w_format, int(swiglu), flags, sm_count, out))
    keys = ("kernel", "grid", "threads", "smem", "n_mma", "stages", "tiles", "units")
    return dict(zip(keys, list(out)))


def device_status(device: int = 0, reset: bool = False) -> int:
    return lib().kl_device_status(device, int(reset))
