"""ctypes binding of libgdn_b200.so (the C ABI declared in include/gdn_b200.h).

The library is the product: there is no CPU or PyTorch fallback.  If the
shared object is missing, importing an op raises immediately.
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libgdn_b200.so")

# status codes (include/gdn_b200.h)
GDN_OK = 0
GDN_ERR_NULL = 1
GDN_ERR_SHAPE = 2
GDN_ERR_DTYPE = 3
GDN_ERR_ALIGN = 4
GDN_ERR_UNSUPPORTED = 5
GDN_ERR_CUDA = 6
GDN_ERR_DEVICE = 7
GDN_ERR_DEVICE_TIMEOUT = 8
GDN_ERR_ARG = 9
GDN_BWD_AUTO, GDN_BWD_TOKEN, GDN_BWD_CHUNKED = 0, 1, 2

GDN_DTYPE_BF16 = 0
GDN_DTYPE_F32 = 1
GDN_LAYOUT_BHTD = 0
GDN_LAYOUT_BTHD = 1
GDN_SCHEDULE_AUTO = 0
GDN_SCHEDULE_SINGLE = 1
GDN_SCHEDULE_PIECED = 2
GDN_SCHEDULE_STREAM = 3
GDN_DECODE_L2NORM_QK = 1
GDN_GATES_BHT = 0
GDN_GATES_BTH = 1

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_Z = ctypes.c_size_t

class ProjOutSeg(ctypes.Structure):
    """gdn_proj_out_seg (include/gdn_b200.h): one output segment of gdn_proj_multi_fwd."""
    _fields_ = [("W", _P), ("y", _P), ("conv_w", _P), ("conv_state_in", _P), ("conv_state_out", _P),
                ("Dout", _I), ("l2norm_group", _I)]


class PrefillOpts(ctypes.Structure):
    """gdn_prefill_opts (include/gdn_b200.h): per-call options of gdn_prefill_fwd_ex."""
    _fields_ = [("schedule", _I), ("gate_layout", _I), ("gate_ld", ctypes.c_long)]


class ProjSegment(ctypes.Structure):
    """gdn_proj_segment (include/gdn_b200.h): one channel segment of gdn_decode_proj_fwd."""
    _fields_ = [("W", _P), ("y", _P), ("conv_w", _P), ("conv_state_in", _P), ("conv_state_out", _P),
                ("C", _I), ("ldy", _I), ("l2_group", _I)]


# name -> argtypes (every entry returns int unless listed in _STR_FUNCS)
SIGNATURES = {
    "gdn_prefill_fwd": [_P, _P, _P, _P, _P, _P, _I, _F, _P, _P, _P, _P, _P,
                        _I, _I, _I, _I, _I, _I, _I, _F, _P],
    "gdn_prefill_fwd_ws": [_P, _P, _P, _P, _P, _P, _I, _F, _P, _P, _P, _P, _P,
                           _I, _I, _I, _I, _I, _I, _I, _F, _P, _Z, _P],
    "gdn_prefill_fwd_ex": [_P, _P, _P, _P, _P, _P, _I, _F, _P, _P, _P, _P, _P,
                           _I, _I, _I, _I, _I, _I, _I, _F, _P, _P, _Z, _P],
    "gdn_prefill_window_ws": [_P, _P, _P, _P, _P, _P, _I, _F, _P, _P, _P, _P, _P,
                              _I, _I, _I, _I, _I, _I, _I, _I, _I, _F, _P, _Z, _P],
    "gdn_prefill_workspace_bytes": [_I, _I, _I, _I, _I],
    "gdn_prefill_fwd_noalloc": [_P, _P, _P, _P, _P, _P, _I, _F, _P, _P, _P, _P, _P,
                                _I, _I, _I, _I, _I, _I, _I, _F, _P],
    "gdn_prefill_varlen_fwd": [_P, _P, _P, _P, _P, _P, _I, _F, _P, _P, _I, _I, _I, _P, _P, _P,
                               _I, _I, _I, _I, _F, _P],
    "gdn_prefill_varlen_fwd_ws": [_P, _P, _P, _P, _P, _P, _I, _F, _P, _P, _I, _I, _I, _P, _P, _P,
                                  _I, _I, _I, _I, _F, _P, _Z, _P],
    "gdn_prefill_varlen_workspace_bytes": [_I, _I, _I, _I, _I],
    "gdn_prefill_host": [_P, _P, _P, _P, _P, _P, _I, _F, _P, _P, _P, _P, _P,
                         _I, _I, _I, _I, _I, _I, _I, _F, _I, _P, _Z, _P],
    "gdn_prefill_host_workspace_bytes": [_I, _I, _I, _I, _I, _I, _I, _I],
    "gdn_prefill_host_segment": [_I, _I, _I, _I, _I, _I, _I, _I],
    "gdn_prefill_host_plan": [_I, _I, _I, _I, _I, _I, _I, _I, ctypes.POINTER(ctypes.c_int), _I],
    "gdn_prefill_bwd": [_P, _P, _P, _P, _P, _P, _I, _F, _P, _P, _P, _P, _I, _P,
                        _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _Z, _P],
    "gdn_prefill_bwd_workspace_bytes": [_I, _I, _I, _I, _I],
    "gdn_prefill_bwd_set_window": [_I],
    "gdn_prefill_bwd_set_algorithm": [_I],
    "gdn_prefill_set_schedule": [_I],
    "gdn_prefill_launch_count": [_I, _I, _I, _I, _I],
    "gdn_prefill_launch_count_ex": [_I, _I, _I, _I, _I, _I],
    "gdn_decode_step": [_P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P],
    "gdn_decode_step_ex": [_P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _I, _P],
    "gdn_decode_step_gated": [_P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P, _F, _P,
                              _I, _I, _I, _I, _I, _F, _I, _P],
    "gdn_rmsnorm_fwd": [_P, _P, _P, _I, _I, _F, _P],
    "gdn_gated_rmsnorm_fwd": [_P, _I, _P, _P, _P, _I, _I, _F, _P],
    "gdn_decode_proj_fwd": [_P, _P, _F, _I, _I, ctypes.POINTER(ProjSegment), _I, _P],
    "gdn_proj_conv_silu_fwd": [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _I, _P],
    "gdn_proj_multi_fwd": [_P, _I, _I, _I, ctypes.POINTER(ProjOutSeg), _I, _P],
    "gdn_outproj_rs_fwd": [_P, _P, ctypes.POINTER(ctypes.c_void_p), _I, _I, _I, _I, _I, _P],
    "gdn_outproj_reduce": [_P, _P, _I, _I, _I, _P],
    "gdn_gather_window": [_P, ctypes.POINTER(ctypes.c_void_p), _I, _I, _I, _I, _I, _I, _I, _I, _I, _P],
    "gdn_check_device_error": [],
    "gdn_test_prefill_hooks": [ctypes.c_longlong, ctypes.c_longlong],
    "gdn_set_launch_overlap": [_I],
    "gdn_last_error": [],
    "gdn_version": [],
}
_STR_FUNCS = {"gdn_last_error", "gdn_version"}
_SIZE_FUNCS = {"gdn_prefill_workspace_bytes", "gdn_prefill_varlen_workspace_bytes", "gdn_prefill_bwd_workspace_bytes",
               "gdn_prefill_host_workspace_bytes"}

_lock = threading.Lock()
_lib = None


class GdnError(RuntimeError):
    """A libgdn_b200 entry point returned a non-zero status."""

    def __init__(self, func: str, status: int, message: str):
        super().__init__(f"{func}: {message} (status {status})")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load libgdn_b200.so once; raise if it has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with `python -m gdn_18646_b200.build` "
                        "(there is no fallback implementation)")
                handle = ctypes.CDLL(LIB_PATH)
                for name, args in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.argtypes = args
                    fn.restype = (ctypes.c_char_p if name in _STR_FUNCS else
                                  ctypes.c_size_t if name in _SIZE_FUNCS else ctypes.c_int)
                _lib = handle
    return _lib


def last_error() -> str:
    return lib().gdn_last_error().decode()


def call(name: str, *args) -> None:
    status = getattr(lib(), name)(*args)
    if status != GDN_OK:
        raise GdnError(name, status, last_error())


def call_status(name: str, *args) -> int:
    """Call without raising; returns the status code."""
    return getattr(lib(), name)(*args)
