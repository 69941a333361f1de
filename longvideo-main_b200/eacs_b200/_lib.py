"""ctypes binding of libeacs_b200.so (the C ABI in include/eacs_b200.h).

There is no CPU or PyTorch fallback: if the library is missing or a call
fails, a RuntimeError is raised with the library's own message.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
# EACS_B200_LIB may point at another build of the same library.
LIB_PATH = os.environ.get("EACS_B200_LIB") or os.path.join(_HERE, "libeacs_b200.so")

EACS_OK = 0
EACS_ERR_INVALID = 1
EACS_ERR_CUDA = 2
EACS_ERR_WORKSPACE = 3
EACS_ERR_TIMEOUT = 4
EACS_ERR_UNSUPPORTED = 5

DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_F = ctypes.c_float
_I = ctypes.c_int
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/eacs_b200.h
SIGNATURES = {
    "eacs_version": (ctypes.c_char_p, []),
    "eacs_last_error": (ctypes.c_char_p, []),
    "eacs_device_status": (_I, [ctypes.POINTER(_I), _P]),
    "eacs_kernel_launches": (ctypes.c_uint64, []),
    "eacs_wait_selftest": (_I, [_I, _P]),
    "eacs_project": (_I, [_P, _I, _P, _P, _F, _P, _I, _I64, _P, _P, _I, _P, _P, _P, _SZ,
                          _I64, _I64, _I64, _I64, _P]),
    "eacs_project_workspace_size": (_SZ, [_I64]),
    "eacs_set_kernel_events": (_I, [_P, _P]),
    "eacs_scan_fwd": (_I, [_P, _P, _P, _I64, _I64, _I64, _I64, _P]),
    "eacs_scan_bwd": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P]),
    "eacs_ssm_fwd": (_I, [_P, _P, _P, _P, _P, _P, _I, _P, _P, _I64, _I64, _I64, _I64, _F, _F, _P]),
    "eacs_zoh_kernels": (_I, [_P, _P, _P, _P, _I64, _I64, _I64, _P]),
    "eacs_ssm_ckpt_size": (_SZ, [_I64, _I64, _I64, _I64]),
    "eacs_ssm_train_fwd": (_I, [_P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _SZ,
                                _I64, _I64, _I64, _I64, _F, _F, _P]),
    "eacs_cell_commits_workspace_size": (_SZ, [_I64, _I64, _I64, _I64]),
    "eacs_cell_commits": (_I, [_P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _F, _F, _F, _F, _F, _F,
                               _I, _I, _F, _F, _P, _P, _P, _P, _P, _P, _P, _P, _P, _SZ,
                               _I64, _I64, _I64, _I64, _P]),
    "eacs_query_index": (_I, [_P, _P, _P, _I64, _I64, _I64, _P]),
    "eacs_query_readout": (_I, [_P] * 11 + [_I64] * 5 + [_F, _F, _P]),
    "eacs_branch_fuse": (_I, [_P, _P, _I, _I, _P, _P, _P, _P, _F, _P, _P, _I64, _I64, _P]),
    "eacs_fc_open": (_I, [ctypes.c_char_p, ctypes.POINTER(_P)]),
    "eacs_fc_info": (_I, [_P, ctypes.POINTER(_I64), ctypes.POINTER(_I64), ctypes.POINTER(_I64),
                          ctypes.POINTER(_I)]),
    "eacs_fc_timestamps": (_I, [_P, _P]),
    "eacs_fc_read": (_I, [_P, _I64, _I64, _P]),
    "eacs_fc_upload": (_I, [_P, _I64, _I64, _P, _SZ, _P, _P]),
    "eacs_fc_close": (None, [_P]),
    "eacs_cell_fwd_host_workspace_size": (_SZ, [_I64] * 5),
    "eacs_cell_fwd_host": (_I, [_P] * 6 + [_I] + [_P] * 3 + [_F] * 6 + [_I, _I, _F, _F]
                           + [_P] * 4 + [_SZ] + [_I64] * 5 + [_P]),
    "eacs_stream_chunk": (_I, [_P] * 6 + [_I] + [_P] * 21 + [_F] * 7 + [_I, _F]
                          + [_I64] * 4 + [_P]),
    "eacs_stream_frame_workspace_size": (_SZ, [_P, _I, _I64, _I64]),
    "eacs_stream_frame": (_I, [_P] * 5 + [_I] + [_P] * 4 + [_F] + [_P] * 6 + [_SZ, _I64, _I64, _P]),
    "eacs_stream_step_bwd_workspace_size": (_SZ, [_I64] * 3),
    "eacs_stream_step_bwd": (_I, [_P] * 41 + [_P, _SZ] + [_F] * 7 + [_I, _F] + [_I64] * 3 + [_P]),
    "eacs_ssm_bwd_workspace_size": (_SZ, [_I64, _I64, _I64, _I64]),
    "eacs_ssm_bwd": (_I, [_P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _SZ,
                          _P, _P, _P, _P, _P, _P, _P, _P, _SZ,
                          _I64, _I64, _I64, _I64, _F, _F, _P]),
    "eacs_cell_fwd_workspace_size": (ctypes.c_size_t, [_I64, _I64, _I64, _I64]),
    "eacs_cell_fwd": (_I, [_P, _P, _P, _I, _P, _P, _P, _P, _P, _P,
                           _F, _F, _F, _F, _F, _F, _I, _I, _F, _F, _I, _F,
                           _P, _P, _P, _P, ctypes.c_size_t, _I64, _I64, _I64, _I64, _P]),
    "eacs_cell_fwd_side_by_side": (_I, [_P, _P, _P, _I, _P, _P, _P, _P, _P, _P,
                                        _F, _F, _F, _F, _F, _F, _I, _I, _F, _F, _I, _F,
                                        _P, _P, _P, _P, ctypes.c_size_t, _I64, _I64, _I64, _I64,
                                        _I, _P]),
    "eacs_cell_train_fwd": (_I, [_P, _P, _P, _I, _P, _P, _P, _P, _P, _P,
                                 _F, _F, _F, _F, _F, _F, _I, _F,
                                 _P, _P, _P, _P, _P, ctypes.c_size_t, _I64, _I64, _I64, _I64, _P]),
    "eacs_cell_train_bwd_workspace_size": (ctypes.c_size_t, [_I64, _I64, _I64, _I64]),
    "eacs_cell_train_bwd": (_I, [_P, _P, _P, _I, _P, _P, _P, _P, _P, _P,
                                 _F, _F, _F, _F, _F, _F, _F,
                                 _P, _P, _P, _P, _P, _P, _P,
                                 _P, _P, _P, _P, _P, _P, _P, _P,
                                 _P, ctypes.c_size_t, _I64, _I64, _I64, _I64, _P]),
    "eacs_cell_train_fwd_ckpt": (_I, [_P, _P, _P, _I, _P, _P, _P, _P, _P, _P,
                                      _F, _F, _F, _F, _F, _F, _I, _F,
                                      _P, _P, _P, _P, _P, ctypes.c_size_t, _P, ctypes.c_size_t,
                                      _I64, _I64, _I64, _I64, _P]),
    "eacs_cell_train_bwd_ckpt": (_I, [_P, _P, _P, _I, _P, _P, _P, _P, _P, _P,
                                      _F, _F, _F, _F, _F, _F, _F,
                                      _P, _P, _P, _P, _P, _P, _P,
                                      _P, _P, _P, _P, _P, _P, _P, _P,
                                      _P, ctypes.c_size_t, _I64, _I64, _I64, _I64, _P]),
    "eacs_cell_train_commits_workspace_size": (_SZ, [_I64, _I64, _I64, _I64]),
    "eacs_cell_train_commits_fwd": (_I, [_P, _P, _P, _I, _P, _P, _P, _P, _P, _P,
                                         _F, _F, _F, _F, _F, _F, _I, _F,
                                         _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                         _P, _SZ, _P, _SZ, _I64, _I64, _I64, _I64, _P]),
    "eacs_cell_train_commits_bwd": (_I, [_P, _P, _P, _I, _P, _P, _P, _P, _P, _P,
                                         _F, _F, _F, _F, _F, _F, _I, _F,
                                         _P, _P, _P, _P, _P, _P,
                                         _P, _P, _P, _P, _P,
                                         _P, _P, _P, _P, _P, _P, _P, _P,
                                         _P, _SZ, _I64, _I64, _I64, _I64, _P]),
    "eacs_query_readout_bwd_workspace_size": (_SZ, [_I64] * 5),
    "eacs_query_readout_bwd": (_I, [_P] * 20 + [_P, _SZ] + [_I64] * 5 + [_F, _F, _P]),
    "eacs_cell_fwd_noalloc": (_I, [_P, _P, _P, _I, _P, _P, _P, _P, _P, _P,
                                   _F, _F, _F, _F, _F, _F, _I, _I, _F, _F, _I, _F,
                                   _P, _P, _P, _I64, _I64, _I64, _I64, _P]),
}

_lib = None
_lock = threading.Lock()
calls = {}  # entry point -> number of successful calls (proves the native path ran)


def lib() -> ctypes.CDLL:
    """Load the shared library (once); raise if it is not built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"eacs_b200: {LIB_PATH} is missing; build it with "
                        "`make -C longvideo-main_b200/csrc` (or __graft_entry__.build())")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def last_error() -> str:
    return lib().eacs_last_error().decode()


def check(rc: int, name: str) -> None:
    if rc != EACS_OK:
        raise RuntimeError(f"eacs_b200.{name} failed (code {rc}): {last_error()}")
    calls[name] = calls.get(name, 0) + 1


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def device_status(device: torch.device | None = None) -> int:
    """Synchronise the current stream and read/clear the device status word."""
    st = _I(0)
    check(lib().eacs_device_status(ctypes.byref(st), stream_ptr(device)), "eacs_device_status")
    return st.value


def kernel_launches() -> int:
    """Kernel launches issued by libeacs_b200.so in this process."""
    return int(lib().eacs_kernel_launches())


def set_kernel_events(start: "torch.cuda.Event | None", stop: "torch.cuda.Event | None") -> None:
    """Record start/stop around the dominant kernel of each later call (this thread)."""
    if start is None or stop is None:
        lib().eacs_set_kernel_events(None, None)
    else:
        lib().eacs_set_kernel_events(start.cuda_event, stop.cuda_event)


def version() -> str:
    return lib().eacs_version().decode()
