"""ctypes binding of libquipsharp_b200.so (the C ABI declared in include/quipsharp_b200.h).

The library is built in-tree by `python -m quipsharp_b200.build_native` (or
`__graft_entry__.build()`).  There is deliberately no fallback: if the library
is missing, every CUDA entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libquipsharp_b200.so")

QS_OK = 0
QS_ERR_INVALID_ARG = 1
QS_ERR_NOT_POW2 = 2
QS_ERR_ODD_DIM = 3
QS_ERR_INDEX = 4
QS_ERR_UNSUPPORTED = 5
QS_ERR_ALIGNMENT = 6
QS_ERR_CUDA = 7
QS_ERR_WORKSPACE = 8
QS_ERR_TIMEOUT = 9

QS_CB_E8P = 0
QS_CB_E8_1BIT = 1

QS_F32, QS_F16, QS_BF16, QS_I16, QS_I32, QS_I64 = range(6)
QS_RHT, QS_RFFT = 0, 1

IO_DTYPES = {torch.float32: QS_F32, torch.float16: QS_F16, torch.bfloat16: QS_BF16}
CODE_DTYPES = {torch.int16: QS_I16, torch.int32: QS_I32, torch.int64: QS_I64}

# name -> (restype, argtypes)
_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_SIGS = {
    "qs_version": (ctypes.c_char_p, []),
    "qs_last_error": (ctypes.c_char_p, []),
    "qs_device_status": (_I, [_P]),
    "qs_set_wait_limit_ns": (_I, [ctypes.c_uint64]),
    "qs_wait_limit_ns": (ctypes.c_uint64, []),
    "qs_codebook_table": (_I, [_I, _P]),
    "qs_decode": (_I, [_I, _P, _I, _L, _P, _P]),
    "qs_rvq_decode": (_I, [_I, _P, _P, _I, _P, _L, _P, _P]),
    "qs_dequantize_linear": (_I, [_P, _I, _P, _P, _P, _L, _L, _P, _P]),
    "qs_fwht": (_I, [_P, _L, _P, _L, _I, _L, _L, _P, _P, _P]),
    "qs_rfft": (_I, [_I, _P, _L, _P, _L, _I, _L, _L, _P, _P]),
    "qs_packed_bytes": (_L, [_I, _P, _L, _L]),
    "qs_pack_codes": (_I, [_P, _I, _P, _L, _L, _P, _L, _P]),
    "qs_linear_workspace_bytes": (_L, [_L, _L, _L]),
    "qs_linear_fwd": (_I, [_P, _I, _L, _L, _L, _P, _I, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P,
                           _P, _L, _P]),
    "qs_linear_fwd_group": (_I, [_P, _I, _L, _L, _I, _P, _P]),
    "qs_linear_fwd_noalloc": (_I, [_P, _I, _L, _L, _L, _P, _I, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P,
                                   _P]),
    "qs_linear_input_bytes": (_L, [_L, _L]),
    "qs_linear_input": (_I, [_P, _I, _L, _L, _I, _P, _P, _P, _L, _P, _L, _P]),
    "qs_linear_matmul": (_I, [_P, _L, _L, _L, _P, _I, _P, _P, _P, _P, _P]),
    "qs_linear_output": (_I, [_P, _L, _L, _L, _L, _I, _P, _P, _P, _P, _I, _P]),
    "qs_ipc_export": (_I, [_P, _P, _P]),
    "qs_ipc_import": (_I, [_P, _L, _P]),
    "qs_ipc_close": (_I, [_P, _L]),
    "qs_linear_tp_workspace_bytes": (_L, [_L, _L, _L]),
    "qs_fit_workspace_bytes": (_L, [_L, _I]),
    "qs_fit_scale_sweep": (_I, [_P, _L, _I, _P, _P, _I, _I, _P, _P, _P, _I, _P, _L, _P, _P, _P]),
    "qs_tp_push": (_I, [_P, _P, _L, _L, _P]),
    "qs_linear_matmul_tp": (_I, [_P, _L, _L, _L, _P, _I, _P, _P, _P, _P, _P, _P]),
    "qs_linear_output_peers": (_I, [_P, _L, _L, _I, _P, _P, _P, _P, _I, _P]),
    "qs_linear_fwd_tp": (_I, [_P, _I, _L, _L, _L, _P, _I, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P, _L, _P,
                              _P]),
}

QS_TP_MAX_RANKS = 8


class TPPeers(ctypes.Structure):
    """qs_tp_peers (include/quipsharp_b200.h): every rank's receive buffer and
    flag array as mapped in this process, and this rank's control words."""
    _fields_ = [("world", ctypes.c_int), ("rank", ctypes.c_int),
                ("recv", ctypes.c_void_p * QS_TP_MAX_RANKS),
                ("flags", ctypes.c_void_p * QS_TP_MAX_RANKS),
                ("ctl", ctypes.c_void_p),
                ("recv_floats", ctypes.c_int64)]


QS_GROUP_MAX_LAYERS = 8


class LinearLayer(ctypes.Structure):
    """qs_linear_layer (include/quipsharp_b200.h): one layer of
    qs_linear_fwd_group."""
    _fields_ = [("m", ctypes.c_int64), ("packed", ctypes.c_void_p), ("stages", ctypes.c_int),
                ("kinds", ctypes.c_void_p), ("stage_scales", ctypes.c_void_p),
                ("layer_scale", ctypes.c_void_p), ("transform", ctypes.c_int),
                ("su", ctypes.c_void_p), ("sv", ctypes.c_void_p),
                ("phase_u", ctypes.c_void_p), ("phase_v", ctypes.c_void_p),
                ("bias", ctypes.c_void_p), ("y", ctypes.c_void_p),
                ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_int64)]


EXPORTS = tuple(_SIGS)

_lib = None
_lock = threading.Lock()


class NativeLibraryMissing(RuntimeError):
    pass


def lib():
    """Load (once) and return the ctypes handle of the CUDA library."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(_LIB_PATH):
                    raise NativeLibraryMissing(
                        f"quipsharp_b200 CUDA library not built ({_LIB_PATH} missing); "
                        "run `python -m quipsharp_b200.build_native`")
                h = ctypes.CDLL(_LIB_PATH)
                for name, (res, args) in _SIGS.items():
                    fn = getattr(h, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = h
    return _lib


def library_path() -> str:
    return _LIB_PATH


def check(status: int) -> None:
    """Raise the exception the reference raises for the same condition."""
    if status == QS_OK:
        return
    msg = (lib().qs_last_error() or b"").decode(errors="replace")
    if status == QS_ERR_NOT_POW2:
        raise ValueError(msg)
    if status == QS_ERR_ODD_DIM:
        raise AssertionError(msg)
    if status == QS_ERR_INDEX:
        raise IndexError(msg)
    if status == QS_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(f"quipsharp_b200 error {status}: {msg}")


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*tensors) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("quipsharp_b200 runs on CUDA tensors only (no CPU path); "
                               f"got a tensor on {t.device}")


def int_array(vals):
    arr = (ctypes.c_int * len(vals))(*vals)
    return arr


def float_array(vals):
    return (ctypes.c_float * len(vals))(*vals)
