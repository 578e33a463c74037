"""ctypes binding of libpackr_b200.so (declarations: include/packr_b200.h).

The library is built in-tree by packr_b200.build.  There is no fallback: if
the library is missing or the device is not sm_100, every op raises.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

# PACKR_B200_LIB selects another build of the library (the same ABI)
_LIB_PATH = Path(os.environ.get("PACKR_B200_LIB") or Path(__file__).resolve().parent / "libpackr_b200.so")
_lock = threading.Lock()
_lib = None

PACKR_OK = 0
PACKR_DTYPE_F32 = 0
PACKR_DTYPE_BF16 = 1
PACKR_DTYPE_F16 = 2

_ERRORS = {
    1: "invalid argument", 2: "bad shape", 3: "misaligned pointer or stride", 4: "workspace too small",
    5: "kernel launch failed", 6: "current device is not sm_100", 7: "device-side wait timed out",
    8: "CUDA error",
}


class PackRError(RuntimeError):
    def __init__(self, fn: str, code: int):
        super().__init__(f"{fn} failed: {_ERRORS.get(code, 'unknown')} (status {code})")
        self.code = code


class AdamTensor(ctypes.Structure):
    _fields_ = [
        ("p", ctypes.c_void_p), ("g", ctypes.c_void_p), ("m", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("m_scale", ctypes.c_void_p), ("v_scale", ctypes.c_void_p), ("numel", ctypes.c_int64),
        ("dtype", ctypes.c_int32), ("reserved", ctypes.c_int32),
    ]


# name -> (restype, argtypes); the exported surface of include/packr_b200.h
_VP, _I64, _I32, _F32, _SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
SIGNATURES = {
    "packr_error_string": (ctypes.c_char_p, [_I32]),
    "packr_abi_version": (_I32, []),
    "packr_device_status": (_I32, [_VP]),
    "packr_adam8_multi": (_I32, [ctypes.POINTER(AdamTensor), _I32, _F32, _F32, _F32, _F32, _F32, _F32, _F32, _VP]),
    "packr_adam8_multi_push": (_I32, [ctypes.POINTER(AdamTensor), _I32, ctypes.POINTER(_VP), _I32, _F32, _F32, _F32,
                                      _F32, _F32, _F32, _F32, _VP]),
    "packr_device_alloc": (_I32, [_SZ, ctypes.POINTER(_VP)]),
    "packr_device_free": (_I32, [_VP]),
    "packr_ipc_export": (_I32, [_VP, _VP]),
    "packr_ipc_open": (_I32, [_VP, ctypes.POINTER(_VP)]),
    "packr_ipc_close": (_I32, [_VP]),
    "packr_forward_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I32]),
    "packr_forward": (_I32, [_VP, _I32, _VP, _VP, _VP, _VP, _I32, _VP, _I64, _I64, _I64, _VP, _SZ, _VP]),
    "packr_forward_decoded_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I32]),
    "packr_forward_decoded": (_I32, [_VP, _I32, _VP, _VP, _I32, _VP, _I64, _I64, _I64, _VP, _SZ, _VP]),
    "packr_backward_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I32, _I32]),
    "packr_backward": (_I32, [_VP, _VP, _I32, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I64, _I64, _I64, _I32, _VP,
                              _SZ, _VP]),
    "packr_bincount256": (_I32, [_VP, _I64, _VP, _VP]),
    "packr_lut_finalize": (_I32, [_VP, _VP, _VP, _VP]),
    "packr_decode_bf16": (_I32, [_VP, _VP, _VP, _VP, _I64, _I64, _VP]),
    "packr_predecode_bf16": (_I32, [_VP, _VP, _VP, _VP, _I64, _I64, _VP]),
    "packr_selfcheck_rounding": (_I32, [_VP, _VP]),
    "packr_backward_decoded_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I32, _I32]),
    "packr_backward_decoded": (_I32, [_VP, _VP, _I32, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I64, _I64,
                                      _I64, _I32, _VP, _SZ, _VP]),
    "packr_predecode_route": (_I32, [_I64, _I64, _I64, _VP, _VP]),
    "packr_abs_order_stats_workspace_bytes": (_SZ, []),
    "packr_abs_order_stats": (_I32, [_VP, _I32, _I64, _I64, _I64, _VP, _VP, _SZ, _VP]),
    "packr_from_linear_encode": (_I32, [_VP, _I32, _I64, _I64, _VP, _VP, _VP, _VP, _VP, _VP, _VP]),
    "packr_state_v_sums": (_I32, [_VP, _I32, _VP, _VP]),
    "packr_backward_static_scratch": (_I32, [_VP, _VP, _I32, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I64, _I64,
                                             _I64, _I32, _VP]),
}
PACKR_BWD_DW_SPLIT = 1
PACKR_IPC_HANDLE_BYTES = 64


class VSumDesc(ctypes.Structure):
    _fields_ = [("v", _VP), ("v_scale", _VP), ("numel", _I64), ("block_size", _I64), ("block_origin", _I64)]


def lib_path() -> Path:
    return _LIB_PATH


def load():
    """Loads (once) and returns the library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not _LIB_PATH.exists():
                raise ImportError(
                    f"{_LIB_PATH} is not built: run `python -m packr_b200.build` (needs nvcc, CUDA 12.9)")
            lib = ctypes.CDLL(str(_LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(fn: str, code: int) -> None:
    if code != PACKR_OK:
        raise PackRError(fn, code)
