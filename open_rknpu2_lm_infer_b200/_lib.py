"""ctypes binding of libqlinear_b200.so (the C ABI declared in include/qlinear.h).

The shared library is built in-tree (``open_rknpu2_lm_infer_b200/lib/``) by
``__graft_entry__.build()`` or ``make -C open_rknpu2_lm_infer_b200/csrc``.  There is no
fallback: if the library is missing, loading it raises ``QLinearUnavailable``.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libqlinear_b200.so")

QLINEAR_OK = 0
QLINEAR_ERR_PARAM = -1
QLINEAR_ERR_ALLOC = -2
QLINEAR_ERR_CUDA = -3
QLINEAR_ERR_UNSUPPORTED = -4
QLINEAR_ERR_TIMEOUT = -5
QLINEAR_ERR_NCCL = -6
QLINEAR_ERR_STATE = -7
QLINEAR_ERR_LIMIT = -8
NOALLOC_MAX_ROWS = 8
NOALLOC_MAX_K = 16384

ROUND_AWAY = 0
ROUND_EVEN = 1

F32, F16, I32 = 0, 1, 2
RUN_SWIGLU = 1


class QLinearUnavailable(RuntimeError):
    pass


BACKEND_W4_PACKED_ONLY = 1
BACKEND_GEMM_STREAM_K = 2
BACKEND_SWIGLU_UNFUSED = 4
IPC_HANDLE_BYTES = 64


class BackendConfig(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("round_mode", ctypes.c_int),
                ("max_rows", ctypes.c_int), ("flags", ctypes.c_uint)]


class WeightConfig(ctypes.Structure):
    _fields_ = [("bits", ctypes.c_int), ("K", ctypes.c_int), ("N", ctypes.c_int),
                ("reserved", ctypes.c_int)]


class WeightInfo(ctypes.Structure):
    _fields_ = [("bits", ctypes.c_int), ("K", ctypes.c_int), ("N", ctypes.c_int),
                ("K_padded", ctypes.c_int), ("N_padded", ctypes.c_int),
                ("device_bytes", ctypes.c_uint64)]


# name -> (restype, argtypes); mirrors include/qlinear.h
_P = ctypes.c_void_p
_I = ctypes.c_int
SIGNATURES = {
    "qlinear_backend_config_init": (None, [ctypes.POINTER(BackendConfig)]),
    "qlinear_backend_create": (_P, [ctypes.POINTER(BackendConfig)]),
    "qlinear_backend_free": (None, [_P]),
    "qlinear_weights_create": (_P, [_P, ctypes.POINTER(WeightConfig), _P, _P]),
    "qlinear_weights_create_shard": (_P, [_P, ctypes.POINTER(WeightConfig), _P, _P, _I, _I]),
    "qlinear_weights_create_checkpoint": (_P, [_P, ctypes.POINTER(WeightConfig), _P, _P]),
    "qlinear_weights_query": (_I, [_P, ctypes.POINTER(WeightInfo)]),
    "qlinear_weights_free": (None, [_P]),
    "qlinear_backend_prepare": (_I, [_P, _I]),
    "qlinear_run_f32": (_I, [_P, _P, _P, _P, _I]),
    "qlinear_run_swiglu_f32": (_I, [_P, _P, _P, _P, _I]),
    "qlinear_run_f32_ex": (_I, [_P, _P, _P, _P, ctypes.c_longlong, _I, ctypes.c_uint]),
    "qlinear_selftest_wait_timeout": (_I, [_P, ctypes.c_ulonglong]),
    "qlinear_run_device_scatter": (_I, [_P, _P, _P, _I, _P, _I, _I, ctypes.c_longlong,
                                        ctypes.c_longlong, _I, ctypes.c_uint, _P]),
    "qlinear_run_device_multicast": (_I, [_P, _P, _P, _I, _P, _I, _P, _I, ctypes.c_longlong,
                                          ctypes.c_longlong, _I, _P]),
    "qlinear_peer_buffer_create": (_I, [_P, ctypes.c_size_t, _P, _P]),
    "qlinear_peer_buffer_open": (_I, [_P, _P, _P]),
    "qlinear_peer_buffer_free": (_I, [_P, _P, _I]),
    "qlinear_peer_signal_wait": (_I, [_P, _P, _I, _I, ctypes.c_ulonglong, ctypes.c_ulonglong, _P]),
    "qlinear_run_device": (_I, [_P, _P, _P, _I, _P, _I, ctypes.c_longlong, _I, ctypes.c_uint, _P]),
    "qlinear_run_mlp_device": (_I, [_P, _P, _P, _P, _I, _P, _I, ctypes.c_longlong, _I, _P]),
    "qlinear_row_amax_device": (_I, [_P, _P, _I, _I, _I, _P, _P]),
    "qlinear_run_device_amax": (_I, [_P, _P, _P, _I, _P, _P, _I, ctypes.c_longlong, _I, _P]),
    "qlinear_dequant_device": (_I, [_P, _P, _P, ctypes.c_longlong, _P, _P, _I, ctypes.c_longlong,
                                    _I, _P]),
    "qlinear_act_quant_device": (_I, [_P, _P, _I, _I, _I, _P, _P, _P, _P]),
    "qlinear_run_device_noalloc": (_I, [_P, _P, _I, _P, _I, ctypes.c_longlong, _I, _P]),
    "qlinear_swiglu_device": (_I, [_P, _P, _I, _I, _P, _I, ctypes.c_longlong, _P]),
    "qlinear_interleave_columns": (_I, [_P, _P, _P, _I, _I, _I, _I, _P]),
    "qlinear_backend_profile": (_I, [_P, _I]),
    "qlinear_backend_profile_collect": (_I, [_P, ctypes.POINTER(ctypes.c_double),
                                             ctypes.POINTER(ctypes.c_double),
                                             ctypes.POINTER(ctypes.c_int)]),
    "qlinear_backend_check": (_I, [_P, _P]),
    "qlinear_backend_stats": (_I, [_P, ctypes.c_char_p, ctypes.c_size_t]),
    "qlinear_backend_launches": (ctypes.c_ulonglong, [_P]),
    "qlinear_strerror": (ctypes.c_char_p, [_I]),
    "qlinear_last_status": (_I, []),
    "qlinear_version": (ctypes.c_char_p, []),
}

_lib = None


def load(path: str | None = None) -> ctypes.CDLL:
    """Load libqlinear_b200.so (once) and declare every C-ABI signature."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or os.environ.get("QLINEAR_LIB", LIB_PATH)
    if not os.path.exists(p):
        raise QLinearUnavailable(
            f"{p} is missing: build it with __graft_entry__.build() or "
            "`make -C open_rknpu2_lm_infer_b200/csrc` (there is no CPU fallback)")
    lib = ctypes.CDLL(p, mode=ctypes.RTLD_GLOBAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def strerror(status: int) -> str:
    return load().qlinear_strerror(status).decode()
