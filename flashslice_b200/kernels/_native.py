"""ctypes binding of the C ABI in ``include/flashslice_b200.h``.

The native library is the only implementation of the ops: there is no
CPU or eager fallback. If the library is missing the first op call raises
with the build command; building it needs ``nvcc`` only (no GPU).
"""

import ctypes
import os
import threading

import torch

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBPATH = os.path.join(_PKG, "_native", "libflashslice_b200.so")

ABI_VERSION = 2

FS_OK, FS_ERR_SHAPE, FS_ERR_ARGUMENT, FS_ERR_WORKSPACE, FS_ERR_CUDA, FS_ERR_TIMEOUT, \
    FS_ERR_UNSUPPORTED = range(7)
OP_SLICE_FWD, OP_DESLICE_FWD, OP_SLICE_BWD, OP_DESLICE_BWD, OP_STATS = range(5)
FAMILY_SINGLE, FAMILY_BLOCKED = 0, 1
FLAG_STATS_IN, FLAG_STATS_OUT = 1, 2

DTYPE_CODE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

# Every entry point the header declares, with its ctypes signature.
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32


class Problem(ctypes.Structure):
    _fields_ = [("B", _I64), ("N", _I64), ("H", _I64), ("D", _I64), ("DV", _I64), ("G", _I64),
                ("act_dtype", _I32), ("dot", _I32), ("family", _I32), ("stats_mode", _I32),
                ("w_batch", _I32), ("w_heads", _I32), ("b_batch", _I32), ("b_heads", _I32),
                ("flags", _I32), ("engine", _I32), ("row_splits", _P)]


class Tensor4(ctypes.Structure):
    _fields_ = [("data", _P), ("stride", _I64 * 4)]


_PP = ctypes.POINTER(Problem)
_PT = ctypes.POINTER(Tensor4)

SIGNATURES = {
    "fs_version": (ctypes.c_int, []),
    "fs_last_error": (ctypes.c_char_p, []),
    "fs_launch_count": (ctypes.c_uint64, []),
    "fs_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int, _PP]),
    "fs_slice_fwd": (ctypes.c_int, [_PP, _PT, _PT, _P, _P, _P, _P, _P, _P, _P, _P,
                                    ctypes.c_size_t, _P]),
    "fs_deslice_fwd": (ctypes.c_int, [_PP, _PT, _P, _P, _P, _P, _P, _P, _PT, _P,
                                      ctypes.c_size_t, _P]),
    "fs_slice_bwd": (ctypes.c_int, [_PP, _PT, _PT, _P, _P, _P, _P, _P, _P, _PT, _PT, _P, _P,
                                    _P, _P, ctypes.c_size_t, _P]),
    "fs_deslice_bwd": (ctypes.c_int, [_PP, _PT, _P, _P, _P, _P, _P, _PT, _PT, _P, _P, _P, _P,
                                      _P, ctypes.c_size_t, _P]),
    "fs_compute_stats": (ctypes.c_int, [_PP, _PT, _P, _P, _P, _P, _P]),
    "fs_slice_fwd_noalloc": (ctypes.c_int, [_PP, _PT, _PT, _P, _P, _P, _P, _P, _P]),
    "fs_device_status": (ctypes.c_int, [ctypes.c_int]),
    "fs_tc_launch_count": (ctypes.c_uint64, []),
    "fs_coupled_bwd": (ctypes.c_int, [_PP, _PT, _PT, _PT, _P, _P, _P, _P, _P, _P, _PT, _PT, _P,
                                      _P, _P, _P, ctypes.c_size_t, _P]),
    "fs_coupled_supported": (ctypes.c_int, [_PP]),
    "fs_rank_sum": (ctypes.c_int, [_P, _P, ctypes.c_int, ctypes.c_int64, _P]),
    "fs_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_uint64, _P]),
    "fs_set_wait_limit_ns": (ctypes.c_int, [ctypes.c_uint64]),
}

ENGINE_AUTO, ENGINE_FMA = 0, 1
ENGINES = {"auto": ENGINE_AUTO, "fma": ENGINE_FMA}

_lib = None
_lock = threading.Lock()


class NativeLibraryMissing(RuntimeError):
    pass


def load():
    """The loaded library (raises NativeLibraryMissing when it is not built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIBPATH):
                raise NativeLibraryMissing(
                    "flashslice_b200 native library not found at %s; build it with "
                    "`python -m flashslice_b200.build` (needs nvcc)" % LIBPATH)
            lib = ctypes.CDLL(LIBPATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            if lib.fs_version() != ABI_VERSION:
                raise NativeLibraryMissing("native library ABI %d, expected %d"
                                           % (lib.fs_version(), ABI_VERSION))
            _lib = lib
    return _lib


def check(rc):
    if rc == FS_OK:
        return
    msg = load().fs_last_error().decode(errors="replace")
    if rc in (FS_ERR_SHAPE, FS_ERR_ARGUMENT, FS_ERR_UNSUPPORTED):
        raise ValueError("flashslice_b200: " + msg)
    raise RuntimeError("flashslice_b200 (status %d): %s" % (rc, msg))


def t4(t):
    """A (B, N, H, width) tensor as the ABI's strided view."""
    if t is None:
        return None
    s = (_I64 * 4)(*t.stride())
    return ctypes.pointer(Tensor4(ctypes.c_void_p(t.data_ptr()), s))


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def workspace(op, prob, device):
    n = load().fs_workspace_bytes(op, ctypes.byref(prob))
    if n == 0:
        return None, 0
    return torch.empty(n, dtype=torch.uint8, device=device), n
