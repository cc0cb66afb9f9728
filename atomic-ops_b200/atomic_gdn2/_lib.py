"""ctypes binding of libgdn2_b200.so (the C ABI declared in include/gdn2_b200.h).

The library is loaded from the package's _lib/ directory (built in-tree by _build.py).  A missing
or unloadable library raises immediately: there is no CPU or framework fallback for the operator.
"""
from __future__ import annotations

import ctypes
import pathlib
import threading

from .precision import ENUM

_LIB_PATH = pathlib.Path(__file__).resolve().parent / "_lib" / "libgdn2_b200.so"
_lock = threading.Lock()
_lib = None

# gdn2_status
OK, ERR_INVALID_ARGUMENT, ERR_CUDA, ERR_UNSUPPORTED = 0, 1, 2, 3
# gdn2_precision
PREC = ENUM
# gdn2_dtype
F32, BF16 = 0, 1
# device status bits
DEV_TIMEOUT, DEV_SPAN, DEV_POSITIVE_GATE = 1, 2, 4


class Gdn2Desc(ctypes.Structure):
    """struct gdn2_desc (include/gdn2_b200.h)."""
    _fields_ = [
        ("B", ctypes.c_int32), ("H", ctypes.c_int32), ("L", ctypes.c_int32), ("D", ctypes.c_int32),
        ("stride_b", ctypes.c_int64), ("stride_h", ctypes.c_int64),
        ("bt", ctypes.c_int32),
        ("scale", ctypes.c_float), ("wy_eps", ctypes.c_float), ("clip", ctypes.c_float),
        ("dot_mode", ctypes.c_int32), ("solve_dot_mode", ctypes.c_int32), ("b3_dot_mode", ctypes.c_int32),
        ("in_dtype", ctypes.c_int32),
    ]


EXPORTS = ("gdn2_residual_bytes", "gdn2_fwd_workspace_bytes", "gdn2_bwd_workspace_bytes", "gdn2_fwd", "gdn2_bwd",
           "gdn2_set_batch_groups", "gdn2_get_batch_groups",
           "gdn2_status_string", "gdn2_selftest_gemm", "gdn2_profile_enable", "gdn2_profile_collect",
           "gdn2_fwd_noalloc", "gdn2_prologue_fwd", "gdn2_prologue_bwd", "gdn2_selftest_engine",
           "gdn2_selftest_wait_timeout")
# kernel ids of gdn2_profile_collect
KERNELS = ("fwd_intra", "fwd_scan", "fwd_out", "bwd_pre", "bwd_scan", "bwd_intra")


def _declare(lib):
    P = ctypes.c_void_p
    lib.gdn2_residual_bytes.restype = ctypes.c_size_t
    lib.gdn2_residual_bytes.argtypes = [ctypes.POINTER(Gdn2Desc)]
    lib.gdn2_fwd_workspace_bytes.restype = ctypes.c_size_t
    lib.gdn2_fwd_workspace_bytes.argtypes = [ctypes.POINTER(Gdn2Desc)]
    lib.gdn2_bwd_workspace_bytes.restype = ctypes.c_size_t
    lib.gdn2_bwd_workspace_bytes.argtypes = [ctypes.POINTER(Gdn2Desc)]
    lib.gdn2_fwd.restype = ctypes.c_int
    lib.gdn2_fwd.argtypes = [ctypes.POINTER(Gdn2Desc)] + [P] * 13
    lib.gdn2_set_batch_groups.restype = ctypes.c_int32
    lib.gdn2_set_batch_groups.argtypes = [ctypes.c_int32]
    lib.gdn2_get_batch_groups.restype = ctypes.c_int32
    lib.gdn2_get_batch_groups.argtypes = []
    lib.gdn2_bwd.restype = ctypes.c_int
    lib.gdn2_bwd.argtypes = [ctypes.POINTER(Gdn2Desc)] + [P] * 20
    lib.gdn2_status_string.restype = ctypes.c_char_p
    lib.gdn2_status_string.argtypes = [ctypes.c_int]
    lib.gdn2_selftest_gemm.restype = ctypes.c_int
    lib.gdn2_selftest_gemm.argtypes = [P, P, P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, P, P]
    lib.gdn2_profile_enable.restype = None
    lib.gdn2_profile_enable.argtypes = [ctypes.c_int32]
    lib.gdn2_profile_collect.restype = ctypes.c_int32
    lib.gdn2_profile_collect.argtypes = [P, P, ctypes.c_int32]
    lib.gdn2_fwd_noalloc.restype = ctypes.c_int
    lib.gdn2_fwd_noalloc.argtypes = [ctypes.POINTER(Gdn2Desc)] + [P] * 11
    lib.gdn2_selftest_engine.restype = ctypes.c_int
    lib.gdn2_selftest_engine.argtypes = [P] * 5 + [ctypes.c_int32] * 3 + [P, P]
    lib.gdn2_selftest_wait_timeout.restype = ctypes.c_int
    lib.gdn2_selftest_wait_timeout.argtypes = [P, ctypes.c_int64, P, P]
    I64 = ctypes.c_int64
    lib.gdn2_prologue_fwd.restype = ctypes.c_int
    lib.gdn2_prologue_fwd.argtypes = [P, I64, I64, I64, I64, ctypes.c_float, ctypes.c_int32] + [P] * 7
    lib.gdn2_prologue_bwd.restype = ctypes.c_int
    lib.gdn2_prologue_bwd.argtypes = [P, I64, I64, I64, I64, ctypes.c_float, ctypes.c_int32] + [P] * 8
    return lib


def set_batch_groups(n: int) -> int:
    """Concurrent batch groups of each gdn2_fwd / gdn2_bwd call (1..8; results do not depend on it).
    Returns the previous value."""
    return int(load().gdn2_set_batch_groups(int(n)))


def batch_groups() -> int:
    return int(load().gdn2_get_batch_groups())


def profile_enable(on: bool) -> None:
    load().gdn2_profile_enable(1 if on else 0)


def profile_collect() -> dict:
    """{kernel: (summed ms, launches)} of the launches timed since the last collect (synchronises)."""
    n = len(KERNELS)
    ms = (ctypes.c_float * n)()
    cnt = (ctypes.c_int32 * n)()
    load().gdn2_profile_collect(ctypes.cast(ms, ctypes.c_void_p), ctypes.cast(cnt, ctypes.c_void_p), n)
    return {k: (float(ms[i]), int(cnt[i])) for i, k in enumerate(KERNELS)}


def lib_path() -> pathlib.Path:
    return _LIB_PATH


def load():
    """Load (once) and return the ctypes handle; raises RuntimeError if the library is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not _LIB_PATH.exists():
                raise RuntimeError(
                    f"{_LIB_PATH} is missing: build it with `python -c \"import __graft_entry__ as g; g.build()\"` "
                    "(nvcc, sm_100a). The GDN-2 operator has no fallback implementation.")
            _lib = _declare(ctypes.CDLL(str(_LIB_PATH)))
    return _lib


def status_string(code: int) -> str:
    return load().gdn2_status_string(int(code)).decode()


def check(code: int, what: str):
    if code == OK:
        return
    msg = f"{what}: {status_string(code)} (status {code})"
    if code == ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    if code == ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)
