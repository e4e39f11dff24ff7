"""ctypes binding of libactcomp.so (the C ABI declared in include/actcomp.h).

The shared library is the only compute path: if it is missing, importing this
module raises, and every op raises ``RuntimeError`` on a non-zero status.  There
is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
#: the in-tree build; ACTCOMP_LIBRARY names another build of the same sources instead
LIB_PATH = os.environ.get("ACTCOMP_LIBRARY") or os.path.join(_HERE, "libactcomp.so")

c_i64 = ctypes.c_int64
c_i32 = ctypes.c_int32
c_vp = ctypes.c_void_p

ABI_VERSION = 2  # ACTCOMP_ABI_VERSION in include/actcomp.h

ACT_OK = 0
ACT_E_INVALID = -1
ACT_E_UNSUPPORTED = -2
ACT_E_ALIGN = -3
ACT_E_CUDA = -4
ACT_E_NODEVICE = -5
ACT_E_WORKSPACE = -6
ACT_E_TIMEOUT = -7
ACT_E_BOUNDS = -8

ACT_OP_DECODE = 0
ACT_OP_MUL = 1
ACT_OP_SILU_BWD = 2
ACT_OP_GELU_BWD = 3

ACT_RC_TWIN_LOWRANK = 1
ACT_RC_HALF_EVEN = 2
ACT_RC_SCALE_BATCH = 4
ACT_RC_ROW_PACK = 8
ACT_RC_OUTLIER_BF16 = 16


class CgDesc(ctypes.Structure):
    _fields_ = [
        ("tokens", c_i64), ("channels", c_i64),
        ("bits", c_i32), ("group", c_i32), ("rank", c_i32), ("n_outlier", c_i32), ("wht", c_i32), ("batch", c_i32),
        ("codes", c_vp), ("scales", c_vp), ("lowrank", c_vp), ("outliers", c_vp), ("outlier_idx", c_vp),
        ("basis_t", c_vp), ("basis", c_vp), ("basis_tile", c_vp),
    ]


class RcArgs(ctypes.Structure):
    _fields_ = [
        ("B", c_i64), ("M", c_i64), ("N", c_i64),
        ("K", c_i32), ("bits", c_i32), ("flags", c_i32), ("outlier", ctypes.c_float),
        ("l", c_vp), ("r", c_vp), ("s", c_vp), ("s_rows", c_i64),
        ("x", c_vp), ("sxb", c_i64), ("sxm", c_i64),
        ("o", c_vp), ("q", c_vp), ("out", c_vp),
    ]


class EwArgs(ctypes.Structure):
    _fields_ = [
        ("B", c_i64), ("M", c_i64), ("N", c_i64),
        ("x", c_vp), ("sxb", c_i64), ("sxm", c_i64),
        ("g", c_vp), ("sgb", c_i64), ("sgm", c_i64),
        ("out", c_vp), ("sob", c_i64), ("som", c_i64),
    ]


class GemmArgs(ctypes.Structure):
    _fields_ = [
        ("M", c_i64), ("N", c_i64), ("K", c_i64),
        ("batch", c_i32), ("in_dtype", c_i32), ("c_dtype", c_i32), ("activation", c_i32),
        ("a_kmajor", c_i32), ("b_kmajor", c_i32),
        ("A", c_vp), ("lda", c_i64), ("sa_batch", c_i64),
        ("B", c_vp), ("ldb", c_i64), ("sb_batch", c_i64),
        ("C", c_vp), ("ldc", c_i64), ("sc_batch", c_i64),
        ("K2", c_i64), ("A2", c_vp), ("lda2", c_i64), ("B2", c_vp), ("ldb2", c_i64),
    ]


#: entry point -> (restype, argtypes); mirrors include/actcomp.h
SIGNATURES = {
    "actcomp_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "actcomp_abi_version": (ctypes.c_int, []),
    "actcomp_last_device_error": (ctypes.c_int, [c_vp, ctypes.POINTER(ctypes.c_uint32)]),
    "actcomp_clear_device_error": (ctypes.c_int, [c_vp]),
    "actcomp_selftest_bounded_wait": (ctypes.c_int, [ctypes.c_uint32, c_i32, c_vp]),
    "actcomp_cg_basis_prepare": (ctypes.c_int, [c_vp, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp, c_vp]),
    "actcomp_cg_encode": (ctypes.c_int, [ctypes.POINTER(CgDesc), c_vp, c_i64, c_vp]),
    "actcomp_cg_decode": (ctypes.c_int, [ctypes.POINTER(CgDesc), c_vp, c_i64, c_vp]),
    "actcomp_cg_consume": (ctypes.c_int, [ctypes.POINTER(CgDesc), c_i32, c_vp, c_i64, c_vp, c_i64, c_vp]),
    "actcomp_cg_softmax_workspace": (ctypes.c_size_t, [ctypes.POINTER(CgDesc)]),
    "actcomp_cg_softmax_bwd": (ctypes.c_int, [ctypes.POINTER(CgDesc), c_vp, c_vp, c_i64, c_i32, c_vp,
                                              ctypes.c_size_t, c_vp]),
    "actcomp_cg_dw_workspace": (ctypes.c_size_t, [ctypes.POINTER(CgDesc), c_i64]),
    "actcomp_cg_dw": (ctypes.c_int, [ctypes.POINTER(CgDesc), c_vp, c_i64, c_i64, c_vp, c_i32, c_i64, c_vp,
                                     ctypes.c_size_t, c_vp]),
    "actcomp_cg_dw_fused_workspace": (ctypes.c_size_t, [ctypes.POINTER(CgDesc), c_i64]),
    "actcomp_cg_dw_fused": (ctypes.c_int, [ctypes.POINTER(CgDesc), c_vp, c_i64, c_i64, c_vp, c_i32, c_i64, c_vp,
                                           ctypes.c_size_t, c_vp]),
    "actcomp_cg_dw_static": (ctypes.c_int, [ctypes.POINTER(CgDesc), c_vp, c_i64, c_i64, c_vp, c_i32, c_i64, c_vp]),
    "actcomp_cg_channel_topk": (ctypes.c_int, [c_vp, c_i64, c_i64, c_i64, c_i32, c_vp, c_vp, c_vp]),
    "actcomp_cg_copy": (ctypes.c_int, [ctypes.POINTER(CgDesc), ctypes.POINTER(CgDesc), c_vp]),
    "actcomp_rc_encode": (ctypes.c_int, [ctypes.POINTER(RcArgs), c_vp]),
    "actcomp_rc_decode": (ctypes.c_int, [ctypes.POINTER(RcArgs), c_i32, c_vp]),
    "actcomp_rc_lowrank_add": (ctypes.c_int, [ctypes.POINTER(RcArgs), c_vp]),
    "actcomp_elementwise": (ctypes.c_int, [ctypes.POINTER(EwArgs), c_i32, c_vp]),
    "actcomp_softmax_bwd": (ctypes.c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp]),
    "actcomp_extract_unstructured": (ctypes.c_int, [c_vp, c_i64, ctypes.c_float, c_vp, c_vp, c_vp]),
    "actcomp_extract_channel": (ctypes.c_int, [c_vp, c_i64, c_i64, c_i64, c_vp, c_i32, c_vp, c_vp]),
    "actcomp_gemm": (ctypes.c_int, [ctypes.POINTER(GemmArgs), c_vp]),
    "actcomp_error_stats": (ctypes.c_int, [c_vp, c_vp, c_i64, c_vp, c_vp]),
    "actcomp_nf4_dequant": (ctypes.c_int, [c_vp, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64,
                                           c_vp, c_vp, c_vp]),
}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load libactcomp.so (building it first only if ACTCOMP_AUTOBUILD=1)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            if os.environ.get("ACTCOMP_AUTOBUILD") == "1":
                from . import build
                build.build()
            else:
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python triton-kernel-test_b200/actcomp/build.py` "
                    "(nvcc, sm_100a). actcomp has no CPU fallback.")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.actcomp_abi_version() != ABI_VERSION:
            raise ImportError(f"{LIB_PATH}: ABI version {lib.actcomp_abi_version()} != {ABI_VERSION}")
        _lib = lib
        return lib


class ActcompError(RuntimeError):
    def __init__(self, fn: str, status: int):
        msg = load().actcomp_strerror(status).decode()
        super().__init__(f"{fn} failed: {msg} ({status})")
        self.status = status


def check(fn: str, status: int) -> None:
    if status != ACT_OK:
        raise ActcompError(fn, status)


def call(name: str, *args) -> None:
    check(name, getattr(load(), name)(*args))
