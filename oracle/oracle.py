"""Python face of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Loads ``oracle/_build/libactcomp_oracle.so`` (built from actcomp_oracle.c by
oracle/Makefile) through ctypes and exposes numpy-in/numpy-out functions.  Only
tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may import
this module; the product code under triton-kernel-test_b200/ never does.

bf16 tensors cross this boundary as ``np.uint16`` arrays holding the raw bits.
Every function cites the reference code it restates; the C file header gives
the exact rounding points.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "libactcomp_oracle.so")
_lock = threading.Lock()
_lib = None

# Flags of the reference-compat restatement (see actcomp_oracle.c).
RC_TWIN_LOWRANK = 1
RC_HALF_EVEN = 2
RC_SCALE_BATCH = 4
RC_ROW_PACK = 8
RC_OUTLIER_BF16 = 16
#: every PyTorch-twin behaviour at once (low_rank_extraction_speed.py:146-156,
#: low_rank_kernel_accuracy_test.py:6-16, ..._decompression_dequantization.py:155-165)
RC_TWIN = RC_TWIN_LOWRANK | RC_HALF_EVEN | RC_SCALE_BATCH | RC_ROW_PACK | RC_OUTLIER_BF16


def build() -> str:
    """Compile the oracle with oracle/Makefile if the shared object is missing or stale."""
    src = os.path.join(_HERE, "actcomp_oracle.c")
    if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            _lib = ctypes.CDLL(_SO)
    return _lib


def _p(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else ctypes.c_void_p(0)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


I64 = ctypes.c_int64
I32 = ctypes.c_int


# ------------------------------------------------------------------ bf16 helpers
def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even binary32 -> bf16 bits (NaN -> 0x7fc0)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FC0
    return r


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ------------------------------------------------------------------ channel-group format
def basis_prepare(V: np.ndarray):
    """V (H x r) float32 -> (Vt bf16 bits r x H, Vq int8 H x r, sV float32 r)."""
    V = _c(V, np.float32)
    H, r = V.shape
    Vt = np.empty((r, H), np.uint16)
    Vq = np.empty((H, r), np.int8)
    sV = np.empty((r,), np.float32)
    lib().cg_basis_prepare(_p(V), I64(H), I32(r), _p(Vt), _p(Vq), _p(sV))
    return Vt, Vq, sV


def project(X: np.ndarray, Vt: np.ndarray) -> np.ndarray:
    """L = X @ Vt^T accumulated in binary64 (X bf16 bits or float32)."""
    x_f32 = X.dtype == np.float32
    X = _c(X, np.float32 if x_f32 else np.uint16)
    T, H = X.shape
    r = Vt.shape[0]
    L = np.empty((T, r), np.float32)
    lib().cg_project(_p(X), I32(int(x_f32)), I64(T), I64(H), I64(H), _p(_c(Vt, np.uint16)), I32(r), _p(L))
    return L


def lr_quantize(L: np.ndarray, sV: np.ndarray):
    L = _c(L, np.float32)
    T, r = L.shape
    Lq = np.empty((T, r), np.int8)
    sL = np.empty((T,), np.float32)
    lib().cg_lr_quantize(_p(L), I64(T), I32(r), _p(_c(sV, np.float32)), _p(Lq), _p(sL))
    return Lq, sL


def encode_given_lr(X, Lq, sL, Vq, idx, bits, group, wht):
    """Channel-group encode of X given its low-rank codes -> (codes, scales, outliers)."""
    x_f32 = X.dtype == np.float32
    X = _c(X, np.float32 if x_f32 else np.uint16)
    T, H = X.shape
    r = 0 if Lq is None else Lq.shape[1]
    idx = _c(idx if idx is not None else np.zeros(0), np.int32)
    k = idx.shape[0]
    codes = np.empty((T, H * bits // 8), np.uint8)
    scales = np.empty((T, H // group), np.float32)
    outl = np.empty((T, k), np.float32 if x_f32 else np.uint16)
    Lq_ = _c(Lq, np.int8) if r else np.zeros((T, 1), np.int8)
    sL_ = _c(sL, np.float32) if r else np.zeros((T,), np.float32)
    Vq_ = _c(Vq, np.int8) if r else np.zeros((H, 1), np.int8)
    lib().cg_encode_given_lr(_p(X), I32(int(x_f32)), I64(T), I64(H), I64(H), _p(Lq_), _p(sL_), _p(Vq_), I32(r),
                             _p(idx), I32(k), I32(bits), I32(group), I32(int(wht)), _p(codes), _p(scales), _p(outl))
    return codes, scales, outl


def encode(X, V_prepared, idx, bits, group, wht):
    """Full channel-group encode: projection (binary64), low-rank codes, residual codes."""
    Vt, Vq, sV = V_prepared
    if Vt.shape[0]:
        L = project(X, Vt)
        Lq, sL = lr_quantize(L, sV)
    else:
        Lq = sL = None
    codes, scales, outl = encode_given_lr(X, Lq, sL, Vq, idx, bits, group, wht)
    return dict(codes=codes, scales=scales, outliers=outl, lr_codes=Lq, lr_scale=sL)


def decode(codes, scales, Lq, sL, Vq, outl, idx, H, bits, group, wht, x_f32=False):
    T = codes.shape[0]
    r = 0 if Lq is None else Lq.shape[1]
    idx = _c(idx if idx is not None else np.zeros(0), np.int32)
    k = idx.shape[0]
    out = np.empty((T, H), np.float32 if x_f32 else np.uint16)
    Lq_ = _c(Lq, np.int8) if r else np.zeros((T, 1), np.int8)
    sL_ = _c(sL, np.float32) if r else np.zeros((T,), np.float32)
    Vq_ = _c(Vq, np.int8) if r else np.zeros((H, 1), np.int8)
    outl_ = _c(outl, np.float32 if x_f32 else np.uint16) if k else np.zeros((T, 1), np.uint16)
    lib().cg_decode(_p(_c(codes, np.uint8)), _p(_c(scales, np.float32)), _p(Lq_), _p(sL_), _p(Vq_), I32(r),
                    _p(outl_), _p(idx), I32(k), I64(T), I64(H), I32(bits), I32(group), I32(int(wht)),
                    I32(int(x_f32)), _p(out))
    return out


def channel_absmax(X):
    X = _c(X, np.uint16)
    T, H = X.shape
    s = np.empty((H,), np.float32)
    lib().cg_channel_absmax(_p(X), I64(T), I64(H), I64(H), _p(s))
    return s


def topk_channels(score, k):
    score = _c(score, np.float32)
    idx = np.empty((k,), np.int32)
    lib().cg_topk_channels(_p(score), I64(score.shape[0]), I32(k), _p(idx))
    return idx


# ------------------------------------------------------------------ consumers
def _unary2(name, x, g):
    x = _c(x, np.uint16)
    g = _c(g, np.uint16)
    out = np.empty_like(x)
    getattr(lib(), name)(_p(x), _p(g), I64(x.size), _p(out))
    return out


def silu_bwd(x, g):
    """silu_backward.py:6-8, binary32 math, one bf16 rounding."""
    return _unary2("orc_silu_bwd", x, g)


def gelu_bwd(x, g):
    """gelu_backward.py:14-21 (tanh approximation), binary32 math."""
    return _unary2("orc_gelu_bwd", x, g)


def mul(a, b):
    """extraction_fuse_hadamard.py:5 elementwise product."""
    return _unary2("orc_mul", a, b)


def softmax_bwd(y, g):
    """softmax_backward.py:6 over the last axis."""
    y = _c(y, np.uint16)
    g = _c(g, np.uint16)
    n = y.shape[-1]
    out = np.empty_like(y)
    lib().orc_softmax_bwd(_p(y), _p(g), I64(y.size // n), I64(n), _p(out))
    return out


def gemm_tn(A, B):
    """C = A^T B, A (K x M) and B (K x N) bf16 bits, binary64 accumulation."""
    A = _c(A, np.uint16)
    B = _c(B, np.uint16)
    K, M = A.shape
    N = B.shape[1]
    C = np.empty((M, N), np.float32)
    lib().orc_gemm_tn(_p(A), _p(B), I64(M), I64(N), I64(K), _p(C))
    return C


# ------------------------------------------------------------------ reference-compat
def rc_encode(l, r, x, s, bits, outlier, flags=0):
    """low_rank_addition_fuse_compression_quantization restated (see C header).

    x (B,M,N) bf16 bits, l (M,K), r (K,N), s (S,N).  Returns (o dense bf16 bits,
    q packed uint8, signed codes int32)."""
    x = _c(x, np.uint16)
    B, M, N = x.shape
    K = l.shape[1]
    s = _c(s, np.uint16).reshape(-1, N)
    o = np.empty((B, M, N), np.uint16)
    q = np.empty((B, M, N * bits // 8), np.uint8)
    sc = np.empty((B, M, N), np.int32)
    lib().rc_encode(_p(_c(l, np.uint16)), _p(_c(r, np.uint16)), _p(x), I64(M * N), I64(N), _p(s), I64(s.shape[0]),
                    I64(B), I64(M), I64(N), I32(K), I32(bits), ctypes.c_float(outlier), I32(flags), _p(o), _p(q),
                    _p(sc))
    return o, q, sc


def rc_decode(l, r, q, o, s, bits, flags=0):
    """low_rank_addition_fuse_decompression_dequantization restated; o may be None."""
    q = _c(q, np.uint8)
    B, M, W = q.shape
    N = W * 8 // bits
    K = l.shape[1]
    s = _c(s, np.uint16).reshape(-1, N)
    x = np.empty((B, M, N), np.uint16)
    lib().rc_decode(_p(_c(l, np.uint16)), _p(_c(r, np.uint16)), _p(q), _p(None if o is None else _c(o, np.uint16)),
                    _p(s), I64(s.shape[0]), I64(B), I64(M), I64(N), I32(K), I32(bits), I32(flags), _p(x))
    return x


# ------------------------------------------------------------------ metrics
def rel_fro(a, b) -> float:
    """||a - b||_F / ||b||_F in binary64 (a, b float arrays or bf16 bits)."""
    a = bf16_to_f32(a) if a.dtype == np.uint16 else a
    b = bf16_to_f32(b) if b.dtype == np.uint16 else b
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


def unpack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """Channel-group format codes (T x H*bits/8) -> unsigned codes (T x H)."""
    if bits == 8:
        return codes.copy()
    lo = codes & 0xF
    hi = codes >> 4
    return np.stack([lo, hi], axis=-1).reshape(codes.shape[0], -1)
